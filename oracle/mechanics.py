"""Oracle for the shifted-window mechanics (numpy, integer index arithmetic).

TEST INFRASTRUCTURE ONLY (see oracle/__init__.py).  Each function builds the
explicit source-index map of the operation and gathers with it, which is an
independent formulation of the reference's roll + view/permute code:

* shift_partition   -- reference torch-ext/crumpet/reference.py:141-160
  (torch.roll by -shift, then window_partition_reference :101-118).
* unshift_unpartition -- reference.py:163-184 (window_reverse_reference
  :121-138, then torch.roll by +shift).
* attn_mask         -- reference.py:50-98 (27-region labels, -100 where the
  labels of two tokens of a window differ), cuda/attn_mask_3d.cu:42-50.
"""

from __future__ import annotations

import numpy as np


def _check(D, H, W, ws, ss):
    if min(ws) <= 0 or D % ws[0] or H % ws[1] or W % ws[2]:
        raise ValueError("D, H and W must be divisible by window_size")
    for a in range(3):
        if not 0 <= ss[a] < ws[a]:
            raise ValueError(f"shift_size[{a}] must satisfy 0 <= shift < window_size[{a}]")


def window_source_index(D, H, W, ws, ss):
    """For every (window, token) of one batch entry, the flat source voxel index.

    Window order (wd, wh, ww) row-major, token order (ld, lh, lw) row-major;
    the token reads voxel ((wd*ws_d + ld + ss_d) % D, ..., ...).
    Returns int64 [nW, N].
    """
    ws = tuple(int(v) for v in ws)
    ss = tuple(int(v) for v in ss)
    _check(D, H, W, ws, ss)
    nwd, nwh, nww = D // ws[0], H // ws[1], W // ws[2]
    wd, wh, ww = np.meshgrid(np.arange(nwd), np.arange(nwh), np.arange(nww), indexing="ij")
    ld, lh, lw = np.meshgrid(np.arange(ws[0]), np.arange(ws[1]), np.arange(ws[2]), indexing="ij")
    win = [a.reshape(-1, 1) for a in (wd, wh, ww)]
    loc = [a.reshape(1, -1) for a in (ld, lh, lw)]
    d = (win[0] * ws[0] + loc[0] + ss[0]) % D
    h = (win[1] * ws[1] + loc[1] + ss[1]) % H
    w = (win[2] * ws[2] + loc[2] + ss[2]) % W
    return ((d * H + h) * W + w).astype(np.int64)


def shift_partition(x: np.ndarray, ws, ss) -> np.ndarray:
    """x [B, D, H, W, C] -> [B * nW, N, C]."""
    B, D, H, W, C = x.shape
    idx = window_source_index(D, H, W, ws, ss)
    flat = x.reshape(B, D * H * W, C)
    return flat[:, idx, :].reshape(B * idx.shape[0], idx.shape[1], C)


def unshift_unpartition(windows: np.ndarray, B, D, H, W, C, ws, ss) -> np.ndarray:
    """windows [B * nW, N, C] -> [B, D, H, W, C] (inverse of shift_partition)."""
    idx = window_source_index(D, H, W, ws, ss)
    nw, n = idx.shape
    if windows.shape != (B * nw, n, C):
        raise ValueError(f"windows must have shape {(B * nw, n, C)}")
    out = np.empty((B, D * H * W, C), dtype=windows.dtype)
    out[:, idx.reshape(-1), :] = windows.reshape(B, nw * n, C)
    return out.reshape(B, D, H, W, C)


def region_labels(D, H, W, ws, ss) -> np.ndarray:
    """Per-voxel roll region label 9*r(d) + 3*r(h) + r(w), int64 [D, H, W]."""

    def r(size, w, s):
        x = np.arange(size)
        return np.where(x < size - w, 0, np.where(x < size - s, 1, 2))

    return (
        9 * r(D, ws[0], ss[0])[:, None, None]
        + 3 * r(H, ws[1], ss[1])[None, :, None]
        + r(W, ws[2], ss[2])[None, None, :]
    )


def attn_mask(D, H, W, ws, ss, dtype=np.float32) -> np.ndarray:
    """Shifted-window mask [nW, N, N]: -100 where labels differ, else 0."""
    ws = tuple(int(v) for v in ws)
    ss = tuple(int(v) for v in ss)
    _check(D, H, W, ws, ss)
    # Labels are gathered without the roll (the mask is defined on the rolled
    # grid directly): window (wd, ...) token (ld, ...) sits at wd*ws_d + ld.
    idx = window_source_index(D, H, W, ws, (0, 0, 0))
    lab = region_labels(D, H, W, ws, ss).reshape(-1)[idx]
    if not any(ss):
        lab = np.zeros_like(lab)
    diff = lab[:, :, None] != lab[:, None, :]
    return np.where(diff, np.asarray(-100.0, dtype=dtype), np.asarray(0.0, dtype=dtype))
