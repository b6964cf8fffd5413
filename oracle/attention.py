"""Oracle for the fused window attention (numpy, float64 math).

TEST INFRASTRUCTURE ONLY (see oracle/__init__.py).  Restates the function
computed by the reference Triton kernel torch-ext/crumpet/fused_attention.py:48-146
and by MONAI's eager WindowAttention chain that torch-ext/crumpet/monai_patch.py:117-198
replaces:

    out[b, h] = softmax(q[b, h] k[b, h]^T * scale + bias[h] + mask[b % nW]) v[b, h]

The mask is applied only to windows whose boundary flag is non-zero
(fused_attention.py:123-129); every window when no flag vector is given.
Inputs are taken at their stored precision (fp16/bf16 values widened
exactly); the arithmetic is float64, so the oracle is the exact answer the
fp32-accumulating kernels approximate.

Also restates MONAI's relative-position index for a 3D window
(the coordinate-difference formula that torch-ext/crumpet/monai_patch.py:160
slices with ``[:n, :n]``).
"""

from __future__ import annotations

import numpy as np


def window_attention(q, k, v, bias, mask=None, boundary=None, scale=None):
    """q, k, v: [B, H, N, D]; bias: [H, N, N]; mask: [nW, N, N] or None."""
    q = np.asarray(q, dtype=np.float64)
    k = np.asarray(k, dtype=np.float64)
    v = np.asarray(v, dtype=np.float64)
    B, H, N, D = q.shape
    if scale is None:
        scale = 1.0 / np.sqrt(D)
    s = np.einsum("bhnd,bhmd->bhnm", q, k) * scale + np.asarray(bias, np.float64)[None]
    if mask is not None:
        m = np.asarray(mask, dtype=np.float64)
        per_window = m[np.arange(B) % m.shape[0]]
        if boundary is not None:
            keep = (np.asarray(boundary).reshape(B) != 0).astype(np.float64)
            per_window = per_window * keep[:, None, None]
        s = s + per_window[:, None]
    s = s - s.max(axis=-1, keepdims=True)
    p = np.exp(s)
    p = p / p.sum(axis=-1, keepdims=True)
    return np.einsum("bhnm,bhmd->bhnd", p, v)


def relative_position_index(window_size) -> np.ndarray:
    """[N, N] index into a ((2wd-1)(2wh-1)(2ww-1), H) relative-position bias table."""
    wd, wh, ww = (int(x) for x in window_size)
    coords = np.stack(
        np.meshgrid(np.arange(wd), np.arange(wh), np.arange(ww), indexing="ij")
    ).reshape(3, -1)
    rel = coords[:, :, None] - coords[:, None, :]
    rel = rel + np.array([wd - 1, wh - 1, ww - 1])[:, None, None]
    return rel[0] * (2 * wh - 1) * (2 * ww - 1) + rel[1] * (2 * ww - 1) + rel[2]


def gather_bias(table, index, n) -> np.ndarray:
    """bias[h, i, j] = table[index[i, j], h] for i, j < n (monai_patch.py:160-162)."""
    idx = np.asarray(index)[:n, :n]
    return np.transpose(np.asarray(table)[idx.reshape(-1)].reshape(n, n, -1), (2, 0, 1))
