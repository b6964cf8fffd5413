"""Oracle for the fused passes around a Swin block's window attention (numpy).

TEST INFRASTRUCTURE ONLY (see oracle/__init__.py).  Restates, in float64, the
glue of the reference's patched ``SwinTransformerBlock.forward_part1``
(torch-ext/crumpet/monai_patch.py:72-114) and the residual add of the Swin
block around it:

* norm_shift_partition -- ``self.norm1(x)`` (LayerNorm over C, biased variance,
  affine), ``F.pad`` of D/H/W at the far end up to a window multiple
  (monai_patch.py:79-89), then ``fused_shift_partition_3d`` (:97).
* unshift_unpartition_crop -- ``fused_unshift_unpartition_3d`` on the padded
  grid (:99-108), the crop ``x[:, :d, :h, :w]`` (:110-111) and, optionally,
  the block's ``shortcut + x``.
* window_geometry -- the clamp rule the patch takes from MONAI's
  ``get_window_size`` (:81): an axis no longer than its window uses the axis
  length as window and no shift.
"""

from __future__ import annotations

import numpy as np

from . import mechanics


def window_geometry(dims, window_size, shift_size):
    ws = list(int(v) for v in window_size)
    ss = list(int(v) for v in shift_size)
    for a in range(3):
        if dims[a] <= ws[a]:
            ws[a] = int(dims[a])
            ss[a] = 0
    return tuple(ws), tuple(ss)


def padded_dims(dims, ws):
    return tuple(-(-int(d) // int(w)) * int(w) for d, w in zip(dims, ws))


def layer_norm(x: np.ndarray, weight: np.ndarray, bias: np.ndarray, eps: float) -> np.ndarray:
    """LayerNorm over the last axis in float64 (biased variance, as torch)."""
    x = x.astype(np.float64)
    mean = x.mean(axis=-1, keepdims=True)
    var = ((x - mean) ** 2).mean(axis=-1, keepdims=True)
    return (x - mean) / np.sqrt(var + eps) * weight.astype(np.float64) + bias.astype(np.float64)


def norm_shift_partition(x: np.ndarray, weight, bias, eps, ws, ss) -> np.ndarray:
    """x [B, D, H, W, C] -> float64 windows [B * nW_padded, N, C]."""
    B, D, H, W, C = x.shape
    y = layer_norm(x, weight, bias, eps)
    Dp, Hp, Wp = padded_dims((D, H, W), ws)
    padded = np.zeros((B, Dp, Hp, Wp, C), dtype=np.float64)
    padded[:, :D, :H, :W] = y
    return mechanics.shift_partition(padded, ws, ss)


def unshift_unpartition_crop(windows: np.ndarray, B, D, H, W, C, ws, ss,
                             residual: np.ndarray | None = None) -> np.ndarray:
    """windows on the padded grid -> [B, D, H, W, C] (+ residual, added in float32
    and cast back for half types, as torch's elementwise add)."""
    Dp, Hp, Wp = padded_dims((D, H, W), ws)
    full = mechanics.unshift_unpartition(windows, B, Dp, Hp, Wp, C, ws, ss)
    out = np.ascontiguousarray(full[:, :D, :H, :W])
    if residual is None:
        return out
    return (residual.astype(np.float32) + out.astype(np.float32)).astype(out.dtype)
