"""Fused memory passes around a Swin block's window attention.

The reference's patched ``forward_part1`` (torch-ext/crumpet/monai_patch.py:72-114)
runs norm1, ``F.pad``, the roll + partition op, (autocast's fp16 cast for the
qkv Linear), the attention, the unpartition op and the crop as separate passes,
and MONAI's block adds the residual in one more.  Two ops replace the passes
on either side of the attention:

* :func:`norm_shift_partition_3d` -- LayerNorm + zero pad to a window multiple
  + roll by ``-shift`` + window partition, written in the dtype the qkv Linear
  consumes;
* :func:`unshift_unpartition_crop_3d` -- window reverse on the padded grid +
  roll by ``+shift`` + crop, optionally adding the block's residual;
* :func:`unshift_unpartition_crop_norm_3d` -- the same plus the LayerNorm of the
  result (the block's ``norm2``, which opens its MLP half);
* :func:`patch_merge_norm_3d` -- the 2x2x2 neighbour concatenation of a stage's
  patch merging and its LayerNorm (the reduction Linear follows as a GEMM);
* :func:`proj_out_norm_3d` -- the Swin trunk's hidden-state normalisation
  (MONAI ``SwinTransformer.proj_out``): LayerNorm over the channels of a
  channels-first stage output, stored channels-last.

All are inference ops (no backward): they raise when autograd would need a
gradient through them.  The MONAI patch uses them only outside autograd.
"""

from __future__ import annotations

from typing import Sequence

import torch

from . import _ops as _native
from . import profiling as _prof


def _triple(name: str, value: Sequence[int]) -> tuple[int, int, int]:
    if len(value) != 3:
        raise ValueError(f"{name} must contain exactly three values")
    return tuple(int(v) for v in value)  # type: ignore[return-value]


def _check_window(window_size, shift_size) -> None:
    if any(v <= 0 for v in window_size):
        raise ValueError("window_size values must be positive")
    for axis, (shift, window) in enumerate(zip(shift_size, window_size)):
        if shift < 0 or shift >= window:
            raise ValueError(f"shift_size[{axis}] must satisfy 0 <= shift < window_size[{axis}]")


def _check_dtype(dtype: torch.dtype) -> None:
    if dtype not in (torch.float32, torch.float16, torch.bfloat16):
        raise TypeError("CRUMPET supports torch.float32, torch.float16 and torch.bfloat16")


def padded_geometry(D: int, H: int, W: int, window_size) -> tuple[tuple[int, int, int], int, int]:
    """(padded dims, number of windows, window volume) for a window-multiple padding."""
    dims = tuple(-(-d // w) * w for d, w in zip((D, H, W), window_size))
    num_windows = (dims[0] // window_size[0]) * (dims[1] // window_size[1]) * (dims[2] // window_size[2])
    volume = window_size[0] * window_size[1] * window_size[2]
    return dims, num_windows, volume  # type: ignore[return-value]


def _nbytes(t: torch.Tensor) -> int:
    return t.numel() * t.element_size()


def _aligned(t: torch.Tensor, nbytes: int) -> torch.Tensor:
    t = t.contiguous()
    return t if t.data_ptr() % nbytes == 0 else t.clone()


def norm_shift_partition_3d(
    x: torch.Tensor,
    weight: torch.Tensor,
    bias: torch.Tensor,
    eps: float,
    window_size: Sequence[int],
    shift_size: Sequence[int],
    out_dtype: torch.dtype | None = None,
) -> torch.Tensor:
    """``partition(roll(pad(layer_norm(x)), -shift))`` in one pass.

    ``x`` is ``[B, D, H, W, C]`` with any D/H/W; the volume is zero-padded at
    the far end of each axis up to a multiple of the window (padding after the
    norm, so padded tokens are exact zeros) and the result is
    ``[B * num_windows, volume, C]`` in ``out_dtype`` (default ``x.dtype``).
    The norm is computed in fp32 with a biased variance, as ``nn.LayerNorm``;
    C must be a multiple of 8 and at most 768.
    """
    if x.ndim != 5:
        raise ValueError("x must have shape [B, D, H, W, C]")
    window_size = _triple("window_size", window_size)
    shift_size = _triple("shift_size", shift_size)
    _check_window(window_size, shift_size)
    _check_dtype(x.dtype)
    out_dtype = x.dtype if out_dtype is None else out_dtype
    _check_dtype(out_dtype)
    B, D, H, W, C = (int(v) for v in x.shape)
    if C % 8 or C > 768 or C == 0:
        raise ValueError("norm_shift_partition_3d needs C a multiple of 8 and at most 768")
    if tuple(weight.shape) != (C,) or tuple(bias.shape) != (C,):
        raise ValueError("weight and bias must have shape [C]")
    _, num_windows, volume = padded_geometry(D, H, W, window_size)
    shape = (B * num_windows, volume, C)
    if x.device.type == "meta":
        return torch.empty(shape, dtype=out_dtype, device=x.device)
    if x.device.type != "cuda":
        raise RuntimeError("crumpet_b200 runs norm_shift_partition_3d on CUDA devices only "
                           f"(got {x.device})")
    if torch.is_grad_enabled() and (x.requires_grad or weight.requires_grad or bias.requires_grad):
        raise RuntimeError("norm_shift_partition_3d has no backward; call it under torch.no_grad()")
    out = torch.empty(shape, dtype=out_dtype, device=x.device)
    w = _aligned(weight.detach().to(device=x.device, dtype=torch.float32), 16)
    b = _aligned(bias.detach().to(device=x.device, dtype=torch.float32), 16)
    token = _prof.kernel_begin("norm_shift_partition_3d",
                               lambda: {"bytes": _nbytes(x) + _nbytes(out)})
    _native.require().norm_shift_partition_3d(out, _aligned(x, 16), w, b, float(eps),
                                              *window_size, *shift_size)
    _prof.count("norm_shift_partition_3d")
    _prof.kernel_end(token)
    return out


def unshift_unpartition_crop_3d(
    windows: torch.Tensor,
    B: int,
    D: int,
    H: int,
    W: int,
    C: int,
    window_size: Sequence[int],
    shift_size: Sequence[int],
    residual: torch.Tensor | None = None,
) -> torch.Tensor:
    """``roll(unpartition(windows), +shift)[:, :D, :H, :W]`` (``+ residual``) in one pass.

    ``windows`` is ``[B * num_windows, volume, C]`` on the grid padded to window
    multiples; the result is ``[B, D, H, W, C]``.  ``residual``, when given,
    has that shape and the dtype of ``windows`` and is added in fp32 with one
    rounding (torch's elementwise add).  Rows of C elements must be a multiple
    of 4 bytes.
    """
    if windows.ndim != 3:
        raise ValueError("windows must have shape [B * num_windows, window_volume, C]")
    window_size = _triple("window_size", window_size)
    shift_size = _triple("shift_size", shift_size)
    _check_window(window_size, shift_size)
    _check_dtype(windows.dtype)
    B, D, H, W, C = int(B), int(D), int(H), int(W), int(C)
    if min(D, H, W) <= 0 or B < 0 or C < 0:
        raise ValueError("D, H and W must be positive")
    _, num_windows, volume = padded_geometry(D, H, W, window_size)
    expected = (B * num_windows, volume, C)
    if tuple(int(v) for v in windows.shape) != expected:
        raise ValueError(f"windows must have shape {expected}")
    if (C * windows.element_size()) % 4:
        raise ValueError("unshift_unpartition_crop_3d needs rows of C elements to be a multiple of 4 bytes")
    if residual is not None:
        if tuple(residual.shape) != (B, D, H, W, C):
            raise ValueError(f"residual must have shape {(B, D, H, W, C)}")
        if residual.dtype != windows.dtype:
            raise TypeError("residual must have the dtype of windows")
    if windows.device.type == "meta":
        return torch.empty((B, D, H, W, C), dtype=windows.dtype, device=windows.device)
    if windows.device.type != "cuda":
        raise RuntimeError("crumpet_b200 runs unshift_unpartition_crop_3d on CUDA devices only "
                           f"(got {windows.device})")
    if torch.is_grad_enabled() and (windows.requires_grad or
                                    (residual is not None and residual.requires_grad)):
        raise RuntimeError("unshift_unpartition_crop_3d has no backward; call it under torch.no_grad()")
    out = torch.empty((B, D, H, W, C), dtype=windows.dtype, device=windows.device)
    res = None if residual is None else _aligned(residual, 16)
    # algorithmic bytes: the windows of the cropped volume, the residual, the output
    token = _prof.kernel_begin("unshift_unpartition_crop_3d",
                               lambda: {"bytes": _nbytes(out) * (3 if res is not None else 2)})
    _native.require().unshift_unpartition_crop_3d(out, _aligned(windows, 16), res, B, D, H, W, C,
                                                  *window_size, *shift_size)
    _prof.count("unshift_unpartition_crop_3d")
    _prof.kernel_end(token)
    return out


def unshift_unpartition_crop_norm_3d(
    windows: torch.Tensor,
    B: int,
    D: int,
    H: int,
    W: int,
    C: int,
    window_size: Sequence[int],
    shift_size: Sequence[int],
    weight: torch.Tensor,
    bias: torch.Tensor,
    eps: float,
    residual: torch.Tensor | None = None,
    norm_dtype: torch.dtype | None = None,
) -> tuple[torch.Tensor, torch.Tensor]:
    """:func:`unshift_unpartition_crop_3d` and the LayerNorm of its result in one pass.

    Returns ``(out, normed)``: ``out`` as :func:`unshift_unpartition_crop_3d`
    (dtype of ``windows``), ``normed = layer_norm(out, weight, bias, eps)`` over C
    in fp32 arithmetic, written in ``norm_dtype`` (default: the dtype of
    ``windows``).  In a Swin block this is the residual add of the attention half
    and the ``norm2`` that opens the MLP half.  C must be a multiple of 8, at most
    768.
    """
    if windows.ndim != 3:
        raise ValueError("windows must have shape [B * num_windows, window_volume, C]")
    window_size = _triple("window_size", window_size)
    shift_size = _triple("shift_size", shift_size)
    _check_window(window_size, shift_size)
    _check_dtype(windows.dtype)
    norm_dtype = windows.dtype if norm_dtype is None else norm_dtype
    _check_dtype(norm_dtype)
    B, D, H, W, C = int(B), int(D), int(H), int(W), int(C)
    if min(D, H, W) <= 0 or B < 0:
        raise ValueError("D, H and W must be positive")
    if C % 8 or C > 768 or C == 0:
        raise ValueError("unshift_unpartition_crop_norm_3d needs C a multiple of 8 and at most 768")
    if tuple(weight.shape) != (C,) or tuple(bias.shape) != (C,):
        raise ValueError("weight and bias must have shape [C]")
    _, num_windows, volume = padded_geometry(D, H, W, window_size)
    expected = (B * num_windows, volume, C)
    if tuple(int(v) for v in windows.shape) != expected:
        raise ValueError(f"windows must have shape {expected}")
    if residual is not None:
        if tuple(residual.shape) != (B, D, H, W, C):
            raise ValueError(f"residual must have shape {(B, D, H, W, C)}")
        if residual.dtype != windows.dtype:
            raise TypeError("residual must have the dtype of windows")
    shape = (B, D, H, W, C)
    if windows.device.type == "meta":
        return (torch.empty(shape, dtype=windows.dtype, device=windows.device),
                torch.empty(shape, dtype=norm_dtype, device=windows.device))
    if windows.device.type != "cuda":
        raise RuntimeError("crumpet_b200 runs unshift_unpartition_crop_norm_3d on CUDA devices only "
                           f"(got {windows.device})")
    if torch.is_grad_enabled() and any(t is not None and t.requires_grad
                                       for t in (windows, residual, weight, bias)):
        raise RuntimeError("unshift_unpartition_crop_norm_3d has no backward; call it under "
                           "torch.no_grad()")
    out = torch.empty(shape, dtype=windows.dtype, device=windows.device)
    normed = torch.empty(shape, dtype=norm_dtype, device=windows.device)
    w = _aligned(weight.detach().to(device=windows.device, dtype=torch.float32), 16)
    b = _aligned(bias.detach().to(device=windows.device, dtype=torch.float32), 16)
    res = None if residual is None else _aligned(residual, 16)
    token = _prof.kernel_begin(
        "unshift_unpartition_crop_norm_3d",
        lambda: {"bytes": _nbytes(out) * (3 if res is not None else 2) + _nbytes(normed)})
    _native.require().unshift_unpartition_crop_norm_3d(out, normed, _aligned(windows, 16), res, w, b,
                                                       float(eps), B, D, H, W, C, *window_size,
                                                       *shift_size)
    _prof.count("unshift_unpartition_crop_norm_3d")
    _prof.kernel_end(token)
    return out, normed


# Neighbour order of the concatenation in patch merging: (i, j, k) offsets along
# (D, H, W) for the eight parts.  itertools.product order (MONAI's PatchMergingV2
# and the bundled network's PatchMerging).
PRODUCT_ORDER = tuple((i, j, k) for i in range(2) for j in range(2) for k in range(2))


def patch_merge_norm_3d(
    x: torch.Tensor,
    weight: torch.Tensor,
    bias: torch.Tensor,
    eps: float,
    order=PRODUCT_ORDER,
    out_dtype: torch.dtype | None = None,
) -> torch.Tensor:
    """``layer_norm(cat([x[:, i::2, j::2, k::2] for (i, j, k) in order], -1))`` in one pass.

    ``x`` is ``[B, D, H, W, C]``; odd dims are zero-padded at the far end (as the
    merging module's ``F.pad``); the result is ``[B, ceil(D/2), ceil(H/2),
    ceil(W/2), 8C]`` in ``out_dtype`` (default ``x.dtype``), the norm computed in
    fp32.  C must be a multiple of 8 with 8C at most 3072.
    """
    if x.ndim != 5:
        raise ValueError("x must have shape [B, D, H, W, C]")
    order = tuple(tuple(int(v) for v in o) for o in order)
    if len(order) != 8 or any(len(o) != 3 or min(o) < 0 or max(o) > 1 for o in order):
        raise ValueError("order must hold eight (i, j, k) offsets in {0, 1}")
    _check_dtype(x.dtype)
    out_dtype = x.dtype if out_dtype is None else out_dtype
    _check_dtype(out_dtype)
    B, D, H, W, C = (int(v) for v in x.shape)
    if C % 8 or 8 * C > 3072 or C == 0:
        raise ValueError("patch_merge_norm_3d needs C a multiple of 8 and 8C at most 3072")
    if tuple(weight.shape) != (8 * C,) or tuple(bias.shape) != (8 * C,):
        raise ValueError("weight and bias must have shape [8C]")
    shape = (B, -(-D // 2), -(-H // 2), -(-W // 2), 8 * C)
    if x.device.type == "meta":
        return torch.empty(shape, dtype=out_dtype, device=x.device)
    if x.device.type != "cuda":
        raise RuntimeError(f"crumpet_b200 runs patch_merge_norm_3d on CUDA devices only (got {x.device})")
    if torch.is_grad_enabled() and (x.requires_grad or weight.requires_grad or bias.requires_grad):
        raise RuntimeError("patch_merge_norm_3d has no backward; call it under torch.no_grad()")
    out = torch.empty(shape, dtype=out_dtype, device=x.device)
    w = _aligned(weight.detach().to(device=x.device, dtype=torch.float32), 16)
    b = _aligned(bias.detach().to(device=x.device, dtype=torch.float32), 16)
    codes = [i | (j << 1) | (k << 2) for i, j, k in order]
    token = _prof.kernel_begin("patch_merge_norm_3d", lambda: {"bytes": _nbytes(x) + _nbytes(out)})
    _native.require().patch_merge_norm_3d(out, _aligned(x, 16), w, b, float(eps), codes)
    _prof.count("patch_merge_norm_3d")
    _prof.kernel_end(token)
    return out


def proj_out_lanes(C: int) -> int:
    """Lanes per voxel of the proj_out norm kernel for C channels (0: unsupported)."""
    if C <= 0 or C > 768 or C % 8:
        return 0
    p = 1
    while p * 24 < C:
        p *= 2
    return p if C % p == 0 else 0


def proj_out_norm_3d(
    x: torch.Tensor,
    eps: float = 1e-5,
    weight: torch.Tensor | None = None,
    bias: torch.Tensor | None = None,
    out_dtype: torch.dtype | None = None,
) -> torch.Tensor:
    """``layer_norm(x.permute(0, 2, 3, 4, 1), [C], weight, bias, eps).permute(0, 4, 1, 2, 3)``.

    ``x`` is a contiguous channels-first ``[B, C, D, H, W]`` volume.  The norm is
    computed in fp32 and written channels-last in ``out_dtype`` (default
    ``x.dtype``); the result is the ``[B, C, D, H, W]`` view of that storage, with
    the strides MONAI's ``SwinTransformer.proj_out`` returns.  C must be a
    multiple of 8, at most 768, and divisible by its lanes per voxel
    (:func:`proj_out_lanes`).
    """
    if x.ndim != 5:
        raise ValueError("x must have shape [B, C, D, H, W]")
    _check_dtype(x.dtype)
    out_dtype = x.dtype if out_dtype is None else out_dtype
    _check_dtype(out_dtype)
    B, C, D, H, W = (int(v) for v in x.shape)
    if proj_out_lanes(C) == 0:
        raise ValueError("proj_out_norm_3d needs C a multiple of 8, at most 768, divisible by "
                         "its lanes per voxel")
    if (weight is None) != (bias is None):
        raise ValueError("weight and bias must both be given or both be None")
    if weight is not None and (tuple(weight.shape) != (C,) or tuple(bias.shape) != (C,)):
        raise ValueError("weight and bias must have shape [C]")
    if x.device.type == "meta":
        return torch.empty((B, D, H, W, C), dtype=out_dtype, device=x.device).permute(0, 4, 1, 2, 3)
    if x.device.type != "cuda":
        raise RuntimeError(f"crumpet_b200 runs proj_out_norm_3d on CUDA devices only (got {x.device})")
    if torch.is_grad_enabled() and any(t is not None and t.requires_grad for t in (x, weight, bias)):
        raise RuntimeError("proj_out_norm_3d has no backward; call it under torch.no_grad()")
    out = torch.empty((B, D, H, W, C), dtype=out_dtype, device=x.device)
    w = b = None
    if weight is not None:
        w = _aligned(weight.detach().to(device=x.device, dtype=torch.float32), 16)
        b = _aligned(bias.detach().to(device=x.device, dtype=torch.float32), 16)
    token = _prof.kernel_begin("proj_out_norm_3d", lambda: {"bytes": _nbytes(x) + _nbytes(out)})
    _native.require().proj_out_norm_3d(out, _aligned(x, 16), w, b, float(eps))
    _prof.count("proj_out_norm_3d")
    _prof.kernel_end(token)
    return out.permute(0, 4, 1, 2, 3)
