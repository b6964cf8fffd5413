"""crumpet_b200: B200-native (sm_100a) 3D shifted-window kernels for Swin UNETR.

Drop-in for the public API of ``crumpet`` (torch-ext/crumpet/__init__.py):
``compute_attn_mask_3d``, ``fused_shift_partition_3d``,
``fused_unshift_unpartition_3d``, ``fused_swin_attention``,
``patch_monai_swin_unetr`` / ``unpatch_monai_swin_unetr``, the mask cache
helpers and the eager ``*_reference`` functions, with the same argument
meaning, validation and error types.  The kernels run through the
``torch.ops.crumpet_ops`` dispatcher ops (same schemas as the reference) over
the C ABI in ``libcrumpet_b200.so``.

Differences from the reference, by design: there is no CPU / Triton fallback
(non-CUDA tensors raise), zero-shift partitions also run the CUDA kernel, and
``fused_swin_attention`` is a dispatcher op backed by a hand-written tcgen05
kernel.
"""

from __future__ import annotations

import contextlib
import os
from typing import Sequence

import torch

from . import _ops as _native
from . import profiling as _prof
from .cache import clear_mask_cache, get_or_compute_mask, make_mask_key, mask_cache_info
from .reference import (
    compute_attn_mask_3d_reference,
    unfused_shift_partition_3d_reference,
    unfused_unshift_unpartition_3d_reference,
    window_partition_reference,
    window_reverse_reference,
)

__version__ = "0.1.0"

_SUPPORTED_DTYPES = (torch.float32, torch.float16, torch.bfloat16)
_OP_NAMES = (
    "compute_attn_mask_3d",
    "fused_shift_partition_3d",
    "fused_shift_partition_3d_backward",
    "fused_unshift_unpartition_3d",
    "fused_unshift_unpartition_3d_backward",
    "fused_swin_attention",
    "swin_window_attention_qkv",
    "norm_shift_partition_3d",
    "unshift_unpartition_crop_3d",
    "unshift_unpartition_crop_norm_3d",
    "patch_merge_norm_3d",
    "proj_out_norm_3d",
    "window_linear",
)


_fakes_registered = False


def _register_fake_impls() -> None:
    # The ops mutate preallocated outputs and return nothing, so their fake
    # (meta) implementations are no-ops (reference: torch-ext/crumpet/__init__.py:50-73).
    global _fakes_registered
    if _fakes_registered or not _native.available():
        return
    _fakes_registered = True
    register = getattr(torch.library, "register_fake", None)
    if register is None:
        return
    for name in _OP_NAMES:
        try:
            register(f"crumpet_ops::{name}")(lambda *args, **kwargs: None)
        except (RuntimeError, AttributeError, ValueError):
            pass


_register_fake_impls()


@contextlib.contextmanager
def _nvtx_range(name: str):
    if os.environ.get("CRUMPET_ENABLE_NVTX", "0") == "1" and torch.cuda.is_available():
        torch.cuda.nvtx.range_push(name)
        try:
            yield
        finally:
            torch.cuda.nvtx.range_pop()
    else:
        yield


def _triple(name: str, value: Sequence[int]) -> tuple[int, int, int]:
    if len(value) != 3:
        raise ValueError(f"{name} must contain exactly three values")
    out = tuple(int(v) for v in value)
    if any(v < 0 for v in out):
        raise ValueError(f"{name} values must be non-negative")
    return out  # type: ignore[return-value]


def _validate_shape(
    D: int, H: int, W: int, window_size: tuple[int, int, int], shift_size: tuple[int, int, int]
) -> None:
    if D <= 0 or H <= 0 or W <= 0:
        raise ValueError("D, H and W must be positive")
    if any(v <= 0 for v in window_size):
        raise ValueError("window_size values must be positive")
    if D % window_size[0] or H % window_size[1] or W % window_size[2]:
        raise ValueError(
            "standalone CRUMPET kernels require D, H and W to be divisible by window_size"
        )
    for axis, (shift, window) in enumerate(zip(shift_size, window_size)):
        if shift < 0 or shift >= window:
            raise ValueError(f"shift_size[{axis}] must satisfy 0 <= shift < window_size[{axis}]")


def _check_dtype(dtype: torch.dtype) -> None:
    if dtype not in _SUPPORTED_DTYPES:
        raise TypeError("CRUMPET supports torch.float32, torch.float16 and torch.bfloat16")


def _require_cuda(t_or_dev, what: str) -> None:
    dev = t_or_dev.device if isinstance(t_or_dev, torch.Tensor) else torch.device(t_or_dev)
    if dev.type != "cuda":
        raise RuntimeError(
            f"crumpet_b200 runs {what} on CUDA devices only (got {dev}); "
            "use the *_reference functions for an eager computation"
        )


def _geometry(D, H, W, window_size):
    volume = window_size[0] * window_size[1] * window_size[2]
    num_windows = (D // window_size[0]) * (H // window_size[1]) * (W // window_size[2])
    return volume, num_windows


def compute_attn_mask_3d(
    D: int,
    H: int,
    W: int,
    window_size: Sequence[int],
    shift_size: Sequence[int],
    dtype: torch.dtype,
    device: torch.device | str,
) -> torch.Tensor:
    """Shifted 3D Swin attention mask ``[num_windows, volume, volume]`` (0 / -100), cached."""
    window_size = _triple("window_size", window_size)
    shift_size = _triple("shift_size", shift_size)
    _check_dtype(dtype)
    D, H, W = int(D), int(H), int(W)
    _validate_shape(D, H, W, window_size, shift_size)
    dev = torch.device(device)
    volume, num_windows = _geometry(D, H, W, window_size)
    if dev.type == "meta":
        return torch.empty((num_windows, volume, volume), dtype=dtype, device=dev)
    _require_cuda(dev, "compute_attn_mask_3d")
    if volume > 1024:
        raise ValueError("compute_attn_mask_3d supports window volumes up to 1024")

    def compute() -> torch.Tensor:
        out = torch.empty((num_windows, volume, volume), dtype=dtype, device=dev)
        with _nvtx_range("crumpet.compute_attn_mask_3d"):
            _native.require().compute_attn_mask_3d(out, D, H, W, *window_size, *shift_size)
            _prof.count("compute_attn_mask_3d")
        return out

    return get_or_compute_mask(make_mask_key(D, H, W, window_size, shift_size, dtype, dev), compute)


class _ShiftPartitionFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, window_size, shift_size):
        x = x.contiguous()
        B, D, H, W, C = (int(v) for v in x.shape)
        volume, num_windows = _geometry(D, H, W, window_size)
        out = torch.empty((B * num_windows, volume, C), dtype=x.dtype, device=x.device)
        _native.require().fused_shift_partition_3d(out, x, *window_size, *shift_size)
        ctx.shape = (B, D, H, W, C)
        ctx.window_size = window_size
        ctx.shift_size = shift_size
        return out

    @staticmethod
    def backward(ctx, grad_output):
        B, D, H, W, C = ctx.shape
        grad_x = torch.empty((B, D, H, W, C), dtype=grad_output.dtype, device=grad_output.device)
        _native.require().fused_shift_partition_3d_backward(
            grad_x, grad_output.contiguous(), B, D, H, W, C, *ctx.window_size, *ctx.shift_size
        )
        return grad_x, None, None


class _UnshiftUnpartitionFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, windows, B, D, H, W, C, window_size, shift_size):
        windows = windows.contiguous()
        out = torch.empty((B, D, H, W, C), dtype=windows.dtype, device=windows.device)
        _native.require().fused_unshift_unpartition_3d(
            out, windows, B, D, H, W, C, *window_size, *shift_size
        )
        ctx.window_size = window_size
        ctx.shift_size = shift_size
        return out

    @staticmethod
    def backward(ctx, grad_output):
        B, D, H, W, C = (int(v) for v in grad_output.shape)
        volume, num_windows = _geometry(D, H, W, ctx.window_size)
        grad_windows = torch.empty(
            (B * num_windows, volume, C), dtype=grad_output.dtype, device=grad_output.device
        )
        _native.require().fused_unshift_unpartition_3d_backward(
            grad_windows, grad_output.contiguous(), *ctx.window_size, *ctx.shift_size
        )
        return grad_windows, None, None, None, None, None, None, None


def fused_shift_partition_3d(
    x: torch.Tensor, window_size: Sequence[int], shift_size: Sequence[int]
) -> torch.Tensor:
    """Cyclic shift by ``-shift_size`` and 3D window partition of ``[B, D, H, W, C]``."""
    if x.ndim != 5:
        raise ValueError("x must have shape [B, D, H, W, C]")
    window_size = _triple("window_size", window_size)
    shift_size = _triple("shift_size", shift_size)
    _check_dtype(x.dtype)
    B, D, H, W, C = (int(v) for v in x.shape)
    _validate_shape(D, H, W, window_size, shift_size)
    volume, num_windows = _geometry(D, H, W, window_size)
    if x.device.type == "meta":
        return torch.empty((B * num_windows, volume, C), dtype=x.dtype, device=x.device)
    _require_cuda(x, "fused_shift_partition_3d")
    with _nvtx_range("crumpet.fused_shift_partition_3d"):
        if torch.is_grad_enabled() and x.requires_grad:
            return _ShiftPartitionFn.apply(x, window_size, shift_size)
        out = torch.empty((B * num_windows, volume, C), dtype=x.dtype, device=x.device)
        _native.require().fused_shift_partition_3d(out, x.contiguous(), *window_size, *shift_size)
        _prof.count("fused_shift_partition_3d")
        return out


def fused_unshift_unpartition_3d(
    windows: torch.Tensor,
    B: int,
    D: int,
    H: int,
    W: int,
    C: int,
    window_size: Sequence[int],
    shift_size: Sequence[int],
) -> torch.Tensor:
    """3D window reverse and cyclic shift by ``+shift_size``: back to ``[B, D, H, W, C]``."""
    if windows.ndim != 3:
        raise ValueError("windows must have shape [B * num_windows, window_volume, C]")
    window_size = _triple("window_size", window_size)
    shift_size = _triple("shift_size", shift_size)
    _check_dtype(windows.dtype)
    B, D, H, W, C = int(B), int(D), int(H), int(W), int(C)
    _validate_shape(D, H, W, window_size, shift_size)
    volume, num_windows = _geometry(D, H, W, window_size)
    expected = (B * num_windows, volume, C)
    if tuple(int(v) for v in windows.shape) != expected:
        raise ValueError(f"windows must have shape {expected}")
    if windows.device.type == "meta":
        return torch.empty((B, D, H, W, C), dtype=windows.dtype, device=windows.device)
    _require_cuda(windows, "fused_unshift_unpartition_3d")
    with _nvtx_range("crumpet.fused_unshift_unpartition_3d"):
        if torch.is_grad_enabled() and windows.requires_grad:
            return _UnshiftUnpartitionFn.apply(windows, B, D, H, W, C, window_size, shift_size)
        out = torch.empty((B, D, H, W, C), dtype=windows.dtype, device=windows.device)
        _native.require().fused_unshift_unpartition_3d(
            out, windows.contiguous(), B, D, H, W, C, *window_size, *shift_size
        )
        _prof.count("fused_unshift_unpartition_3d")
        return out


from .fused_attention import (  # noqa: E402
    fused_swin_attention,
    swin_window_attention_qkv,
    window_linear,
)
from .block_fusion import (  # noqa: E402
    norm_shift_partition_3d,
    unshift_unpartition_crop_3d,
    unshift_unpartition_crop_norm_3d,
    patch_merge_norm_3d,
    proj_out_norm_3d,
)


def patch_monai_swin_unetr(swin_module=None) -> bool:
    """Route MONAI Swin UNETR blocks through the crumpet_b200 kernels (idempotent).

    ``swin_module`` defaults to ``monai.networks.nets.swin_unetr``; pass
    ``crumpet_b200.swin_unetr`` (the bundled MONAI-architecture model) when
    MONAI is not installed.
    """
    from .monai_patch import patch_monai_swin_unetr as patch

    return patch(swin_module)


def unpatch_monai_swin_unetr() -> bool:
    """Undo :func:`patch_monai_swin_unetr`."""
    from .monai_patch import unpatch_monai_swin_unetr as unpatch

    return unpatch()


__all__ = [
    "compute_attn_mask_3d",
    "fused_shift_partition_3d",
    "fused_unshift_unpartition_3d",
    "fused_swin_attention",
    "swin_window_attention_qkv",
    "norm_shift_partition_3d",
    "unshift_unpartition_crop_3d",
    "unshift_unpartition_crop_norm_3d",
    "patch_merge_norm_3d",
    "proj_out_norm_3d",
    "window_linear",
    "patch_monai_swin_unetr",
    "unpatch_monai_swin_unetr",
    "clear_mask_cache",
    "mask_cache_info",
    "window_partition_reference",
    "window_reverse_reference",
    "unfused_shift_partition_3d_reference",
    "unfused_unshift_unpartition_3d_reference",
    "compute_attn_mask_3d_reference",
]
