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
from typing import NamedTuple, Sequence

import torch

from . import _ops as _native
from . import profiling as _prof
from .cache import (clear_mask_cache, get_or_compute_mask, make_mask_key, mask_cache_info,
                    remember_mask_geometry)
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
    "fused_swin_attention_shifted",
    "swin_window_attention_qkv",
    "attention_bias_tiles",
    "swin_window_attention_qkv_tiles",
    "norm_shift_partition_3d",
    "unshift_unpartition_crop_3d",
    "unshift_unpartition_crop_norm_3d",
    "patch_merge_norm_3d",
    "proj_out_norm_3d",
    "window_linear",
)


_fakes_registered = False


def _register_fake_impls() -> None:
    """Shape-only (fake / meta) implementations for the ops.  They mutate preallocated
    outputs and return nothing, so each fake is a no-op (reference:
    torch-ext/crumpet/__init__.py:50-73).  Runs once, when the native library loads."""
    global _fakes_registered
    register = getattr(torch.library, "register_fake", None)
    if _fakes_registered or register is None or not _native.loaded():
        return
    _fakes_registered = True
    noop = lambda *args, **kwargs: None  # noqa: E731
    for name in _OP_NAMES:
        try:
            register(f"crumpet_ops::{name}")(noop)
        except (RuntimeError, AttributeError, ValueError):
            pass  # already registered (a second package import in the same process)


_native.on_load(_register_fake_impls)


def _nvtx(name: str):
    """An NVTX range around a launch when CRUMPET_ENABLE_NVTX=1 and CUDA is up."""
    if os.environ.get("CRUMPET_ENABLE_NVTX", "0") == "1" and torch.cuda.is_available():
        return torch.cuda.nvtx.range(name)
    return contextlib.nullcontext()


def _as_triple(name: str, value: Sequence[int]) -> tuple[int, int, int]:
    items = tuple(int(v) for v in value)
    if len(items) != 3:
        raise ValueError(f"{name} must contain exactly three values")
    if min(items) < 0:
        raise ValueError(f"{name} values must be non-negative")
    return items  # type: ignore[return-value]


class _Grid(NamedTuple):
    """A volume [D, H, W] cut into windows, with the cyclic shift of a Swin block."""

    dims: tuple[int, int, int]
    window: tuple[int, int, int]
    shift: tuple[int, int, int]

    @property
    def tokens(self) -> int:  # tokens per window
        return self.window[0] * self.window[1] * self.window[2]

    @property
    def windows(self) -> int:  # windows per batch entry
        return ((self.dims[0] // self.window[0]) * (self.dims[1] // self.window[1])
                * (self.dims[2] // self.window[2]))

    def windows_shape(self, B: int, C: int) -> tuple[int, int, int]:
        return (B * self.windows, self.tokens, C)


# The rules a grid must meet, checked in this order; each is (violated?, message).  The
# messages and the order are the reference's (torch-ext/crumpet/__init__.py:89-117): its
# tests match on "divisible" and "shift_size".
_GRID_RULES = (
    (lambda g: min(g.dims) <= 0, lambda g: "D, H and W must be positive"),
    (lambda g: min(g.window) <= 0, lambda g: "window_size values must be positive"),
    (lambda g: any(d % w for d, w in zip(g.dims, g.window)),
     lambda g: "standalone CRUMPET kernels require D, H and W to be divisible by window_size"),
    (lambda g: _first_bad_shift(g) is not None,
     lambda g: "shift_size[{0}] must satisfy 0 <= shift < window_size[{0}]".format(_first_bad_shift(g))),
)


def _first_bad_shift(g: _Grid) -> int | None:
    return next((a for a in range(3) if not 0 <= g.shift[a] < g.window[a]), None)


def _grid(D, H, W, window_size, shift_size) -> _Grid:
    g = _Grid((int(D), int(H), int(W)), _as_triple("window_size", window_size),
              _as_triple("shift_size", shift_size))
    for violated, message in _GRID_RULES:
        if violated(g):
            raise ValueError(message(g))
    return g


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
    ws = _as_triple("window_size", window_size)
    ss = _as_triple("shift_size", shift_size)
    _check_dtype(dtype)
    g = _grid(D, H, W, ws, ss)
    dev = torch.device(device)
    shape = (g.windows, g.tokens, g.tokens)
    if dev.type == "meta":
        return torch.empty(shape, dtype=dtype, device=dev)
    _require_cuda(dev, "compute_attn_mask_3d")
    if g.tokens > 1024:
        raise ValueError("compute_attn_mask_3d supports window volumes up to 1024")

    def compute() -> torch.Tensor:
        out = torch.empty(shape, dtype=dtype, device=dev)
        with _nvtx("crumpet.compute_attn_mask_3d"):
            _native.require().compute_attn_mask_3d(out, *g.dims, *g.window, *g.shift)
            _prof.count("compute_attn_mask_3d")
        # fused_swin_attention recognises this mask (while nobody writes to it) and adds
        # it on chip from the window geometry
        remember_mask_geometry(out, tuple(d // w for d, w in zip(g.dims, g.window)),
                               g.window, g.shift)
        return out

    return get_or_compute_mask(make_mask_key(*g.dims, g.window, g.shift, dtype, dev), compute)


# The two window permutations and their gradients.  Each is one op; the gradient of
# one permutation is the other permutation, registered under the reference's
# *_backward op names (torch-ext/torch_binding.cpp:23-25,29-31).
#   (to_windows, gradient) -> op name
_PERMUTE_OPS = {
    (True, False): "fused_shift_partition_3d",
    (False, False): "fused_unshift_unpartition_3d",
    (False, True): "fused_shift_partition_3d_backward",
    (True, True): "fused_unshift_unpartition_3d_backward",
}


def _permute(t: torch.Tensor, to_windows: bool, g: _Grid, B: int, C: int,
             gradient: bool = False) -> torch.Tensor:
    """Launch one window permutation of ``t`` into a new tensor: volume [B, D, H, W, C]
    -> windows (``to_windows``) or windows -> volume."""
    name = _PERMUTE_OPS[(to_windows, gradient)]
    op = getattr(_native.require(), name)
    src = t.contiguous()
    if to_windows:
        out = torch.empty(g.windows_shape(B, C), dtype=t.dtype, device=t.device)
        op(out, src, *g.window, *g.shift)
    else:
        out = torch.empty((B, *g.dims, C), dtype=t.dtype, device=t.device)
        op(out, src, B, *g.dims, C, *g.window, *g.shift)
    _prof.count(name)
    return out


class _WindowPermute(torch.autograd.Function):
    """Autograd for both permutations: the backward runs the inverse permutation."""

    @staticmethod
    def forward(ctx, t, to_windows, g, B, C):
        ctx.args = (to_windows, g, B, C)
        return _permute(t, to_windows, g, B, C)

    @staticmethod
    def backward(ctx, grad):
        to_windows, g, B, C = ctx.args
        return _permute(grad, not to_windows, g, B, C, gradient=True), None, None, None, None


def _run_permute(t: torch.Tensor, to_windows: bool, g: _Grid, B: int, C: int) -> torch.Tensor:
    with _nvtx("crumpet." + _PERMUTE_OPS[(to_windows, False)]):
        if torch.is_grad_enabled() and t.requires_grad:
            return _WindowPermute.apply(t, to_windows, g, B, C)
        return _permute(t, to_windows, g, B, C)


def fused_shift_partition_3d(
    x: torch.Tensor, window_size: Sequence[int], shift_size: Sequence[int]
) -> torch.Tensor:
    """Cyclic shift by ``-shift_size`` and 3D window partition of ``[B, D, H, W, C]``."""
    if x.ndim != 5:
        raise ValueError("x must have shape [B, D, H, W, C]")
    ws = _as_triple("window_size", window_size)
    ss = _as_triple("shift_size", shift_size)
    _check_dtype(x.dtype)
    B, D, H, W, C = (int(v) for v in x.shape)
    g = _grid(D, H, W, ws, ss)
    if x.device.type == "meta":
        return torch.empty(g.windows_shape(B, C), dtype=x.dtype, device=x.device)
    _require_cuda(x, "fused_shift_partition_3d")
    return _run_permute(x, True, g, B, C)


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
    ws = _as_triple("window_size", window_size)
    ss = _as_triple("shift_size", shift_size)
    _check_dtype(windows.dtype)
    B, C = int(B), int(C)
    g = _grid(D, H, W, ws, ss)
    expected = g.windows_shape(B, C)
    if tuple(int(v) for v in windows.shape) != expected:
        raise ValueError(f"windows must have shape {expected}")
    if windows.device.type == "meta":
        return torch.empty((B, *g.dims, C), dtype=windows.dtype, device=windows.device)
    _require_cuda(windows, "fused_unshift_unpartition_3d")
    return _run_permute(windows, False, g, B, C)


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


def device_status(clear: bool = False, device: torch.device | int | None = None) -> int:
    """The device error word of crumpet_b200's kernels on ``device`` (default: the current
    CUDA device): 0 while healthy; non-zero once a kernel gave up on one of its bounded
    waits (it then stopped early, so its output is incomplete) or met an out-of-range
    relative-position index.  ``clear`` resets it.  Reading it waits for the device."""
    with torch.cuda.device(device if device is not None else torch.cuda.current_device()):
        value = int(_native.capi().crumpet_device_status(1 if clear else 0))
    if value < 0:
        raise RuntimeError(f"crumpet_b200: cannot read the device error word ({value})")
    return value


def check_device_status(device: torch.device | int | None = None) -> None:
    """Raise RuntimeError (and clear the word) if :func:`device_status` is non-zero."""
    value = device_status(clear=True, device=device)
    if value:
        raise RuntimeError(
            f"crumpet_b200 kernel reported device error {value}: a bounded wait expired or "
            "an input was out of range, so an output is incomplete")


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
    "device_status",
    "check_device_status",
    "window_partition_reference",
    "window_reverse_reference",
    "unfused_shift_partition_3d_reference",
    "unfused_unshift_unpartition_3d_reference",
    "compute_attn_mask_3d_reference",
]
