"""Loader for the native crumpet_b200 libraries.

``libcrumpet_b200.so`` (kernels + C ABI) and ``_C.so`` (the ``crumpet_ops``
torch dispatcher registration) are built in-tree by ``crumpet_b200._build``.
There is no fallback: if the libraries are missing, every op raises with the
load error, so a silent CPU or eager path can never stand in for a kernel.
"""

from __future__ import annotations

import ctypes
from pathlib import Path

import torch

_PKG = Path(__file__).resolve().parent
LIB_PATH = _PKG / "libcrumpet_b200.so"
EXT_PATH = _PKG / "_C.so"

_load_error: Exception | None = None
ops = None
_on_load: list = []


def _try_load() -> bool:
    global ops, _load_error
    if ops is not None:
        return True
    try:
        torch.ops.load_library(str(EXT_PATH))
        ops = torch.ops.crumpet_ops
        _load_error = None
    except Exception as exc:  # pragma: no cover - exercised only without a build
        _load_error = exc
        return False
    for hook in _on_load:
        hook()
    return True


def on_load(hook) -> None:
    """Run ``hook()`` once the libraries are loaded (now, if they already are)."""
    _on_load.append(hook)
    if ops is not None:
        hook()


def reload() -> bool:
    """Load the libraries now (for example after a build in the same process); True once
    they are loaded.  Importing the package maps no native library: the first op call,
    ``require()``, ``available()`` or ``capi()`` does."""
    return _try_load()


def loaded() -> bool:
    """Whether the libraries are mapped into this process, without trying to load them."""
    return ops is not None


def available() -> bool:
    return _try_load()


def require():
    """Return ``torch.ops.crumpet_ops`` (loading it on first use) or raise the reason it
    is unavailable."""
    if ops is None and not _try_load():
        raise RuntimeError(
            "crumpet_b200 native kernels are not built or failed to load "
            f"({EXT_PATH}): {_load_error!r}. Run `python -m crumpet_b200._build`."
        )
    return ops


_capi = None


def capi() -> ctypes.CDLL:
    """The C ABI library (include/crumpet_b200.h) opened through ctypes."""
    global _capi
    if _capi is None:
        lib = ctypes.CDLL(str(LIB_PATH))
        i64, vp, i32 = ctypes.c_int64, ctypes.c_void_p, ctypes.c_int
        copy_args = [vp, vp, i32] + [i64] * 11 + [vp]
        for name in (
            "crumpet_fused_shift_partition_3d",
            "crumpet_fused_unshift_unpartition_3d",
            "crumpet_fused_shift_partition_3d_backward",
            "crumpet_fused_unshift_unpartition_3d_backward",
        ):
            getattr(lib, name).argtypes = copy_args
            getattr(lib, name).restype = i32
        lib.crumpet_compute_attn_mask_3d.argtypes = [vp, i32] + [i64] * 9 + [vp]
        lib.crumpet_compute_attn_mask_3d.restype = i32
        lib.crumpet_fused_swin_attention.argtypes = [
            vp, vp, vp, vp, vp, vp, i64, vp, i32, i64, i64, i64, i64, ctypes.c_float, vp,
        ]
        lib.crumpet_fused_swin_attention.restype = i32
        lib.crumpet_fused_swin_attention_shifted.argtypes = (
            [vp, vp, vp, vp, vp, vp, i32] + [i64] * 13 + [ctypes.c_float, vp])
        lib.crumpet_fused_swin_attention_shifted.restype = i32
        lib.crumpet_swin_window_attention_qkv.argtypes = (
            [vp, vp, vp, i32, i64, vp] + [i64] * 10 + [i32] + [i64] * 4 + [ctypes.c_float, vp])
        lib.crumpet_swin_window_attention_qkv.restype = i32
        lib.crumpet_attention_bias_tiles_bytes.argtypes = [i64, i64]
        lib.crumpet_attention_bias_tiles_bytes.restype = i64
        lib.crumpet_attention_bias_tiles.argtypes = [vp, vp, i32, i64, vp, i64, i32, i64, i64,
                                                     ctypes.c_float, vp]
        lib.crumpet_attention_bias_tiles.restype = i32
        lib.crumpet_swin_window_attention_qkv_tiles.argtypes = (
            [vp, vp, vp] + [i64] * 9 + [i32] + [i64] * 4 + [ctypes.c_float, vp])
        lib.crumpet_swin_window_attention_qkv_tiles.restype = i32
        lib.crumpet_swin_window_attention_qkv_static_tiles.argtypes = (
            [vp, vp, vp, i32, i64, vp] + [i64] * 10 + [i32] + [i64] * 4 + [ctypes.c_float, vp])
        lib.crumpet_swin_window_attention_qkv_static_tiles.restype = i32
        lib.crumpet_norm_shift_partition_3d.argtypes = (
            [vp, i32, vp, i32, vp, vp, ctypes.c_float] + [i64] * 11 + [vp])
        lib.crumpet_norm_shift_partition_3d.restype = i32
        lib.crumpet_unshift_unpartition_crop_3d.argtypes = [vp, vp, vp, i32] + [i64] * 11 + [vp]
        lib.crumpet_unshift_unpartition_crop_3d.restype = i32
        lib.crumpet_unshift_unpartition_crop_norm_3d.argtypes = (
            [vp, vp, i32, vp, vp, i32, vp, vp, ctypes.c_float] + [i64] * 11 + [vp])
        lib.crumpet_unshift_unpartition_crop_norm_3d.restype = i32
        lib.crumpet_patch_merge_norm_3d.argtypes = (
            [vp, i32, vp, i32, vp, vp, ctypes.c_float] + [i64] * 5 + [vp, vp])
        lib.crumpet_patch_merge_norm_3d.restype = i32
        lib.crumpet_proj_out_norm_3d.argtypes = (
            [vp, i32, vp, i32, vp, vp, ctypes.c_float] + [i64] * 5 + [vp])
        lib.crumpet_proj_out_norm_3d.restype = i32
        lib.crumpet_window_linear.argtypes = [vp, vp, vp, vp, i32] + [i64] * 3 + [vp]
        lib.crumpet_window_linear.restype = i32
        roi = [i64] * 3
        lib.crumpet_roi_gather.argtypes = [vp, i32, vp, i32] + [i64] * 4 + [vp, i64] + roi + [vp]
        lib.crumpet_roi_gather.restype = i32
        lib.crumpet_roi_accumulate.argtypes = [vp, vp, i32] + [i64] * 4 + [vp, i64] + roi + [vp]
        lib.crumpet_roi_accumulate.restype = i32
        lib.crumpet_roi_argmax.argtypes = [vp, vp, vp, vp, vp, vp] + [i64] * 4 + [vp]
        lib.crumpet_roi_argmax.restype = i32
        lib.crumpet_last_error.argtypes = []
        lib.crumpet_last_error.restype = ctypes.c_char_p
        lib.crumpet_abi_version.argtypes = []
        lib.crumpet_abi_version.restype = i32
        lib.crumpet_test_stall_attention.argtypes = [i32]
        lib.crumpet_test_stall_attention.restype = i32
        lib.crumpet_device_status.argtypes = [i32]
        lib.crumpet_device_status.restype = i32
        _capi = lib
    return _capi


def last_error() -> str:
    return capi().crumpet_last_error().decode()
