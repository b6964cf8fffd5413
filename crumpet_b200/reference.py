"""Eager PyTorch forms of the shifted-window mechanics.

These are the public ``*_reference`` functions of the crumpet API
(torch-ext/crumpet/reference.py:50-184): plain torch.roll / view / permute
implementations that run on any device.  crumpet_b200 never routes a kernel
call through them; they serve the eager (unpatched) Swin UNETR blocks in
``crumpet_b200.swin_unetr`` and users who want the eager form explicitly.
"""

from __future__ import annotations

from typing import Sequence

import torch


def _as3(name: str, value: Sequence[int]) -> tuple[int, int, int]:
    if len(value) != 3:
        raise ValueError(f"{name} must contain exactly three values")
    out = tuple(int(v) for v in value)
    if min(out) < 0:
        raise ValueError(f"{name} values must be non-negative")
    return out  # type: ignore[return-value]


def _require_divisible(D: int, H: int, W: int, ws: tuple[int, int, int]) -> None:
    if min(ws) <= 0:
        raise ValueError("window_size values must be positive")
    if D % ws[0] or H % ws[1] or W % ws[2]:
        raise ValueError(
            "standalone CRUMPET kernels require D, H and W to be divisible by window_size"
        )


def _require_shift(ws: tuple[int, int, int], ss: tuple[int, int, int]) -> None:
    for axis in range(3):
        if not 0 <= ss[axis] < ws[axis]:
            raise ValueError(
                f"shift_size[{axis}] must satisfy 0 <= shift < window_size[{axis}]"
            )


def window_partition_reference(x: torch.Tensor, window_size: Sequence[int]) -> torch.Tensor:
    """``[B, D, H, W, C]`` -> ``[B * nW, ws_d * ws_h * ws_w, C]`` (window-major, row-major)."""
    if x.ndim != 5:
        raise ValueError("window_partition_reference expects [B, D, H, W, C]")
    wd, wh, ww = _as3("window_size", window_size)
    B, D, H, W, C = x.shape
    _require_divisible(D, H, W, (wd, wh, ww))
    blocks = x.reshape(B, D // wd, wd, H // wh, wh, W // ww, ww, C)
    blocks = blocks.permute(0, 1, 3, 5, 2, 4, 6, 7)
    return blocks.reshape(-1, wd * wh * ww, C)


def window_reverse_reference(
    windows: torch.Tensor, window_size: Sequence[int], dims: Sequence[int]
) -> torch.Tensor:
    """Inverse of :func:`window_partition_reference`; ``dims`` is ``[B, D, H, W(, C)]``."""
    wd, wh, ww = _as3("window_size", window_size)
    if len(dims) not in (4, 5):
        raise ValueError("dims must be [B, D, H, W] or [B, D, H, W, C]")
    B, D, H, W = (int(v) for v in list(dims)[:4])
    _require_divisible(D, H, W, (wd, wh, ww))
    grid = windows.reshape(B, D // wd, H // wh, W // ww, wd, wh, ww, -1)
    grid = grid.permute(0, 1, 4, 2, 5, 3, 6, 7)
    return grid.reshape(B, D, H, W, -1)


def compute_attn_mask_3d_reference(
    D: int,
    H: int,
    W: int,
    window_size: Sequence[int],
    shift_size: Sequence[int],
    dtype: torch.dtype,
    device: torch.device | str,
) -> torch.Tensor:
    """MONAI's shifted-window mask: -100 between tokens of different roll regions."""
    ws = _as3("window_size", window_size)
    ss = _as3("shift_size", shift_size)
    _require_divisible(D, H, W, ws)
    _require_shift(ws, ss)
    n = ws[0] * ws[1] * ws[2]
    nw = (D // ws[0]) * (H // ws[1]) * (W // ws[2])
    if not any(ss):
        return torch.zeros((nw, n, n), dtype=dtype, device=device)

    def region(size: int, w: int, s: int) -> torch.Tensor:
        idx = torch.arange(size, device=device)
        r = torch.full((size,), 2, dtype=torch.int64, device=device)
        r[idx < size - s] = 1
        r[idx < size - w] = 0
        return r

    label = (
        9 * region(D, ws[0], ss[0]).view(D, 1, 1)
        + 3 * region(H, ws[1], ss[1]).view(1, H, 1)
        + region(W, ws[2], ss[2]).view(1, 1, W)
    )
    lw = window_partition_reference(label.view(1, D, H, W, 1), ws).squeeze(-1)
    differs = lw.unsqueeze(1) != lw.unsqueeze(2)
    out = torch.zeros((nw, n, n), dtype=dtype, device=device)
    out.masked_fill_(differs, -100.0)
    return out


def unfused_shift_partition_3d_reference(
    x: torch.Tensor, window_size: Sequence[int], shift_size: Sequence[int]
) -> torch.Tensor:
    """``torch.roll(x, -shift)`` over (D, H, W) followed by the window partition."""
    if x.ndim != 5:
        raise ValueError("x must have shape [B, D, H, W, C]")
    ws = _as3("window_size", window_size)
    ss = _as3("shift_size", shift_size)
    _require_divisible(int(x.shape[1]), int(x.shape[2]), int(x.shape[3]), ws)
    _require_shift(ws, ss)
    if any(ss):
        x = torch.roll(x, shifts=(-ss[0], -ss[1], -ss[2]), dims=(1, 2, 3))
    return window_partition_reference(x, ws)


def unfused_unshift_unpartition_3d_reference(
    windows: torch.Tensor,
    B: int,
    D: int,
    H: int,
    W: int,
    C: int,
    window_size: Sequence[int],
    shift_size: Sequence[int],
) -> torch.Tensor:
    """Window reverse followed by ``torch.roll(+shift)`` over (D, H, W)."""
    ws = _as3("window_size", window_size)
    ss = _as3("shift_size", shift_size)
    _require_divisible(D, H, W, ws)
    _require_shift(ws, ss)
    x = window_reverse_reference(windows, ws, (B, D, H, W))
    if int(x.shape[-1]) != int(C):
        raise ValueError("C does not match the windows tensor")
    if any(ss):
        x = torch.roll(x, shifts=ss, dims=(1, 2, 3))
    return x


__all__ = [
    "compute_attn_mask_3d_reference",
    "window_partition_reference",
    "window_reverse_reference",
    "unfused_shift_partition_3d_reference",
    "unfused_unshift_unpartition_3d_reference",
]
