"""Fused 3D Swin window attention (hand-written sm_100a kernel).

Python entry point with the signature of the reference Triton launcher
(torch-ext/crumpet/fused_attention.py:149-226):

    fused_swin_attention(q, k, v, relative_position_bias, mask, boundary=None,
                         scale=None, block_m=64, block_n=32) -> out

``q``, ``k``, ``v``: ``[B, H, N, head_dim]`` (B = batch * windows);
``relative_position_bias``: ``[H, N, N]``; ``mask``: ``[num_windows, N, N]``
(window ``b`` uses ``mask[b % num_windows]``, which covers the reference's
``mask.shape[0] in (1, B)`` cases and MONAI's sliding-window tiling without a
``repeat``) or ``None``; ``boundary``: per-window flag, mask rows are read only
where it is non-zero.  ``block_m`` / ``block_n`` are accepted for API
compatibility and ignored: the tile shapes are fixed by the kernels' designs.

Inputs: float16, bfloat16 or float32; head_dim a power of two from 16 to 256 (the
reference's Triton kernel takes power-of-two head dims >= 16); any N >= 1.  float16
/ bfloat16 with head_dim 16 or 32 and N <= 352 run the tcgen05 tensor-core kernel;
the rest runs an fp32 SIMT kernel (float32 arithmetic throughout).
"""

from __future__ import annotations

import torch

from . import _ops as _native
from . import profiling as _prof
from .cache import mask_geometry

_ATTN_DTYPES = (torch.float32, torch.float16, torch.bfloat16)


def head_dim_supported(head_dim: int) -> bool:
    """Head dims the attention kernels take: powers of two from 16 to 256."""
    return head_dim in (16, 32, 64, 128, 256)


def fused_swin_attention(
    q: torch.Tensor,
    k: torch.Tensor,
    v: torch.Tensor,
    relative_position_bias: torch.Tensor,
    mask: torch.Tensor | None,
    boundary: torch.Tensor | None = None,
    scale: float | None = None,
    block_m: int = 64,
    block_n: int = 32,
) -> torch.Tensor:
    del block_m, block_n  # tile shape is fixed by the kernel design
    if not (q.is_cuda and k.is_cuda and v.is_cuda):
        raise RuntimeError("fused_swin_attention runs on CUDA tensors only")
    if q.shape != k.shape or q.shape != v.shape:
        raise ValueError("Q/K/V shape mismatch")
    if q.ndim != 4:
        raise ValueError("q, k and v must have shape [B, H, N, head_dim]")
    B, H, N, D = (int(s) for s in q.shape)
    if tuple(relative_position_bias.shape) != (H, N, N):
        raise ValueError(f"relative_position_bias must have shape {(H, N, N)}")
    if q.dtype not in _ATTN_DTYPES:
        raise TypeError("fused_swin_attention supports torch.float32, torch.float16 and "
                        "torch.bfloat16")
    if not head_dim_supported(D):
        raise ValueError("fused_swin_attention requires a power-of-two head_dim between 16 and 256")
    if scale is None:
        scale = 1.0 / (D ** 0.5)
    if not 0.0 < float(scale) < float("inf"):
        raise ValueError("fused attention requires a finite scale > 0")
    bias = relative_position_bias.to(q.dtype).contiguous()
    mask_t = None
    bnd = None
    geometry = None
    if mask is not None:
        if mask.ndim != 3 or tuple(mask.shape[1:]) != (N, N):
            raise ValueError(f"mask must have shape [num_windows, {N}, {N}]")
        if B % int(mask.shape[0]) != 0:
            raise ValueError(f"mask shape {int(mask.shape[0])} incompatible with B={B}")
        # A mask that compute_attn_mask_3d built (and nobody has written to since) is the
        # shifted-window mask of a known window grid: the kernel adds it on chip instead of
        # reading its rows (the same values, up to fp32 rounding)
        geometry = mask_geometry(mask)
        if geometry is not None:
            nw, win, _ = geometry
            if nw[0] * nw[1] * nw[2] != int(mask.shape[0]) or win[0] * win[1] * win[2] != N:
                geometry = None
        mask_t = None if geometry is not None else mask.to(q.dtype).contiguous()
        if boundary is not None:
            bnd = boundary if boundary.dtype == torch.uint8 else boundary.to(torch.uint8)
            bnd = bnd.contiguous()
    out = torch.empty_like(q, memory_format=torch.contiguous_format)
    ops = _native.require()
    q, k, v = q.contiguous(), k.contiguous(), v.contiguous()
    token = None
    if _prof._active:
        esize = q.element_size()
        masked = 0 if mask_t is None else (B if bnd is None else bnd)  # rows read from HBM
        token = _prof.kernel_begin("fused_swin_attention", {
            # algorithmic bytes: q, k, v, out, the bias once, plus the mask rows
            # of masked windows (resolved when the timer is summarised)
            "bytes": 4 * B * H * N * D * esize + H * N * N * esize,
            "mask_bytes": (masked, N * N * esize),
            "flops": 4 * B * H * N * N * D,
            "exps": B * H * N * N,
        })
    if geometry is not None:
        ops.fused_swin_attention_shifted(out, q, k, v, bias, bnd, list(geometry[0]),
                                         list(geometry[1]), list(geometry[2]), float(scale))
    else:
        ops.fused_swin_attention(out, q, k, v, bias, mask_t, bnd, float(scale))
    _prof.count("fused_swin_attention")
    _prof.kernel_end(token)
    return out


def tensor_core_attention(dtype: torch.dtype, N: int, head_dim: int) -> bool:
    """Whether the tcgen05 kernel runs these windows (else the fp32 SIMT kernel)."""
    return dtype in (torch.float16, torch.bfloat16) and head_dim in (16, 32) and 1 <= N <= 352


def attention_bias_tiles(relative_position_bias_table: torch.Tensor,
                         relative_position_index: torch.Tensor, N: int, scale: float,
                         dtype: torch.dtype) -> torch.Tensor:
    """The tensor-core kernel's relative-position bias operands for windows of N tokens,
    built once: one tile per (head, 128-row query tile), gathered from
    ``table[index[:N, :N]]`` and divided by ``scale`` in ``dtype``.  Pass the result as
    ``bias_tiles`` to :func:`swin_window_attention_qkv` with the same N, scale and dtype;
    rebuild it when the table changes."""
    table = relative_position_bias_table.detach()
    if table.dtype not in (torch.float32, dtype):
        table = table.float()
    H = int(table.shape[1])
    nbytes = int(_native.capi().crumpet_attention_bias_tiles_bytes(H, int(N)))
    if nbytes <= 0 or dtype not in (torch.float16, torch.bfloat16):
        raise ValueError("bias tiles exist for float16 / bfloat16 windows of 1 to 352 tokens")
    tiles = torch.empty(nbytes, dtype=torch.uint8, device=table.device)
    _native.require().attention_bias_tiles(tiles, table.contiguous(),
                                           relative_position_index.contiguous(), int(N),
                                           float(scale), dtype)
    _prof.count("attention_bias_tiles")
    return tiles


def swin_window_attention_qkv(
    qkv: torch.Tensor,
    relative_position_bias_table: torch.Tensor,
    relative_position_index: torch.Tensor,
    num_windows=(1, 1, 1),
    window_size=None,
    shift_size=(0, 0, 0),
    scale: float | None = None,
    bias_tiles: torch.Tensor | None = None,
) -> torch.Tensor:
    """Window attention straight from the packed qkv Linear output.

    ``qkv``: ``[B, N, 3, H, head_dim]`` (the qkv Linear output viewed per head);
    returns ``[B, N, H * head_dim]`` ready for the proj Linear.  The bias is
    gathered in the kernel from ``relative_position_bias_table[index[:N, :N]]``
    and, when ``shift_size`` is non-zero, the shifted-window mask of a grid of
    ``num_windows`` windows of ``window_size`` is computed on chip (window ``b``
    is ``b % prod(num_windows)``).  This is the whole body of MONAI's
    ``WindowAttention.forward`` between its two Linears
    (torch-ext/crumpet/monai_patch.py:152-196 does the same with eager glue).
    ``bias_tiles`` (from :func:`attention_bias_tiles`, tensor-core windows only) replaces
    the per-CTA gather with a copy of the prebuilt operands.
    """
    if not qkv.is_cuda:
        raise RuntimeError("swin_window_attention_qkv runs on CUDA tensors only")
    if qkv.ndim != 5 or qkv.shape[2] != 3:
        raise ValueError("qkv must have shape [B, N, 3, H, head_dim]")
    B, N, _, H, D = (int(s) for s in qkv.shape)
    if not head_dim_supported(D):
        raise ValueError("swin_window_attention_qkv requires a power-of-two head_dim between 16 "
                         "and 256")
    if qkv.dtype not in _ATTN_DTYPES:
        raise TypeError("swin_window_attention_qkv supports torch.float32, torch.float16 and "
                        "torch.bfloat16")
    if window_size is None:
        window_size = (N, 1, 1)
    if scale is None:
        scale = 1.0 / (D ** 0.5)
    if not 0.0 < float(scale) < float("inf"):
        raise ValueError("fused attention requires a finite scale > 0")
    table = relative_position_bias_table
    if table.dtype not in (torch.float32, qkv.dtype):
        table = table.float()
    out = torch.empty((B, N, H * D), dtype=qkv.dtype, device=qkv.device)
    ops = _native.require()
    token = None
    if _prof._active:
        esize = qkv.element_size()
        token = _prof.kernel_begin("swin_window_attention_qkv", {
            # algorithmic bytes: q, k, v, out (the bias is gathered on chip and
            # the mask computed on chip)
            "bytes": 4 * B * H * N * D * esize,
            "flops": 4 * B * H * N * N * D,
            "exps": B * H * N * N,
        })
    if bias_tiles is not None and tensor_core_attention(qkv.dtype, N, D):
        ops.swin_window_attention_qkv_tiles(out, qkv.contiguous(), bias_tiles, list(num_windows),
                                            list(window_size), list(shift_size), float(scale))
    else:
        ops.swin_window_attention_qkv(out, qkv.contiguous(), table.contiguous(),
                                      relative_position_index.contiguous(), list(num_windows),
                                      list(window_size), list(shift_size), float(scale))
    _prof.count("swin_window_attention_qkv")
    _prof.kernel_end(token)
    return out


__all__ = ["fused_swin_attention", "swin_window_attention_qkv", "attention_bias_tiles",
           "head_dim_supported", "tensor_core_attention"]


def window_linear(x: torch.Tensor, weight: torch.Tensor, bias: torch.Tensor | None = None) -> torch.Tensor:
    """``F.linear(x, weight, bias)`` for float16 / bfloat16 window tokens on the tensor cores.

    ``x [..., K]``, ``weight [N, K]`` (cast to ``x.dtype``, as autocast does for
    ``nn.Linear``), ``bias [N]`` (rounded to ``x.dtype``, added in fp32 before the one
    rounding of the output); the shapes of :func:`window_linear_supported`.
    """
    if x.dtype not in (torch.float16, torch.bfloat16):
        raise TypeError("window_linear takes float16 or bfloat16 tokens")
    K = int(x.shape[-1])
    if weight.ndim != 2 or int(weight.shape[1]) != K:
        raise ValueError("weight must have shape [N, K]")
    N = int(weight.shape[0])
    if not window_linear_supported(K, N):
        raise ValueError("window_linear supports K = 48 (N <= 256) or K = 96 (N <= 160), "
                         "N a multiple of 16")
    if bias is not None and tuple(bias.shape) != (N,):
        raise ValueError("bias must have shape [N]")
    if x.device.type == "meta":
        return torch.empty((*x.shape[:-1], N), dtype=x.dtype, device=x.device)
    if x.device.type != "cuda":
        raise RuntimeError(f"crumpet_b200 runs window_linear on CUDA devices only (got {x.device})")
    if torch.is_grad_enabled() and any(t is not None and t.requires_grad for t in (x, weight, bias)):
        raise RuntimeError("window_linear has no backward; call it under torch.no_grad()")
    x2 = x.reshape(-1, K)
    if not x2.is_contiguous():
        x2 = x2.contiguous()
    if x2.data_ptr() % 16:
        x2 = x2.clone()
    w = weight.detach().to(device=x.device, dtype=x.dtype).contiguous()
    b = None
    if bias is not None:
        b = bias.detach().to(device=x.device, dtype=x.dtype).to(torch.float32).contiguous()
    out = torch.empty((x2.shape[0], N), dtype=x.dtype, device=x.device)
    token = _prof.kernel_begin("window_linear", lambda: {
        "bytes": x2.numel() * x2.element_size() + out.numel() * out.element_size()})
    _native.require().window_linear(out, x2, w, b)
    _prof.count("window_linear")
    _prof.kernel_end(token)
    return out.view(*x.shape[:-1], N)


def window_linear_supported(K: int, N: int) -> bool:
    """Shapes :func:`window_linear` runs: K = 48 with N <= 256, or K = 96 with N <= 160; N a
    multiple of 16 (the qkv and proj Linears of feature-size-48 stages 1 and 2, except the
    stage-2 qkv with N = 288)."""
    if N < 16 or N % 16:
        return False
    return (K == 48 and N <= 256) or (K == 96 and N <= 160)
