"""Reversible patch of MONAI-architecture Swin UNETR blocks onto crumpet_b200.

Same contract as the reference patch (torch-ext/crumpet/monai_patch.py:235-275):
``patch_monai_swin_unetr`` replaces

* ``SwinTransformerBlock.forward_part1``: LayerNorm -> pad -> fused roll +
  partition -> attention -> fused unpartition + reverse roll -> crop
  (reference :72-114), with norm1, the pad, the roll + partition and the
  autocast cast for the qkv Linear in one kernel (``norm_shift_partition_3d``)
  and the unpartition, roll back and crop in another
  (``unshift_unpartition_crop_3d``);
* ``SwinTransformerBlock.forward`` (not patched by the reference): in eval
  mode without checkpointing, the residual add of the attention half and the
  block's norm2 are folded into the unpartition + crop kernel
  (``unshift_unpartition_crop_norm_3d``), which hands norm2(x) to the MLP;
* ``BasicLayer.forward``: channels-last permute, the cached shifted-window mask
  from ``compute_attn_mask_3d`` on the padded grid, blocks, downsample
  (reference :201-232); a recognised patch merging (neighbour concatenation in
  itertools.product order: MONAI's PatchMergingV2 or the bundled module) runs as
  one gather + LayerNorm kernel and a channels-first reduction GEMM, which also
  removes the final permute copy;
* ``WindowAttention.forward``: qkv Linear -> fused window attention -> proj
  Linear (reference :117-198), falling back to the module's own eager forward
  where the reference does (training, attention dropout, head_dim < 16) and for
  head dims that are not a power of two up to 256 (the reference's Triton kernel
  cannot compile those); fp16 / bf16 head_dim 16 / 32 windows of up to 352 tokens
  run the tcgen05 kernel, the rest (fp32 activations included) the fp32 SIMT one;
* ``SwinTransformer.proj_out`` (not patched by the reference; only when the
  module has it): the hidden-state LayerNorm of every stage output runs as one
  kernel that reads the channels-first volume and writes the channels-last
  normalised result (``proj_out_norm_3d``) instead of a permute, an autocast
  cast, a contiguous copy and torch's LayerNorm;

returns True when it installs the patch and False when it is already active;
``unpatch_monai_swin_unetr`` restores the originals.  It raises RuntimeError
when the target module lacks one of the patched names.

``swin_module`` selects the module to patch: MONAI's
``monai.networks.nets.swin_unetr`` by default (as in the reference), or
``crumpet_b200.swin_unetr``, the bundled MONAI-architecture network.

Differences from the reference glue, all of them removals of work: for masks
built by the patched ``BasicLayer`` (which records their window geometry on
the tensor), attention runs ``swin_window_attention_qkv`` -- q/k/v read in
place from the qkv Linear output, bias gathered and shifted-window mask
computed inside the kernel, output written proj-ready -- so the q/k/v copies,
bias gather, mask ``repeat``, per-call ``abs().amax()`` mask scan and output
transpose disappear.  Masks without recorded geometry take the dense-mask
kernel, indexed modulo the number of windows and with boundary flags derived
once per mask.
"""

from __future__ import annotations

import functools
import inspect
import os
from typing import Any

import torch
import torch.nn.functional as F

from . import compute_attn_mask_3d, fused_shift_partition_3d, fused_unshift_unpartition_3d
from .block_fusion import (
    PRODUCT_ORDER,
    patch_merge_norm_3d,
    proj_out_lanes,
    proj_out_norm_3d,
    norm_shift_partition_3d,
    unshift_unpartition_crop_3d,
    unshift_unpartition_crop_norm_3d,
)
from .fused_attention import (
    attention_bias_tiles,
    fused_swin_attention,
    head_dim_supported,
    swin_window_attention_qkv,
    tensor_core_attention,
    window_linear,
    window_linear_supported,
)

_STATE: dict[str, Any] = {}
_MISSING = object()
_BOUNDARY_ATTR = "_crumpet_boundary"
_GEOMETRY_ATTR = "_crumpet_geometry"


def _fused_attn_enabled() -> bool:
    """Opt out of the fused attention with CRUMPET_DISABLE_FUSED_ATTN=1."""
    return os.environ.get("CRUMPET_DISABLE_FUSED_ATTN", "0") != "1"


def _load_swin(swin_module):
    if swin_module is None:
        try:
            import monai.networks.nets.swin_unetr as swin_module  # type: ignore
        except Exception as exc:
            raise RuntimeError("MONAI Swin UNETR is not importable") from exc
    for name in ("SwinTransformerBlock", "BasicLayer", "WindowAttention", "get_window_size"):
        if not hasattr(swin_module, name):
            raise RuntimeError(f"{swin_module.__name__} is missing {name}")
    return swin_module


def _as_triple(value) -> tuple[int, int, int]:
    if len(value) != 3:
        raise RuntimeError("crumpet_b200 MONAI patch only supports 3D Swin blocks")
    return tuple(int(v) for v in value)  # type: ignore[return-value]


def boundary_flags(dims, window_size, shift_size, device) -> torch.Tensor:
    """uint8 [nW]: 1 for windows whose shifted mask has a -100 entry.

    A window's mask is non-zero exactly when it is the last window along an
    axis with a non-zero shift (the roll seam); this is the closed form of
    the reference's ``mask.abs().amax(dim=1) > 0`` (monai_patch.py:177-178).
    """
    nd, nh, nw_ = (dims[a] // window_size[a] for a in range(3))
    idx = [torch.arange(n) for n in (nd, nh, nw_)]
    last = [(i == n - 1) & (shift_size[a] > 0) for a, (i, n) in enumerate(zip(idx, (nd, nh, nw_)))]
    flags = last[0][:, None, None] | last[1][None, :, None] | last[2][None, None, :]
    return flags.reshape(-1).to(torch.uint8).to(device, non_blocking=True)


def _block_fusion_enabled() -> bool:
    """Opt out of the fused norm/partition and unpartition/crop with CRUMPET_DISABLE_BLOCK_FUSION=1."""
    return os.environ.get("CRUMPET_DISABLE_BLOCK_FUSION", "0") != "1"


_FUSED_DTYPES = (torch.float32, torch.float16, torch.bfloat16)


def _no_grad_needed(*tensors) -> bool:
    return not torch.is_grad_enabled() or not any(t is not None and t.requires_grad for t in tensors)


def _norm_fusable(norm, x: torch.Tensor) -> bool:
    c = x.shape[-1]
    return (
        _block_fusion_enabled()
        and isinstance(norm, torch.nn.LayerNorm)
        and norm.weight is not None
        and norm.bias is not None
        and tuple(norm.normalized_shape) == (c,)
        and c % 8 == 0
        and c <= 768
        and x.is_cuda
        and x.dtype in _FUSED_DTYPES
        and _no_grad_needed(x, norm.weight, norm.bias)
    )


def _norm_out_dtype(x: torch.Tensor) -> torch.dtype:
    # Under autocast the norm runs in fp32 and the qkv Linear casts its input to
    # the autocast dtype: the fused op writes that dtype directly.
    if torch.is_autocast_enabled("cuda"):
        return torch.get_autocast_dtype("cuda")
    return x.dtype


def _crop_fusable(windows: torch.Tensor) -> bool:
    return (
        _block_fusion_enabled()
        and windows.is_cuda
        and windows.dtype in _FUSED_DTYPES
        and (windows.shape[-1] * windows.element_size()) % 4 == 0
        and _no_grad_needed(windows)
    )


def _attention_branch(self, x, mask_matrix, swin, residual=None, next_norm=None):
    """norm1 -> pad -> roll + partition -> attn -> unpartition + roll back -> crop
    (reference monai_patch.py:72-114), plus ``residual +`` when given.

    With ``next_norm`` (the block's norm2) the result is ``(out, next_norm(out))``
    when both come out of one fused kernel, else just ``out``."""
    b, d, h, w, c = x.shape
    window_size, shift_size = swin.get_window_size((d, h, w), self.window_size, self.shift_size)
    window_size = _as_triple(window_size)
    shift_size = _as_triple(shift_size)
    attn_mask = mask_matrix if any(s > 0 for s in shift_size) else None
    pad_d = (window_size[0] - d % window_size[0]) % window_size[0]
    pad_h = (window_size[1] - h % window_size[1]) % window_size[1]
    pad_w = (window_size[2] - w % window_size[2]) % window_size[2]
    if _norm_fusable(self.norm1, x):
        x_windows = norm_shift_partition_3d(x, self.norm1.weight, self.norm1.bias, self.norm1.eps,
                                            window_size, shift_size, _norm_out_dtype(x))
    else:
        xn = F.pad(self.norm1(x), (0, 0, 0, pad_w, 0, pad_h, 0, pad_d))
        x_windows = fused_shift_partition_3d(xn, window_size, shift_size)
    attn_windows = self.attn(x_windows, mask=attn_mask)
    if _crop_fusable(attn_windows):
        fuse_res = (residual is not None and residual.dtype == attn_windows.dtype
                    and residual.device == attn_windows.device and _no_grad_needed(residual))
        if (next_norm is not None and (fuse_res or residual is None)
                and _norm_fusable(next_norm, attn_windows)):
            return unshift_unpartition_crop_norm_3d(
                attn_windows, b, d, h, w, c, window_size, shift_size, next_norm.weight,
                next_norm.bias, next_norm.eps, residual=residual,
                norm_dtype=_norm_out_dtype(attn_windows))
        out = unshift_unpartition_crop_3d(attn_windows, b, d, h, w, c, window_size, shift_size,
                                          residual=residual if fuse_res else None)
        if residual is not None and not fuse_res:
            out = residual + out
        return out
    out = fused_unshift_unpartition_3d(attn_windows, b, d + pad_d, h + pad_h, w + pad_w, c,
                                       window_size, shift_size)
    if pad_d or pad_h or pad_w:
        out = out[:, :d, :h, :w, :].contiguous()
    return out if residual is None else residual + out


def _patched_forward_part1(original, swin):
    @functools.wraps(original)
    def forward_part1(self, x, mask_matrix):
        if x.dim() != 5:
            return original(self, x, mask_matrix)
        return _attention_branch(self, x, mask_matrix, swin)

    return forward_part1


def _patched_block_forward(original, swin):
    """``x + attention_branch(x)`` with the residual folded into the crop, then the MLP half.

    Inference only (eval mode, no activation checkpointing): there drop_path is
    the identity and the block is ``x = x + part1(x); x = x + mlp(norm2(x))``.  The
    crop kernel also writes ``norm2(x)`` when norm2 is a LayerNorm it can fuse.
    """

    @functools.wraps(original)
    def forward(self, x, mask_matrix):
        if (x.dim() != 5 or self.training or getattr(self, "use_checkpoint", False)
                or not _block_fusion_enabled()):
            return original(self, x, mask_matrix)
        norm2 = getattr(self, "norm2", None) if hasattr(self, "mlp") else None
        out = _attention_branch(self, x, mask_matrix, swin, residual=x, next_norm=norm2)
        if isinstance(out, tuple):
            x, x_norm2 = out
            return x + self.mlp(x_norm2)
        return out + self.forward_part2(out)

    return forward


def _linear(mod, x: torch.Tensor) -> torch.Tensor:
    """``mod(x)`` for the qkv / proj ``nn.Linear`` of a window attention; on the tensor-core
    GEMM (:func:`window_linear`) when it applies -- float16 / bfloat16 tokens already in the
    dtype the Linear would compute in (the autocast dtype, else the tokens' own), K = 48 or 96,
    N within :func:`window_linear_supported`, no gradient -- else through the module."""
    if (isinstance(mod, torch.nn.Linear)
            and x.is_cuda
            and x.dtype in (torch.float16, torch.bfloat16)
            and window_linear_supported(int(x.shape[-1]), int(mod.out_features))
            and _no_grad_needed(x, mod.weight, mod.bias)):
        compute = torch.get_autocast_dtype("cuda") if torch.is_autocast_enabled("cuda") else None
        if compute is None:
            compute = x.dtype if mod.weight.dtype == x.dtype else None
        if compute == x.dtype:
            return window_linear(x, mod.weight, mod.bias)
    return mod(x)


_TILES_ATTR = "_crumpet_bias_tiles"


def _bias_tiles(attn, n: int, head_dim: int, dtype: torch.dtype):
    """The module's prebuilt bias operands for windows of n tokens (see
    ``attention_bias_tiles``), cached on the module and rebuilt when the table or index
    tensor, its in-place version, n, the dtype or the scale changes; None where the
    tensor-core kernel does not run these windows (it then gathers the bias itself)."""
    if not tensor_core_attention(dtype, n, head_dim):
        return None
    table, index = attn.relative_position_bias_table, attn.relative_position_index
    key = (table.data_ptr(), table._version, index.data_ptr(), index._version, n, dtype,
           float(attn.scale), table.device)
    cached = getattr(attn, _TILES_ATTR, None)
    if cached is None or cached[0] != key:
        cached = (key, attention_bias_tiles(table, index, n, attn.scale, dtype))
        object.__setattr__(attn, _TILES_ATTR, cached)
    return cached[1]


def _patched_window_attention_forward(original):
    @functools.wraps(original)
    def forward(self, x, mask):
        if self.training or self.attn_drop.p != 0.0 or not _fused_attn_enabled():
            return original(self, x, mask)
        b, n, c = x.shape
        heads = self.num_heads
        head_dim = c // heads
        # The reference's own fallbacks (training, attention dropout, head_dim < 16;
        # torch-ext/crumpet/monai_patch.py:137-151), plus head dims no kernel here takes
        # (not a power of two, or above 256), where the reference's Triton compile fails.
        if head_dim < 16 or not head_dim_supported(head_dim) or not x.is_cuda:
            return original(self, x, mask)
        qkv = _linear(self.qkv, x)
        if qkv.dtype not in (torch.float32, torch.float16, torch.bfloat16):
            return original(self, x, mask)
        geometry = None if mask is None else getattr(mask, _GEOMETRY_ATTR, None)
        if mask is None or geometry is not None:
            # Fast path: packed qkv in, proj-ready [b, n, c] out, bias gathered and
            # shifted-window mask computed inside the kernel.
            num_windows, window_size, shift_size = geometry or ((1, 1, 1), (n, 1, 1), (0, 0, 0))
            out = swin_window_attention_qkv(
                qkv.view(b, n, 3, heads, head_dim), self.relative_position_bias_table,
                self.relative_position_index, num_windows, window_size, shift_size, self.scale,
                bias_tiles=_bias_tiles(self, n, head_dim, qkv.dtype))
            return self.proj_drop(_linear(self.proj, out))
        # A mask from elsewhere: dense mask path.
        qkv = qkv.reshape(b, n, 3, heads, head_dim).permute(2, 0, 3, 1, 4)
        q, k, v = qkv[0], qkv[1], qkv[2]
        index = self.relative_position_index[:n, :n].reshape(-1)
        rel_bias = self.relative_position_bias_table[index].reshape(n, n, -1)
        rel_bias = rel_bias.permute(2, 0, 1).contiguous().to(qkv.dtype)
        boundary = None
        if mask is not None:
            flags = getattr(mask, _BOUNDARY_ATTR, None)
            if flags is None:
                flags = (mask.reshape(mask.shape[0], -1).abs().amax(dim=1) > 0).to(torch.uint8)
            boundary = flags.repeat(b // mask.shape[0]) if b != mask.shape[0] else flags
            mask = mask.to(qkv.dtype)
        out = fused_swin_attention(q.contiguous(), k.contiguous(), v.contiguous(), rel_bias, mask,
                                   boundary, scale=self.scale)
        out = out.transpose(1, 2).reshape(b, n, c)
        return self.proj_drop(_linear(self.proj, out))

    return forward


def _merge_order(ds):
    """Neighbour order of a recognised patch-merging module, or None (then eager)."""
    name = type(ds).__name__
    if name == "PatchMergingV2" or (name == "PatchMerging"
                                    and type(ds).__module__ == "crumpet_b200.swin_unetr"):
        return PRODUCT_ORDER
    return None


def _merge_fusable(ds, x: torch.Tensor) -> bool:
    norm, red = getattr(ds, "norm", None), getattr(ds, "reduction", None)
    c = x.shape[-1]
    return (
        _block_fusion_enabled()
        and _merge_order(ds) is not None
        and isinstance(norm, torch.nn.LayerNorm)
        and norm.weight is not None
        and norm.bias is not None
        and tuple(norm.normalized_shape) == (8 * c,)
        and isinstance(red, torch.nn.Linear)
        and red.bias is None
        and red.in_features == 8 * c
        and c % 8 == 0
        and 8 * c <= 3072
        and x.is_cuda
        and x.dtype in _FUSED_DTYPES
        and _no_grad_needed(x, norm.weight, norm.bias, red.weight)
    )


def _merge_channels_first(ds, x: torch.Tensor) -> torch.Tensor:
    """Patch merging of channels-last ``x`` returned channels-first: the neighbour
    concatenation and LayerNorm in one kernel, then the reduction Linear computed as
    ``W @ X^T`` so its output is already [B, 2C, D', H', W'] (no permute copy)."""
    xm = patch_merge_norm_3d(x, ds.norm.weight, ds.norm.bias, ds.norm.eps, order=_merge_order(ds),
                             out_dtype=_norm_out_dtype(x))
    b, d2, h2, w2, c8 = xm.shape
    out = torch.matmul(ds.reduction.weight, xm.view(b, d2 * h2 * w2, c8).transpose(1, 2))
    return out.view(b, -1, d2, h2, w2)


def _patched_basic_layer_forward(original, swin):
    @functools.wraps(original)
    def forward(self, x):
        if x.dim() != 5:
            return original(self, x)
        b, c, d, h, w = x.shape
        window_size, shift_size = swin.get_window_size((d, h, w), self.window_size, self.shift_size)
        window_size = _as_triple(window_size)
        shift_size = _as_triple(shift_size)
        x = x.permute(0, 2, 3, 4, 1).contiguous()
        dims = tuple(-(-s // ws) * ws for s, ws in zip((d, h, w), window_size))
        attn_mask = compute_attn_mask_3d(*dims, window_size, shift_size, x.dtype, x.device)
        if getattr(attn_mask, _BOUNDARY_ATTR, None) is None:
            setattr(attn_mask, _BOUNDARY_ATTR, boundary_flags(dims, window_size, shift_size, x.device))
            num_windows = tuple(d // w for d, w in zip(dims, window_size))
            setattr(attn_mask, _GEOMETRY_ATTR, (num_windows, window_size, shift_size))
        for blk in self.blocks:
            x = blk(x, attn_mask)
        x = x.view(b, d, h, w, -1)
        if self.downsample is not None:
            if _merge_fusable(self.downsample, x):
                return _merge_channels_first(self.downsample, x)
            x = self.downsample(x)
        return x.permute(0, 4, 1, 2, 3).contiguous()

    return forward


def _proj_out_fusable(x: torch.Tensor) -> bool:
    return (
        _block_fusion_enabled()
        and x.dim() == 5
        and x.is_cuda
        and x.dtype in _FUSED_DTYPES
        and x.is_contiguous()
        and proj_out_lanes(int(x.shape[1])) > 0
        and _no_grad_needed(x)
    )


def _patched_proj_out(raw):
    """``proj_out(x, normalize)`` with the 5D LayerNorm branch as one kernel.

    MONAI's version (an instance method; a static method in the bundled network)
    permutes x to channels-last, applies ``F.layer_norm(x, [C])`` -- fp32 under
    autocast -- and permutes back; the result here has the same values up to fp32
    LayerNorm rounding, the same dtype and the same (channels-last) strides.
    """
    static = isinstance(raw, staticmethod)
    fn = raw.__func__ if static else raw

    @functools.wraps(fn)
    def proj_out(self, x, normalize=False):
        if normalize and _proj_out_fusable(x):
            out_dtype = torch.float32 if torch.is_autocast_enabled(x.device.type) else x.dtype
            return proj_out_norm_3d(x, out_dtype=out_dtype)
        return fn(x, normalize) if static else fn(self, x, normalize)

    return proj_out


def patch_monai_swin_unetr(swin_module=None) -> bool:
    """Install the patch; True on the installing call, False if already active."""
    if _STATE.get("patched"):
        return False
    swin = _load_swin(swin_module)
    _STATE.update(
        patched=True,
        swin=swin,
        forward_part1=swin.SwinTransformerBlock.forward_part1,
        block_forward=swin.SwinTransformerBlock.forward,
        basic_layer_forward=swin.BasicLayer.forward,
    )
    swin.SwinTransformerBlock.forward_part1 = _patched_forward_part1(_STATE["forward_part1"], swin)
    swin.SwinTransformerBlock.forward = _patched_block_forward(_STATE["block_forward"], swin)
    swin.BasicLayer.forward = _patched_basic_layer_forward(_STATE["basic_layer_forward"], swin)
    if _fused_attn_enabled():
        _STATE["window_attention_forward"] = swin.WindowAttention.forward
        swin.WindowAttention.forward = _patched_window_attention_forward(swin.WindowAttention.forward)
    trunk = getattr(swin, "SwinTransformer", None)
    if trunk is not None and hasattr(trunk, "proj_out"):
        _STATE["proj_out"] = (trunk, trunk.__dict__.get("proj_out", _MISSING))
        trunk.proj_out = _patched_proj_out(inspect.getattr_static(trunk, "proj_out"))
    return True


def unpatch_monai_swin_unetr() -> bool:
    """Restore the original methods; True if a patch was removed."""
    if not _STATE.get("patched"):
        return False
    swin = _STATE["swin"]
    swin.SwinTransformerBlock.forward_part1 = _STATE["forward_part1"]
    swin.SwinTransformerBlock.forward = _STATE["block_forward"]
    swin.BasicLayer.forward = _STATE["basic_layer_forward"]
    if "window_attention_forward" in _STATE:
        swin.WindowAttention.forward = _STATE["window_attention_forward"]
    if "proj_out" in _STATE:
        trunk, raw = _STATE["proj_out"]
        if raw is _MISSING:
            delattr(trunk, "proj_out")
        else:
            setattr(trunk, "proj_out", raw)
    _STATE.clear()
    return True
