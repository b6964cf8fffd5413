"""MONAI-architecture 3D Swin UNETR, eager PyTorch (MONAI is not a dependency).

The end-to-end workload of crumpet_b200 is MONAI's ``SwinUNETR`` (Hatamizadeh
et al., "Swin UNETR: Swin Transformers for Semantic Segmentation of Brain
Tumors in MRI Images", 2022) run by sliding-window inference.  MONAI is not
installed in this environment, so this module provides the same network,
written from the published architecture, with the class, method and
attribute names that crumpet's MONAI patch touches
(torch-ext/crumpet/monai_patch.py:55-63, 72-232):

* ``get_window_size``, ``SwinTransformerBlock.forward_part1``,
  ``BasicLayer.forward`` (channels-first in, channels-first out, builds the
  shifted-window mask on the padded grid), ``WindowAttention.forward`` with
  ``qkv``, ``proj``, ``scale``, ``attn_drop``, ``num_heads``,
  ``relative_position_bias_table`` and ``relative_position_index`` (built
  for the configured window and sliced ``[:n, :n]`` at run time, which
  reproduces MONAI's behaviour on windows clamped to a smaller volume).

Everything here is the eager (unpatched) path; ``patch_monai_swin_unetr(
crumpet_b200.swin_unetr)`` routes the three methods through the kernels.
Weights are randomly initialised (the benchmark uses synthetic data).
"""

from __future__ import annotations

import itertools
from typing import Sequence

import torch
import torch.nn as nn
import torch.nn.functional as F

from .reference import window_partition_reference, window_reverse_reference


def get_window_size(x_size, window_size, shift_size=None):
    """Clamp the window to the volume on each axis; no shift where clamped."""
    use_window = list(window_size)
    use_shift = list(shift_size) if shift_size is not None else None
    for i, size in enumerate(x_size):
        if size <= window_size[i]:
            use_window[i] = size
            if use_shift is not None:
                use_shift[i] = 0
    if use_shift is None:
        return tuple(use_window)
    return tuple(use_window), tuple(use_shift)


def window_partition(x: torch.Tensor, window_size) -> torch.Tensor:
    return window_partition_reference(x, window_size)


def window_reverse(windows: torch.Tensor, window_size, dims) -> torch.Tensor:
    return window_reverse_reference(windows, window_size, dims)


def compute_mask(dims, window_size, shift_size, device) -> torch.Tensor:
    """Shifted-window attention mask [nW, N, N] (float32, 0 / -100) on the padded grid."""
    d, h, w = dims
    label = torch.zeros((1, d, h, w, 1), device=device)
    count = 0
    cuts = [
        (slice(-window_size[a]), slice(-window_size[a], -shift_size[a]), slice(-shift_size[a], None))
        for a in range(3)
    ]
    for sd, sh, sw in itertools.product(*cuts):
        label[:, sd, sh, sw, :] = count
        count += 1
    lw = window_partition(label, window_size).squeeze(-1)
    diff = lw.unsqueeze(1) - lw.unsqueeze(2)
    return diff.masked_fill(diff != 0, -100.0).masked_fill(diff == 0, 0.0)


class MLPBlock(nn.Module):
    """Transformer MLP: Linear -> GELU -> Linear (dropout 0)."""

    def __init__(self, hidden_size: int, mlp_dim: int):
        super().__init__()
        self.linear1 = nn.Linear(hidden_size, mlp_dim)
        self.linear2 = nn.Linear(mlp_dim, hidden_size)
        self.fn = nn.GELU()

    def forward(self, x):
        return self.linear2(self.fn(self.linear1(x)))


class WindowAttention(nn.Module):
    """Window multi-head self-attention with a learned relative-position bias."""

    def __init__(self, dim: int, num_heads: int, window_size: Sequence[int], qkv_bias: bool = False,
                 attn_drop: float = 0.0, proj_drop: float = 0.0):
        super().__init__()
        self.dim = dim
        self.window_size = tuple(window_size)
        self.num_heads = num_heads
        head_dim = dim // num_heads
        self.scale = head_dim ** -0.5
        wd, wh, ww = self.window_size
        self.relative_position_bias_table = nn.Parameter(
            torch.zeros((2 * wd - 1) * (2 * wh - 1) * (2 * ww - 1), num_heads)
        )
        coords = torch.stack(torch.meshgrid(torch.arange(wd), torch.arange(wh), torch.arange(ww),
                                            indexing="ij")).flatten(1)
        rel = (coords[:, :, None] - coords[:, None, :]).permute(1, 2, 0).contiguous()
        rel[:, :, 0] += wd - 1
        rel[:, :, 1] += wh - 1
        rel[:, :, 2] += ww - 1
        index = rel[:, :, 0] * (2 * wh - 1) * (2 * ww - 1) + rel[:, :, 1] * (2 * ww - 1) + rel[:, :, 2]
        self.register_buffer("relative_position_index", index)
        self.qkv = nn.Linear(dim, dim * 3, bias=qkv_bias)
        self.attn_drop = nn.Dropout(attn_drop)
        self.proj = nn.Linear(dim, dim)
        self.proj_drop = nn.Dropout(proj_drop)
        nn.init.trunc_normal_(self.relative_position_bias_table, std=0.02)
        self.softmax = nn.Softmax(dim=-1)

    def forward(self, x, mask):
        b, n, c = x.shape
        qkv = self.qkv(x).reshape(b, n, 3, self.num_heads, c // self.num_heads).permute(2, 0, 3, 1, 4)
        q, k, v = qkv[0], qkv[1], qkv[2]
        q = q * self.scale
        attn = q @ k.transpose(-2, -1)
        bias = self.relative_position_bias_table[self.relative_position_index[:n, :n].reshape(-1)]
        attn = attn + bias.reshape(n, n, -1).permute(2, 0, 1).unsqueeze(0)
        if mask is not None:
            nw = mask.shape[0]
            attn = attn.view(b // nw, nw, self.num_heads, n, n) + mask.unsqueeze(1).unsqueeze(0)
            attn = attn.view(-1, self.num_heads, n, n)
        attn = self.attn_drop(self.softmax(attn)).to(v.dtype)
        x = (attn @ v).transpose(1, 2).reshape(b, n, c)
        return self.proj_drop(self.proj(x))


class SwinTransformerBlock(nn.Module):
    def __init__(self, dim: int, num_heads: int, window_size: Sequence[int], shift_size: Sequence[int],
                 mlp_ratio: float = 4.0, qkv_bias: bool = True, drop: float = 0.0,
                 attn_drop: float = 0.0, norm_layer=nn.LayerNorm):
        super().__init__()
        self.dim = dim
        self.num_heads = num_heads
        self.window_size = tuple(window_size)
        self.shift_size = tuple(shift_size)
        self.norm1 = norm_layer(dim)
        self.attn = WindowAttention(dim, num_heads, self.window_size, qkv_bias, attn_drop, drop)
        self.norm2 = norm_layer(dim)
        self.mlp = MLPBlock(dim, int(dim * mlp_ratio))

    def forward_part1(self, x, mask_matrix):
        x = self.norm1(x)
        b, d, h, w, c = x.shape
        window_size, shift_size = get_window_size((d, h, w), self.window_size, self.shift_size)
        pad_d = (window_size[0] - d % window_size[0]) % window_size[0]
        pad_h = (window_size[1] - h % window_size[1]) % window_size[1]
        pad_w = (window_size[2] - w % window_size[2]) % window_size[2]
        x = F.pad(x, (0, 0, 0, pad_w, 0, pad_h, 0, pad_d))
        _, dp, hp, wp, _ = x.shape
        if any(s > 0 for s in shift_size):
            shifted = torch.roll(x, shifts=tuple(-s for s in shift_size), dims=(1, 2, 3))
            attn_mask = mask_matrix
        else:
            shifted = x
            attn_mask = None
        windows = window_partition(shifted, window_size)
        attn_windows = self.attn(windows, mask=attn_mask)
        shifted = window_reverse(attn_windows, window_size, (b, dp, hp, wp))
        if any(s > 0 for s in shift_size):
            x = torch.roll(shifted, shifts=tuple(shift_size), dims=(1, 2, 3))
        else:
            x = shifted
        if pad_d or pad_h or pad_w:
            x = x[:, :d, :h, :w, :].contiguous()
        return x

    def forward_part2(self, x):
        return self.mlp(self.norm2(x))

    def forward(self, x, mask_matrix):
        x = x + self.forward_part1(x, mask_matrix)
        return x + self.forward_part2(x)


class PatchMerging(nn.Module):
    """2x2x2 neighbourhood concatenation (8C) -> LayerNorm -> Linear to 2C."""

    def __init__(self, dim: int, norm_layer=nn.LayerNorm, spatial_dims: int = 3):
        super().__init__()
        self.dim = dim
        self.norm = norm_layer(8 * dim)
        self.reduction = nn.Linear(8 * dim, 2 * dim, bias=False)

    def forward(self, x):
        b, d, h, w, c = x.shape
        if d % 2 or h % 2 or w % 2:
            x = F.pad(x, (0, 0, 0, w % 2, 0, h % 2, 0, d % 2))
        parts = [x[:, i::2, j::2, k::2, :] for i, j, k in itertools.product(range(2), repeat=3)]
        return self.reduction(self.norm(torch.cat(parts, -1)))


class BasicLayer(nn.Module):
    """One Swin stage: alternating unshifted / shifted blocks, then patch merging."""

    def __init__(self, dim: int, depth: int, num_heads: int, window_size: Sequence[int],
                 mlp_ratio: float = 4.0, qkv_bias: bool = True, drop: float = 0.0,
                 attn_drop: float = 0.0, norm_layer=nn.LayerNorm, downsample=None):
        super().__init__()
        self.window_size = tuple(window_size)
        self.shift_size = tuple(i // 2 for i in window_size)
        self.no_shift = tuple(0 for _ in window_size)
        self.depth = depth
        self.blocks = nn.ModuleList([
            SwinTransformerBlock(dim, num_heads, self.window_size,
                                 self.no_shift if i % 2 == 0 else self.shift_size,
                                 mlp_ratio, qkv_bias, drop, attn_drop, norm_layer)
            for i in range(depth)
        ])
        self.downsample = downsample(dim=dim, norm_layer=norm_layer) if downsample else None

    def forward(self, x):
        b, c, d, h, w = x.shape
        window_size, shift_size = get_window_size((d, h, w), self.window_size, self.shift_size)
        x = x.permute(0, 2, 3, 4, 1).contiguous()
        dp = -(-d // window_size[0]) * window_size[0]
        hp = -(-h // window_size[1]) * window_size[1]
        wp = -(-w // window_size[2]) * window_size[2]
        attn_mask = compute_mask((dp, hp, wp), window_size, shift_size, x.device)
        for blk in self.blocks:
            x = blk(x, attn_mask)
        x = x.view(b, d, h, w, -1)
        if self.downsample is not None:
            x = self.downsample(x)
        return x.permute(0, 4, 1, 2, 3).contiguous()


class PatchEmbed(nn.Module):
    def __init__(self, patch_size, in_chans: int, embed_dim: int):
        super().__init__()
        self.proj = nn.Conv3d(in_chans, embed_dim, kernel_size=patch_size, stride=patch_size)

    def forward(self, x):
        return self.proj(x)


class SwinTransformer(nn.Module):
    def __init__(self, in_chans: int, embed_dim: int, window_size, patch_size, depths, num_heads,
                 mlp_ratio: float = 4.0, qkv_bias: bool = True, drop_rate: float = 0.0,
                 attn_drop_rate: float = 0.0, norm_layer=nn.LayerNorm):
        super().__init__()
        self.patch_embed = PatchEmbed(patch_size, in_chans, embed_dim)
        self.pos_drop = nn.Dropout(drop_rate)
        for i in range(len(depths)):
            layer = BasicLayer(int(embed_dim * 2 ** i), depths[i], num_heads[i], window_size,
                               mlp_ratio, qkv_bias, drop_rate, attn_drop_rate, norm_layer,
                               PatchMerging)
            setattr(self, f"layers{i + 1}", nn.ModuleList([layer]))
        self.num_layers = len(depths)

    @staticmethod
    def proj_out(x, normalize: bool = False):
        if normalize:
            c = x.shape[1]
            x = F.layer_norm(x.permute(0, 2, 3, 4, 1), [c]).permute(0, 4, 1, 2, 3)
        return x

    def forward(self, x, normalize: bool = True):
        x0 = self.pos_drop(self.patch_embed(x))
        outs = [self.proj_out(x0, normalize)]
        h = x0
        for i in range(self.num_layers):
            h = getattr(self, f"layers{i + 1}")[0](h.contiguous())
            outs.append(self.proj_out(h, normalize))
        return outs


class UnetResBlock(nn.Module):
    """conv3 -> InstanceNorm -> LeakyReLU -> conv3 -> InstanceNorm, + (1x1 conv) residual."""

    def __init__(self, in_channels: int, out_channels: int, kernel_size: int = 3, stride: int = 1):
        super().__init__()
        pad = kernel_size // 2
        self.conv1 = nn.Conv3d(in_channels, out_channels, kernel_size, stride, pad, bias=False)
        self.conv2 = nn.Conv3d(out_channels, out_channels, kernel_size, 1, pad, bias=False)
        self.norm1 = nn.InstanceNorm3d(out_channels)
        self.norm2 = nn.InstanceNorm3d(out_channels)
        self.lrelu = nn.LeakyReLU(negative_slope=0.01, inplace=True)
        self.downsample = in_channels != out_channels or stride != 1
        if self.downsample:
            self.conv3 = nn.Conv3d(in_channels, out_channels, 1, stride, bias=False)
            self.norm3 = nn.InstanceNorm3d(out_channels)

    def forward(self, inp):
        out = self.lrelu(self.norm1(self.conv1(inp)))
        out = self.norm2(self.conv2(out))
        res = self.norm3(self.conv3(inp)) if self.downsample else inp
        return self.lrelu(out + res)


class UnetrBasicBlock(nn.Module):
    def __init__(self, in_channels: int, out_channels: int, kernel_size: int = 3, stride: int = 1):
        super().__init__()
        self.layer = UnetResBlock(in_channels, out_channels, kernel_size, stride)

    def forward(self, x):
        return self.layer(x)


class UnetrUpBlock(nn.Module):
    def __init__(self, in_channels: int, out_channels: int, kernel_size: int = 3, upsample: int = 2):
        super().__init__()
        self.transp_conv = nn.ConvTranspose3d(in_channels, out_channels, upsample, upsample, bias=False)
        self.conv_block = UnetResBlock(2 * out_channels, out_channels, kernel_size, 1)

    def forward(self, inp, skip):
        return self.conv_block(torch.cat((self.transp_conv(inp), skip), dim=1))


class UnetOutBlock(nn.Module):
    def __init__(self, in_channels: int, out_channels: int):
        super().__init__()
        self.conv = nn.Conv3d(in_channels, out_channels, 1, bias=True)

    def forward(self, x):
        return self.conv(x)


class SwinUNETR(nn.Module):
    """Swin UNETR for 3D segmentation (MONAI defaults: window 7, patch 2, instance norm)."""

    def __init__(self, in_channels: int = 1, out_channels: int = 14, feature_size: int = 48,
                 depths=(2, 2, 2, 2), num_heads=(3, 6, 12, 24), normalize: bool = True,
                 window_size=(7, 7, 7), patch_size=(2, 2, 2)):
        super().__init__()
        f = feature_size
        self.normalize = normalize
        self.swinViT = SwinTransformer(in_channels, f, window_size, patch_size, depths, num_heads)
        self.encoder1 = UnetrBasicBlock(in_channels, f)
        self.encoder2 = UnetrBasicBlock(f, f)
        self.encoder3 = UnetrBasicBlock(2 * f, 2 * f)
        self.encoder4 = UnetrBasicBlock(4 * f, 4 * f)
        self.encoder10 = UnetrBasicBlock(16 * f, 16 * f)
        self.decoder5 = UnetrUpBlock(16 * f, 8 * f)
        self.decoder4 = UnetrUpBlock(8 * f, 4 * f)
        self.decoder3 = UnetrUpBlock(4 * f, 2 * f)
        self.decoder2 = UnetrUpBlock(2 * f, f)
        self.decoder1 = UnetrUpBlock(f, f)
        self.out = UnetOutBlock(f, out_channels)

    def forward(self, x_in):
        hs = self.swinViT(x_in, self.normalize)
        enc0 = self.encoder1(x_in)
        enc1 = self.encoder2(hs[0])
        enc2 = self.encoder3(hs[1])
        enc3 = self.encoder4(hs[2])
        dec4 = self.encoder10(hs[4])
        dec3 = self.decoder5(dec4, hs[3])
        dec2 = self.decoder4(dec3, enc3)
        dec1 = self.decoder3(dec2, enc2)
        dec0 = self.decoder2(dec1, enc1)
        out = self.decoder1(dec0, enc0)
        return self.out(out)


__all__ = [
    "SwinUNETR", "SwinTransformer", "BasicLayer", "SwinTransformerBlock", "WindowAttention",
    "PatchMerging", "get_window_size", "compute_mask", "window_partition", "window_reverse",
]
