"""swin_window_attention_qkv (packed qkv in, proj-ready out, in-kernel bias gather,
on-chip shifted-window mask) against the float64 oracle, through the torch op and
the C ABI."""

from __future__ import annotations

import zlib

import numpy as np
import pytest
import torch

import inputs as I
from crumpet_b200 import _ops
from crumpet_b200.fused_attention import swin_window_attention_qkv
from helpers import DTYPE_CODE, ptr, stream_ptr
from oracle import attention as OA
from oracle import mechanics as OM

pytestmark = pytest.mark.gpu

# (name, grid dims (padded), window, shift, heads, batch repeats, configured window, dtype
#  [, head_dim (default 16)])
CASES = [
    ("shift_n343_h3", (14, 14, 14), (7, 7, 7), (3, 3, 3), 3, 2, (7, 7, 7), "float16"),
    ("shift_n343_h6_28", (28, 28, 28), (7, 7, 7), (3, 3, 3), 6, 1, (7, 7, 7), "float16"),
    ("noshift_n343_h3", (14, 14, 14), (7, 7, 7), (0, 0, 0), 3, 1, (7, 7, 7), "float16"),
    ("quirk_n216_h24", (6, 6, 6), (6, 6, 6), (0, 0, 0), 24, 3, (7, 7, 7), "float16"),
    ("mixed_shift", (14, 21, 7), (7, 7, 7), (3, 0, 2), 3, 1, (7, 7, 7), "float16"),
    ("shift_n64_h2", (8, 8, 8), (4, 4, 4), (2, 2, 2), 2, 2, (4, 4, 4), "float16"),
    ("shift_n343_bf16", (14, 14, 14), (7, 7, 7), (3, 3, 3), 3, 1, (7, 7, 7), "bfloat16"),
    ("shift_n343_h3_d32", (14, 14, 14), (7, 7, 7), (3, 3, 3), 3, 2, (7, 7, 7), "float16", 32),
    ("quirk_n216_h12_d32", (6, 6, 6), (6, 6, 6), (0, 0, 0), 12, 2, (7, 7, 7), "float16", 32),
    ("shift_n343_d32_bf16", (14, 14, 14), (7, 7, 7), (3, 3, 3), 2, 1, (7, 7, 7), "bfloat16", 32),
]


def make_case(case, dev, table_dtype=torch.float32, oracle=True):
    name, dims, ws, ss, H, reps, cfg, dtype = case[:8]
    hd = case[8] if len(case) > 8 else 16
    g = torch.Generator().manual_seed(zlib.crc32(name.encode()))
    nw = tuple(d // w for d, w in zip(dims, ws))
    nwin = nw[0] * nw[1] * nw[2]
    B, N = nwin * reps, ws[0] * ws[1] * ws[2]
    dt = getattr(torch, dtype)
    qkv = torch.randn((B, N, 3, H, hd), generator=g).to(dt)
    ncfg = cfg[0] * cfg[1] * cfg[2]
    table = (torch.randn(((2 * cfg[0] - 1) * (2 * cfg[1] - 1) * (2 * cfg[2] - 1), H), generator=g)
             * 0.5).to(table_dtype)
    index = torch.from_numpy(OA.relative_position_index(cfg)).long()
    assert index.shape == (ncfg, ncfg)
    # oracle inputs: bias rounded to the activation dtype, as the reference does
    bias = torch.from_numpy(OA.gather_bias(table.float().numpy(), index.numpy(), N)).to(dt)
    inputs = (qkv.to(dev), table.to(dev), index.to(dev), nw, ws, ss)
    if not oracle:
        return inputs, None
    mask = None
    if any(ss):
        mask = OM.attn_mask(*dims, ws, ss, np.float32)
    q, k, v = (qkv[:, :, i].permute(0, 2, 1, 3) for i in range(3))
    want = OA.window_attention(q.float().numpy(), k.float().numpy(), v.float().numpy(),
                               bias.float().numpy(), mask)
    want = np.transpose(want, (0, 2, 1, 3)).reshape(B, N, H * hd)
    return inputs, want


def tol(dtype):
    return 1.6e-2 if dtype == torch.bfloat16 else 2e-3


@pytest.mark.parametrize("case", CASES, ids=[c[0] for c in CASES])
def test_packed_attention_matches_oracle(case, cuda_device):
    (qkv, table, index, nw, ws, ss), want = make_case(case, cuda_device)
    out = swin_window_attention_qkv(qkv, table, index, nw, ws, ss, qkv.shape[-1] ** -0.5)
    torch.cuda.synchronize()
    err = np.abs(out.float().cpu().numpy() - want).max()
    assert err <= tol(qkv.dtype), err
    assert _ops.capi().crumpet_device_status(1) == 0


def test_packed_attention_capi_fp16_table(cuda_device):
    case = CASES[0]
    (qkv, table, index, nw, ws, ss), want = make_case(case, cuda_device, torch.float16)
    B, N, _, H, D = qkv.shape
    out = torch.empty((B, N, H * D), dtype=qkv.dtype, device=cuda_device)
    rc = _ops.capi().crumpet_swin_window_attention_qkv(
        ptr(out), ptr(qkv), ptr(table), 0, table.shape[0], ptr(index), index.shape[1], *nw, *ws, *ss,
        DTYPE_CODE[qkv.dtype], B, H, N, D, 0.25, stream_ptr())
    assert rc == 0, _ops.last_error()
    torch.cuda.synchronize()
    assert np.abs(out.float().cpu().numpy() - want).max() <= 2e-3


def test_packed_matches_dense_kernel(cuda_device):
    # the packed/analytic kernel and the dense-mask kernel agree
    import crumpet_b200 as crumpet

    case = CASES[0]
    (qkv, table, index, nw, ws, ss), _ = make_case(case, cuda_device)
    B, N, _, H, D = qkv.shape
    packed = swin_window_attention_qkv(qkv, table, index, nw, ws, ss, 0.25)
    bias = table[index[:N, :N].reshape(-1)].reshape(N, N, H).permute(2, 0, 1).contiguous().half()
    mask = crumpet.compute_attn_mask_3d(14, 14, 14, ws, ss, torch.float16, cuda_device)
    q, k, v = (qkv[:, :, i].permute(0, 2, 1, 3).contiguous() for i in range(3))
    dense = crumpet.fused_swin_attention(q, k, v, bias, mask, None, 0.25)
    dense = dense.transpose(1, 2).reshape(B, N, H * D)
    assert (packed.float() - dense.float()).abs().max().item() <= 2e-3


def test_cfg3_full_size_sampled_windows(cuda_device):
    """The BASELINE attention workload at full size: 2744 windows x 3 heads of a 98^3 stage
    (ws 7, ss 3), through the dense-mask kernel (mask [2744, 343, 343] + boundary flags) and
    the packed on-chip-mask kernel.  Sampled interior and boundary windows against the float64
    oracle; the two kernels against each other on every window; no device error."""
    import crumpet_b200 as crumpet
    from crumpet_b200.monai_patch import boundary_flags

    g = torch.Generator().manual_seed(33)
    B, N, H, D = 2744, 343, 3, 16
    ws, ss, nw = (7, 7, 7), (3, 3, 3), (14, 14, 14)
    qkv = torch.randn((B, N, 3, H, D), generator=g).half().to(cuda_device)
    table = (0.5 * torch.randn((13 ** 3, H), generator=g)).to(cuda_device)
    index = torch.from_numpy(I.relative_index(ws)).to(cuda_device)
    scale = D ** -0.5
    packed = swin_window_attention_qkv(qkv, table, index, nw, ws, ss, scale)
    bias = table[index.reshape(-1)].reshape(N, N, H).permute(2, 0, 1).contiguous().half()
    mask = crumpet.compute_attn_mask_3d(98, 98, 98, ws, ss, torch.float16, cuda_device)
    boundary = boundary_flags((98, 98, 98), ws, ss, cuda_device)
    q, k, v = (qkv[:, :, i].permute(0, 2, 1, 3).contiguous() for i in range(3))
    dense = crumpet.fused_swin_attention(q, k, v, bias, mask, boundary, scale)
    torch.cuda.synchronize()
    assert _ops.capi().crumpet_device_status(1) == 0
    dense_bnc = dense.transpose(1, 2).reshape(B, N, H * D)
    assert (packed.float() - dense_bnc.float()).abs().max().item() <= 2e-3
    # interior windows and windows on the roll seam of one, two and three axes
    sel = [0, 1, 100, 1000, 13, 13 * 14, 13 * 196, 13 + 13 * 14, 2743]
    assert all(boundary[s].item() == (1 if s in (13, 182, 2548, 195, 2743) else 0) for s in sel)
    want = OA.window_attention(q[sel].float().cpu().numpy(), k[sel].float().cpu().numpy(),
                               v[sel].float().cpu().numpy(), bias.float().cpu().numpy(),
                               mask[sel].float().cpu().numpy(), None, scale)
    assert np.abs(dense[sel].float().cpu().numpy() - want).max() <= 2e-3
    got = packed[sel].reshape(len(sel), N, H, D).permute(0, 2, 1, 3)
    assert np.abs(got.float().cpu().numpy() - want).max() <= 2e-3


def test_out_of_range_index_is_flagged_not_read(cuda_device):
    """A relative-position index value outside the bias table is not read: its bias is
    taken as 0, the device error word gets bit 2, and check_device_status raises."""
    import crumpet_b200 as crumpet

    (qkv, table, index, nw, ws, ss), _ = make_case(CASES[0], cuda_device)
    bad = index.clone()
    bad[5, 7] = table.shape[0]
    bad[100, 3] = -1
    bad[200, 300] = -12345
    assert crumpet.device_status(clear=True) == 0
    out = swin_window_attention_qkv(qkv, table, bad, nw, ws, ss, 0.25)
    torch.cuda.synchronize()
    assert torch.isfinite(out).all()
    assert crumpet.device_status() == 2
    with pytest.raises(RuntimeError, match="device error 2"):
        crumpet.check_device_status()
    assert crumpet.device_status() == 0
    # the same call with the valid index leaves the word clear
    swin_window_attention_qkv(qkv, table, index, nw, ws, ss, 0.25)
    crumpet.check_device_status()


TILE_CASES = [c for c in CASES if c[7] != "float32" and c[0] != "shift_n64_h2"] + [
    ("stage2_n343_h12_b8", (14, 14, 14), (7, 7, 7), (3, 3, 3), 12, 8, (7, 7, 7), "float16"),
    # 686 windows x 3 heads: enough windows that, with prebuilt tiles, the CTAs left over by
    # the 9 (head, query tile) pairs take the last 10 windows of every pair (spanning several
    # pairs each), while the gather path leaves them idle -- the outputs must still agree
    ("helpers_n343_h3_b686", (49, 49, 49), (7, 7, 7), (3, 3, 3), 3, 2, (7, 7, 7), "float16"),
]


@pytest.mark.parametrize("case", TILE_CASES, ids=[c[0] for c in TILE_CASES])
def test_prebuilt_bias_tiles_equal_the_gather(case, cuda_device):
    """The per-module bias operands built once give bit-identical outputs to the per-CTA
    gather (same operand image, same kernel arithmetic)."""
    from crumpet_b200.fused_attention import attention_bias_tiles

    (qkv, table, index, nw, ws, ss), _ = make_case(case, cuda_device, oracle=False)
    B, N, _, H, D = qkv.shape
    scale = D ** -0.5
    tiles = attention_bias_tiles(table, index, N, scale, qkv.dtype)
    gathered = swin_window_attention_qkv(qkv, table, index, nw, ws, ss, scale)
    tiled = swin_window_attention_qkv(qkv, table, index, nw, ws, ss, scale, bias_tiles=tiles)
    torch.cuda.synchronize()
    assert torch.equal(tiled, gathered)
    # through the C ABI
    out = torch.empty_like(tiled)
    rc = _ops.capi().crumpet_swin_window_attention_qkv_tiles(
        ptr(out), ptr(qkv), ptr(tiles), *nw, *ws, *ss, DTYPE_CODE[qkv.dtype], B, H, N, D, scale,
        stream_ptr())
    assert rc == 0, _ops.last_error()
    torch.cuda.synchronize()
    assert torch.equal(out, gathered)
    assert _ops.capi().crumpet_device_status(1) == 0


def test_bias_tile_cache_follows_the_table(cuda_device):
    """The patched WindowAttention caches its bias tiles and rebuilds them when the
    table changes in place (as load_state_dict does)."""
    import crumpet_b200 as crumpet
    from crumpet_b200 import monai_patch, swin_unetr

    torch.manual_seed(0)
    attn = swin_unetr.WindowAttention(48, 3, (7, 7, 7), qkv_bias=True).to(cuda_device).eval()
    x = torch.randn((8, 343, 48), device=cuda_device).half()
    crumpet.patch_monai_swin_unetr(swin_unetr)
    try:
        with torch.no_grad(), torch.autocast("cuda", dtype=torch.float16):
            first = attn(x, None)
            tiles = getattr(attn, monai_patch._TILES_ATTR)[1]
            again = attn(x, None)
            assert getattr(attn, monai_patch._TILES_ATTR)[1] is tiles  # reused
            attn.relative_position_bias_table.add_(0.5)
            changed = attn(x, None)
            assert getattr(attn, monai_patch._TILES_ATTR)[1] is not tiles
    finally:
        crumpet.unpatch_monai_swin_unetr()
    with torch.no_grad(), torch.autocast("cuda", dtype=torch.float16):
        eager = attn(x, None)
    assert torch.equal(first, again)
    assert not torch.equal(first, changed)
    assert (changed.float() - eager.float()).abs().max().item() < 2e-2


def test_bias_tiles_reject_the_simt_domain(cuda_device):
    from crumpet_b200.fused_attention import attention_bias_tiles

    table = torch.randn((13 ** 3, 2), device=cuda_device)
    index = torch.from_numpy(OA.relative_position_index((7, 7, 7))).long().to(cuda_device)
    with pytest.raises(ValueError, match="352"):
        attention_bias_tiles(table, index, 512, 0.25, torch.float16)
    with pytest.raises(ValueError):
        attention_bias_tiles(table, index, 343, 0.25, torch.float32)
