"""LayerNorm + pad + roll + partition and unpartition + crop (+ residual) on the GPU.

Pinned to the outputs of the reference's own patched ``forward_part1``
(tests/golden/block_ref.npz, monai_patch.py:72-114), then checked against the
float64 oracle for every input/output dtype pair at the Swin UNETR stage shapes,
bit-exact for the unpartition + crop (a pure gather) and for the residual add
(torch's fp32-then-round add), through the torch ops and the C ABI, and inside a
patched Swin block against the unfused glue.
"""

from __future__ import annotations

import json
from pathlib import Path

import numpy as np
import pytest
import torch

import crumpet_b200 as crumpet
import inputs as I
from crumpet_b200 import _ops, monai_patch, swin_unetr
from helpers import DTYPE_CODE, ptr, sha, stream_ptr
from oracle import block as OB
from oracle import mechanics as OM

pytestmark = pytest.mark.gpu
GOLDEN = Path(__file__).resolve().parent / "golden"
MANIFEST = json.loads((GOLDEN / "manifest.json").read_text())
BLOCK_REF = np.load(GOLDEN / "block_ref.npz")
DTYPES = [torch.float32, torch.float16, torch.bfloat16]
# (B, D, H, W, C, configured window, shift): the four Swin UNETR stages of a
# 96^3 ROI (48^3 pads to 49^3, 24^3 to 28^3, 12^3 to 14^3; 6^3 clamps to a 6^3
# window without shift) and a ragged volume
STAGES = [
    (2, 48, 48, 48, 48, (7, 7, 7), (3, 3, 3)),
    (2, 24, 24, 24, 96, (7, 7, 7), (3, 3, 3)),
    (4, 12, 12, 12, 192, (7, 7, 7), (3, 3, 3)),
    (4, 6, 6, 6, 384, (7, 7, 7), (3, 3, 3)),
    (3, 17, 5, 23, 64, (7, 7, 7), (3, 3, 3)),
    (2, 4, 4, 4, 768, (7, 7, 7), (3, 3, 3)),  # last stage of a feature-size-96 network
]
STAGE_IDS = ["s48_C48", "s24_C96", "s12_C192", "s6_C384", "ragged_C64", "s4_C768"]


# |got - want| <= rel * |want| + abs: one rounding to the output type (fp16/bf16:
# within one unit in the last place) on top of the fp32 arithmetic's error
TOL = {torch.float32: (1e-6, 1e-5), torch.float16: (2.0**-10, 1e-5),
       torch.bfloat16: (2.0**-7, 1e-5)}


def _valid_token_mask(B, D, H, W, ws, ss) -> np.ndarray:
    ones = np.ones((B, D, H, W, 1), dtype=np.float64)
    Dp, Hp, Wp = OB.padded_dims((D, H, W), ws)
    padded = np.zeros((B, Dp, Hp, Wp, 1))
    padded[:, :D, :H, :W] = ones
    return OM.shift_partition(padded, ws, ss)[..., 0] > 0


def _stage_inputs(B, D, H, W, C, seed, dtype):
    x = (I.randn(seed, (B, D, H, W, C), "float32") * 1.5 + 0.25).to(dtype)
    w = 1.0 + 0.2 * I.randn(seed + 1, (C,), "float32")
    b = 0.1 * I.randn(seed + 2, (C,), "float32")
    return x, w, b


@pytest.mark.parametrize("case", I.BLOCK_CASES, ids=[c[0] for c in I.BLOCK_CASES])
def test_norm_partition_matches_reference_forward_part1(case, cuda_device):
    name, shape, window, shift, _ = case
    x, w, b, eps = I.block_inputs(case)
    ws, ss = OB.window_geometry(shape[1:4], window, shift)
    win = crumpet.norm_shift_partition_3d(x.to(cuda_device), w.to(cuda_device), b.to(cuda_device),
                                          eps, ws, ss)
    ref = torch.from_numpy(BLOCK_REF[name + ".windows"])
    assert list(win.shape) == list(ref.shape)
    torch.testing.assert_close(win.cpu(), ref, rtol=0, atol=2e-5)
    valid = torch.from_numpy(_valid_token_mask(shape[0], *shape[1:4], ws, ss))
    assert torch.count_nonzero(win.cpu()[~valid]) == 0  # padded tokens are exact zeros
    attn = I.block_attn_output(case, tuple(win.shape)).to(cuda_device)
    out = crumpet.unshift_unpartition_crop_3d(attn, *shape, ws, ss)
    assert sha(out) == MANIFEST["block"][name]["out_sha256"]


@pytest.mark.parametrize("out_dtype", DTYPES, ids=["out_f32", "out_f16", "out_bf16"])
@pytest.mark.parametrize("in_dtype", DTYPES, ids=["in_f32", "in_f16", "in_bf16"])
@pytest.mark.parametrize("stage", STAGES, ids=STAGE_IDS)
def test_norm_partition_matches_oracle(stage, in_dtype, out_dtype, cuda_device):
    B, D, H, W, C, window, shift = stage
    if C >= 192 and (in_dtype, out_dtype) not in ((torch.float16, torch.float16),
                                                  (torch.float32, torch.bfloat16)):
        pytest.skip("dtype matrix covered at the smaller stages")
    ws, ss = OB.window_geometry((D, H, W), window, shift)
    x, w, b = _stage_inputs(B, D, H, W, C, 60 + C, in_dtype)
    got = crumpet.norm_shift_partition_3d(x.to(cuda_device), w.to(cuda_device), b.to(cuda_device),
                                          1e-5, ws, ss, out_dtype)
    torch.cuda.synchronize()
    want = OB.norm_shift_partition(x.double().numpy(), w.numpy(), b.numpy(), 1e-5, ws, ss)
    assert tuple(got.shape) == want.shape
    g = got.double().cpu().numpy()
    rel, atol = TOL[out_dtype]
    bad = np.abs(g - want) > np.abs(want) * rel + atol
    assert not bad.any(), (np.abs(g - want).max(), int(bad.sum()))
    if out_dtype != torch.float32:
        exact = (got.cpu() == torch.from_numpy(want).to(out_dtype)).float().mean().item()
        assert exact >= 0.995
    valid = torch.from_numpy(_valid_token_mask(B, D, H, W, ws, ss))
    assert torch.count_nonzero(got.cpu()[~valid]) == 0


@pytest.mark.parametrize("dtype", DTYPES, ids=["f32", "f16", "bf16"])
@pytest.mark.parametrize("stage", STAGES, ids=STAGE_IDS)
def test_unpartition_crop_residual_bit_exact(stage, dtype, cuda_device):
    B, D, H, W, C, window, shift = stage
    ws, ss = OB.window_geometry((D, H, W), window, shift)
    (Dp, Hp, Wp), nw, n = crumpet.block_fusion.padded_geometry(D, H, W, ws)
    windows = I.randn(70 + C, (B * nw, n, C), "float32").to(dtype)
    residual = I.randn(71 + C, (B, D, H, W, C), "float32").to(dtype)
    raw = windows.view(torch.int16) if dtype == torch.bfloat16 else windows
    crop = torch.from_numpy(OB.unshift_unpartition_crop(raw.numpy(), B, D, H, W, C, ws, ss))
    crop = crop.view(torch.bfloat16) if dtype == torch.bfloat16 else crop
    wd, rd = windows.to(cuda_device), residual.to(cuda_device)
    out = crumpet.unshift_unpartition_crop_3d(wd, B, D, H, W, C, ws, ss)
    assert torch.equal(out.cpu(), crop)
    out_r = crumpet.unshift_unpartition_crop_3d(wd, B, D, H, W, C, ws, ss, residual=rd)
    assert torch.equal(out_r.cpu(), residual + crop)  # torch's add: fp32 then one rounding
    assert torch.equal(out_r, rd + out)


def test_block_fusion_through_the_c_abi(cuda_device):
    B, D, H, W, C = 2, 13, 10, 9, 48
    ws, ss = (7, 7, 7), (3, 3, 3)
    x, w, b = _stage_inputs(B, D, H, W, C, 81, torch.float16)
    xd, wd, bd = x.to(cuda_device), w.to(cuda_device), b.to(cuda_device)
    want = crumpet.norm_shift_partition_3d(xd, wd, bd, 1e-5, ws, ss, torch.float16)
    out = torch.empty_like(want)
    lib = _ops.capi()
    rc = lib.crumpet_norm_shift_partition_3d(ptr(out), DTYPE_CODE[torch.float16], ptr(xd),
                                             DTYPE_CODE[torch.float16], ptr(wd), ptr(bd), 1e-5, B, D,
                                             H, W, C, *ws, *ss, stream_ptr())
    assert rc == 0, _ops.last_error()
    assert torch.equal(out, want)
    res = torch.randn(B, D, H, W, C, device=cuda_device).half()
    back = torch.empty_like(res)
    rc = lib.crumpet_unshift_unpartition_crop_3d(ptr(back), ptr(out), ptr(res),
                                                 DTYPE_CODE[torch.float16], B, D, H, W, C, *ws, *ss,
                                                 stream_ptr())
    assert rc == 0, _ops.last_error()
    assert torch.equal(back, res + crumpet.unshift_unpartition_crop_3d(out, B, D, H, W, C, ws, ss))


def test_batch_entries_match_single_entry_launches(cuda_device):
    # the bench's sliding-window batch: 8 ROIs at the first stage
    B, D, H, W, C = 8, 48, 48, 48, 48
    ws, ss = (7, 7, 7), (3, 3, 3)
    g = torch.Generator(device=cuda_device).manual_seed(5)
    x = torch.randn((B, D, H, W, C), device=cuda_device, generator=g).half()
    w = torch.ones(C, device=cuda_device)
    b = torch.zeros(C, device=cuda_device)
    win = crumpet.norm_shift_partition_3d(x, w, b, 1e-5, ws, ss, torch.float16)
    for e in (0, 5, 7):
        one = crumpet.norm_shift_partition_3d(x[e:e + 1], w, b, 1e-5, ws, ss, torch.float16)
        assert torch.equal(win[e * 343:(e + 1) * 343], one)
    back = crumpet.unshift_unpartition_crop_3d(win, B, D, H, W, C, ws, ss, residual=x)
    for e in (0, 7):
        one = crumpet.unshift_unpartition_crop_3d(win[e * 343:(e + 1) * 343], 1, D, H, W, C, ws,
                                                  ss, residual=x[e:e + 1])
        assert torch.equal(back[e:e + 1], one)


@pytest.mark.parametrize("shift", [(0, 0, 0), (3, 3, 3)], ids=["noshift", "shift"])
def test_patched_block_matches_unfused_glue(shift, cuda_device, monkeypatch):
    """A Swin block under fp16 autocast: fused glue vs the reference-style glue
    (norm1 -> pad -> partition op ... unpartition op -> crop -> residual add)
    with the same attention kernel."""
    torch.manual_seed(0)
    blk = swin_unetr.SwinTransformerBlock(48, 3, (7, 7, 7), shift).to(cuda_device).eval()
    x = torch.randn(2, 24, 24, 24, 48, device=cuda_device).half()
    dims = (28, 28, 28)
    mask = crumpet.compute_attn_mask_3d(*dims, (7, 7, 7), (3, 3, 3), torch.float16,
                                        cuda_device).clone()
    crumpet.patch_monai_swin_unetr(swin_unetr)
    try:
        setattr(mask, monai_patch._GEOMETRY_ATTR, ((4, 4, 4), (7, 7, 7), (3, 3, 3)))
        with torch.no_grad(), torch.autocast("cuda", dtype=torch.float16):
            fused = blk(x, mask)
            monkeypatch.setenv("CRUMPET_DISABLE_BLOCK_FUSION", "1")
            unfused = blk(x, mask)
        torch.cuda.synchronize()
    finally:
        crumpet.unpatch_monai_swin_unetr()
    assert fused.dtype == unfused.dtype == torch.float16
    diff = (fused.float() - unfused.float()).abs()
    # only the LayerNorm's last-place rounding differs between the two glues
    assert diff.max().item() < 2e-2 and diff.mean().item() < 1e-4


@pytest.mark.parametrize("norm_dtype", [torch.float16, torch.float32], ids=["norm_f16", "norm_f32"])
@pytest.mark.parametrize("dtype", DTYPES, ids=["f32", "f16", "bf16"])
@pytest.mark.parametrize("stage", STAGES, ids=STAGE_IDS)
def test_unpartition_crop_residual_norm(stage, dtype, norm_dtype, cuda_device):
    """The residual add of the attention half and norm2 in the crop pass: ``out``
    bit-exact (torch's add), ``normed`` the float64 LayerNorm of ``out`` within
    one unit in the last place."""
    B, D, H, W, C, window, shift = stage
    if C >= 192 and dtype != torch.float16:
        pytest.skip("dtype matrix covered at the smaller stages")
    ws, ss = OB.window_geometry((D, H, W), window, shift)
    (Dp, Hp, Wp), nw, n = crumpet.block_fusion.padded_geometry(D, H, W, ws)
    windows = I.randn(90 + C, (B * nw, n, C), "float32").to(dtype)
    residual = I.randn(91 + C, (B, D, H, W, C), "float32").to(dtype)
    w = 1.0 + 0.2 * I.randn(92 + C, (C,), "float32")
    b = 0.1 * I.randn(93 + C, (C,), "float32")
    raw = windows.view(torch.int16) if dtype == torch.bfloat16 else windows
    crop = torch.from_numpy(OB.unshift_unpartition_crop(raw.numpy(), B, D, H, W, C, ws, ss))
    crop = crop.view(torch.bfloat16) if dtype == torch.bfloat16 else crop
    out, normed = crumpet.unshift_unpartition_crop_norm_3d(
        windows.to(cuda_device), B, D, H, W, C, ws, ss, w.to(cuda_device), b.to(cuda_device), 1e-5,
        residual=residual.to(cuda_device), norm_dtype=norm_dtype)
    torch.cuda.synchronize()
    want_out = residual + crop
    assert torch.equal(out.cpu(), want_out)
    want = OB.layer_norm(want_out.double().numpy(), w.numpy(), b.numpy(), 1e-5)
    g = normed.double().cpu().numpy()
    rel, atol = TOL[norm_dtype]
    bad = np.abs(g - want) > np.abs(want) * rel + atol
    assert not bad.any(), (np.abs(g - want).max(), int(bad.sum()))


def test_unpartition_crop_norm_through_the_c_abi(cuda_device):
    B, D, H, W, C = 2, 13, 10, 9, 48
    ws, ss = (7, 7, 7), (3, 3, 3)
    (Dp, Hp, Wp), nw, n = crumpet.block_fusion.padded_geometry(D, H, W, ws)
    windows = torch.randn((B * nw, n, C), device=cuda_device).half()
    res = torch.randn((B, D, H, W, C), device=cuda_device).half()
    w = torch.rand(C, device=cuda_device) + 0.5
    b = torch.randn(C, device=cuda_device) * 0.1
    want_out, want_norm = crumpet.unshift_unpartition_crop_norm_3d(windows, B, D, H, W, C, ws, ss, w,
                                                                   b, 1e-5, residual=res)
    out, normed = torch.empty_like(res), torch.empty_like(res)
    rc = _ops.capi().crumpet_unshift_unpartition_crop_norm_3d(
        ptr(out), ptr(normed), DTYPE_CODE[torch.float16], ptr(windows), ptr(res),
        DTYPE_CODE[torch.float16], ptr(w), ptr(b), 1e-5, B, D, H, W, C, *ws, *ss, stream_ptr())
    assert rc == 0, _ops.last_error()
    assert torch.equal(out, want_out) and torch.equal(normed, want_norm)
    # norm2 of the block, computed the eager way, agrees to fp16 rounding
    eager = torch.nn.functional.layer_norm(want_out.float(), (C,), w, b, 1e-5).half()
    assert (normed.float() - eager.float()).abs().max().item() <= 4e-3


MERGE_CASES = [  # (B, D, H, W, C)
    (8, 48, 48, 48, 48),   # stage 1 of an 8-ROI batch: 8C = 384
    (2, 24, 24, 24, 96),   # stage 2: 8C = 768
    (2, 7, 6, 5, 16),      # odd dims: zero-padded neighbours
    (8, 12, 12, 12, 192),  # stage 3: 8C = 1536 (32 lanes, 6 groups each)
    (8, 6, 6, 6, 384),     # stage 4: 8C = 3072 (32 lanes, 12 groups each)
    (2, 5, 7, 3, 384),     # wide and odd
]


@pytest.mark.parametrize("out_dtype", [torch.float16, torch.float32], ids=["out_f16", "out_f32"])
@pytest.mark.parametrize("in_dtype", [torch.float16, torch.float32], ids=["in_f16", "in_f32"])
@pytest.mark.parametrize("case", MERGE_CASES,
                         ids=["s48_C48", "s24_C96", "odd_C16", "s12_C192", "s6_C384", "odd_C384"])
def test_patch_merge_norm_matches_eager(case, in_dtype, out_dtype, cuda_device):
    """Neighbour concatenation + LayerNorm of patch merging against the module's eager
    F.pad + strided slices + cat + layer_norm, in float64."""
    B, D, H, W, C = case
    x = (I.randn(100 + C, case, "float32") * 1.5 + 0.25).to(in_dtype)
    w = 1.0 + 0.2 * I.randn(101 + C, (8 * C,), "float32")
    b = 0.1 * I.randn(102 + C, (8 * C,), "float32")
    got = crumpet.patch_merge_norm_3d(x.to(cuda_device), w.to(cuda_device), b.to(cuda_device), 1e-5,
                                      out_dtype=out_dtype)
    torch.cuda.synchronize()
    xp = torch.nn.functional.pad(x.double(), (0, 0, 0, W % 2, 0, H % 2, 0, D % 2))
    cat = torch.cat([xp[:, i::2, j::2, k::2, :] for i, j, k in crumpet.block_fusion.PRODUCT_ORDER], -1)
    want = OB.layer_norm(cat.numpy(), w.numpy(), b.numpy(), 1e-5)
    g = got.double().cpu().numpy()
    assert g.shape == want.shape
    rel, atol = TOL[out_dtype]
    bad = np.abs(g - want) > np.abs(want) * rel + atol
    assert not bad.any(), (np.abs(g - want).max(), int(bad.sum()))


def test_patch_merge_custom_order_and_c_abi(cuda_device):
    B, D, H, W, C = 1, 6, 6, 6, 8
    order = [(1, 1, 1), (0, 0, 0), (1, 0, 0), (0, 1, 0), (0, 0, 1), (1, 1, 0), (1, 0, 1), (0, 1, 1)]
    x = torch.randn((B, D, H, W, C), device=cuda_device).half()
    w = torch.ones(8 * C, device=cuda_device)
    b = torch.zeros(8 * C, device=cuda_device)
    got = crumpet.patch_merge_norm_3d(x, w, b, 1e-5, order=order)
    cat = torch.cat([x[:, i::2, j::2, k::2, :] for i, j, k in order], -1).float()
    want = torch.nn.functional.layer_norm(cat, (8 * C,), w, b, 1e-5).half()
    assert (got.float() - want.float()).abs().max().item() <= 4e-3
    out = torch.empty_like(got)
    import ctypes
    codes = (ctypes.c_int * 8)(*[i | (j << 1) | (k << 2) for i, j, k in order])
    rc = _ops.capi().crumpet_patch_merge_norm_3d(ptr(out), DTYPE_CODE[torch.float16], ptr(x),
                                                 DTYPE_CODE[torch.float16], ptr(w), ptr(b), 1e-5, B,
                                                 D, H, W, C, codes, stream_ptr())
    assert rc == 0, _ops.last_error()
    assert torch.equal(out, got)


# (B, C, D, H, W): the hidden states of an 8-ROI batch of feature size 48 (x0 .. x4);
# volumes whose plane rows are 16-byte multiples take the cp.async kernel (also with
# partial last tiles: 1200 and 240 voxels, C = 40 and 64), the others (343, 210,
# 135 and 27 voxels) the one-tile-per-CTA kernel
PROJ_CASES = [
    (8, 48, 48, 48, 48),
    (8, 96, 24, 24, 24),
    (8, 192, 12, 12, 12),
    (8, 384, 6, 6, 6),
    (8, 768, 3, 3, 3),
    (2, 96, 10, 10, 12),
    (3, 64, 8, 5, 6),
    (2, 40, 4, 4, 4),
    (2, 96, 7, 7, 7),
    (1, 24, 5, 6, 7),
    (3, 64, 9, 3, 5),
]
PROJ_IDS = [f"B{b}_C{c}_{d}x{h}x{w}" for b, c, d, h, w in PROJ_CASES]


@pytest.mark.parametrize("out_dtype", DTYPES, ids=["out_f32", "out_f16", "out_bf16"])
@pytest.mark.parametrize("in_dtype", [torch.float16, torch.float32], ids=["in_f16", "in_f32"])
@pytest.mark.parametrize("case", PROJ_CASES, ids=PROJ_IDS)
def test_proj_out_norm_matches_eager(case, in_dtype, out_dtype, cuda_device):
    """proj_out's permute + layer_norm + permute back, against float64 on the same
    input values; the result has the eager path's shape and strides."""
    B, C, D, H, W = case
    x = (I.randn(300 + C + D, case, "float32") * 1.7 - 0.3).to(in_dtype)
    got = crumpet.proj_out_norm_3d(x.to(cuda_device), out_dtype=out_dtype)
    torch.cuda.synchronize()
    eager = torch.nn.functional.layer_norm(x.float().permute(0, 2, 3, 4, 1), [C]).permute(0, 4, 1, 2, 3)
    assert got.shape == eager.shape and got.stride() == eager.stride()
    assert got.dtype == out_dtype
    cl = x.double().permute(0, 2, 3, 4, 1).numpy()
    want = OB.layer_norm(cl, np.ones(C), np.zeros(C), 1e-5)
    g = got.permute(0, 2, 3, 4, 1).double().cpu().numpy()
    rel, atol = TOL[out_dtype]
    bad = np.abs(g - want) > np.abs(want) * rel + atol
    assert not bad.any(), (np.abs(g - want).max(), int(bad.sum()))


@pytest.mark.parametrize("shape", [(2, 96, 10, 9, 11), (2, 96, 10, 10, 12)],
                         ids=["scalar_loads", "cp_async"])
def test_proj_out_norm_affine_and_c_abi(shape, cuda_device):
    B, C, D, H, W = shape
    x = torch.randn((B, C, D, H, W), device=cuda_device).half()
    w = 1.0 + 0.3 * torch.randn(C, device=cuda_device)
    b = 0.2 * torch.randn(C, device=cuda_device)
    got = crumpet.proj_out_norm_3d(x, 1e-6, w, b, out_dtype=torch.float32)
    want = torch.nn.functional.layer_norm(x.float().permute(0, 2, 3, 4, 1), [C], w, b, 1e-6)
    assert (got.permute(0, 2, 3, 4, 1) - want).abs().max().item() <= 2e-5
    out = torch.empty((B, D, H, W, C), dtype=torch.float32, device=cuda_device)
    rc = _ops.capi().crumpet_proj_out_norm_3d(ptr(out), DTYPE_CODE[torch.float32], ptr(x),
                                              DTYPE_CODE[torch.float16], ptr(w), ptr(b), 1e-6, B, C,
                                              D, H, W, stream_ptr())
    assert rc == 0, _ops.last_error()
    assert torch.equal(out, got.permute(0, 2, 3, 4, 1))
    ops_out = torch.empty_like(out)
    _ops.require().proj_out_norm_3d(ops_out, x, None, None, 1e-5)
    plain = torch.nn.functional.layer_norm(x.float().permute(0, 2, 3, 4, 1), [C])
    assert (ops_out - plain).abs().max().item() <= 2e-5


def test_patched_proj_out_under_autocast(cuda_device):
    """The patched trunk's hidden-state norm returns what MONAI's proj_out returns
    under fp16 autocast: fp32, channels-last strides, the same values."""
    trunk = swin_unetr.SwinTransformer(1, 48, (7, 7, 7), (2, 2, 2), (1, 1, 1, 1), (3, 3, 3, 3))
    x = torch.randn((2, 48, 24, 24, 24), device=cuda_device).half()
    with torch.no_grad(), torch.autocast("cuda", dtype=torch.float16):
        want = trunk.proj_out(x, True)
        assert crumpet.patch_monai_swin_unetr(swin_unetr)
        try:
            got = trunk.proj_out(x, True)
        finally:
            crumpet.unpatch_monai_swin_unetr()
    assert got.dtype == want.dtype == torch.float32
    assert got.stride() == want.stride()
    assert (got - want).abs().max().item() <= 2e-5
