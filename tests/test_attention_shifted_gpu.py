"""fused_swin_attention given a mask that compute_attn_mask_3d built: the kernel adds that
shifted-window mask on chip (fused_swin_attention_shifted) instead of reading it, and must
give what the dense-mask path gives for the same mask -- with and without boundary flags,
on the tensor-core and the SIMT kernels -- and fall back to reading the mask once anyone
has written to it."""

from __future__ import annotations

import numpy as np
import pytest
import torch

import crumpet_b200 as crumpet
from crumpet_b200 import _ops
from crumpet_b200.cache import mask_geometry
from helpers import DTYPE_CODE, ptr, stream_ptr
from oracle import attention as OA

pytestmark = pytest.mark.gpu

TOL = {torch.float16: 2e-3, torch.bfloat16: 1.6e-2, torch.float32: 1e-4}


def _inputs(dev, grid, ws, ss, H, reps, dtype, hd=16, seed=0):
    g = torch.Generator().manual_seed(seed)
    N = ws[0] * ws[1] * ws[2]
    nw = tuple(d // w for d, w in zip(grid, ws))
    B = nw[0] * nw[1] * nw[2] * reps
    q, k, v = ((torch.randn((B, H, N, hd), generator=g) * 0.5).to(dtype).to(dev)
               for _ in range(3))
    bias = (torch.randn((H, N, N), generator=g) * 0.5).to(dtype).to(dev)
    mask = crumpet.compute_attn_mask_3d(*grid, ws, ss, dtype, dev)
    return q, k, v, bias, mask


CASES = [
    # (grid, window, shift, heads, batch repeats, dtype, head_dim)
    ((14, 14, 14), (7, 7, 7), (3, 3, 3), 3, 2, torch.float16, 16),
    ((14, 21, 7), (7, 7, 7), (3, 0, 2), 2, 1, torch.bfloat16, 16),
    ((14, 14, 14), (7, 7, 7), (3, 3, 3), 2, 1, torch.float16, 32),
    ((8, 8, 8), (4, 4, 4), (2, 2, 2), 2, 2, torch.float32, 16),   # SIMT kernel
    ((8, 8, 8), (4, 4, 4), (2, 2, 2), 2, 1, torch.float16, 64),   # SIMT kernel
]
IDS = ["f16_n343", "bf16_mixed_shift", "f16_d32", "f32_simt", "f16_d64_simt"]


@pytest.mark.parametrize("case", CASES, ids=IDS)
def test_recognised_mask_matches_dense_path(case, cuda_device):
    grid, ws, ss, H, reps, dtype, hd = case
    q, k, v, bias, mask = _inputs(cuda_device, grid, ws, ss, H, reps, dtype, hd)
    assert mask_geometry(mask) is not None
    dense = mask.clone()  # a copy is not recognised: read as given
    assert mask_geometry(dense) is None
    B = q.shape[0]
    true_flags = (mask.view(mask.shape[0], -1).abs().amax(1) > 0).to(torch.uint8)
    true_flags = true_flags.repeat(B // mask.shape[0])
    some = true_flags.clone()
    some[::3] = 0  # unflag some masked windows: they must come out unmasked on both paths
    for bnd in (None, true_flags, some):
        got = crumpet.fused_swin_attention(q, k, v, bias, mask, bnd)
        want = crumpet.fused_swin_attention(q, k, v, bias, dense, bnd)
        err = (got.float() - want.float()).abs().max().item()
        assert err <= TOL[dtype], (None if bnd is None else int(bnd.sum()), err)
    # and against the float64 oracle (mask applied to flagged windows only)
    got = crumpet.fused_swin_attention(q, k, v, bias, mask, some)
    f = lambda t: t.float().cpu().numpy()
    ref = OA.window_attention(f(q), f(k), f(v), f(bias), f(mask), some.cpu().numpy())
    assert np.abs(f(got) - ref).max() <= TOL[dtype]


def test_unflagged_windows_are_unmasked(cuda_device):
    q, k, v, bias, mask = _inputs(cuda_device, (14, 14, 14), (7, 7, 7), (3, 3, 3), 3, 1,
                                  torch.float16)
    none = torch.zeros(q.shape[0], dtype=torch.uint8, device=cuda_device)
    got = crumpet.fused_swin_attention(q, k, v, bias, mask, none)
    want = crumpet.fused_swin_attention(q, k, v, bias, None, None)
    assert (got.float() - want.float()).abs().max().item() <= TOL[torch.float16]


def test_written_mask_is_read_as_given(cuda_device):
    # a grid no other test uses, so the cached mask written to here stays private
    q, k, v, bias, mask = _inputs(cuda_device, (12, 12, 12), (6, 6, 6), (3, 3, 3), 2, 1,
                                  torch.float16, seed=7)
    try:
        assert mask_geometry(mask) is not None
        mask[-1, 0, :] = 0  # unmask one row of the last window: no longer the analytic mask
        assert mask_geometry(mask) is None
        got = crumpet.fused_swin_attention(q, k, v, bias, mask, None)
        want = crumpet.fused_swin_attention(q, k, v, bias, mask.clone(), None)
        assert torch.equal(got, want)
        m = mask.float().cpu().numpy()
        ref = OA.window_attention(q.float().cpu().numpy(), k.float().cpu().numpy(),
                                  v.float().cpu().numpy(), bias.float().cpu().numpy(), m)
        assert np.abs(got.float().cpu().numpy() - ref).max() <= TOL[torch.float16]
    finally:
        crumpet.clear_mask_cache()


def test_shifted_entry_through_the_c_abi(cuda_device):
    grid, ws, ss, H = (14, 14, 14), (7, 7, 7), (3, 3, 3), 3
    q, k, v, bias, mask = _inputs(cuda_device, grid, ws, ss, H, 1, torch.float16)
    B, N = q.shape[0], q.shape[2]
    out = torch.empty_like(q)
    lib = _ops.capi()
    rc = lib.crumpet_fused_swin_attention_shifted(
        ptr(out), ptr(q), ptr(k), ptr(v), ptr(bias), ptr(None), DTYPE_CODE[torch.float16], B,
        H, N, 16, 2, 2, 2, 7, 7, 7, 3, 3, 3, 0.25, stream_ptr())
    assert rc == 0, _ops.last_error()
    want = crumpet.fused_swin_attention(q, k, v, bias, mask.clone(), None)
    torch.cuda.synchronize()
    assert (out.float() - want.float()).abs().max().item() <= TOL[torch.float16]


def test_masks_built_in_inference_mode_are_read(cuda_device):
    # inference tensors keep no version counter, so such a mask is always read as given
    try:
        with torch.inference_mode():
            q, k, v, bias, mask = _inputs(cuda_device, (10, 10, 10), (5, 5, 5), (2, 2, 2), 2, 1,
                                          torch.float16, seed=3)
            assert mask_geometry(mask) is None
            got = crumpet.fused_swin_attention(q, k, v, bias, mask, None)
            want = crumpet.fused_swin_attention(q, k, v, bias, mask.clone(), None)
        assert torch.equal(got, want)
    finally:
        crumpet.clear_mask_cache()
