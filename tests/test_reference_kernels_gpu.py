"""The reference's own GPU kernels, as bench.py times them beside this repository's:
built from the reference's sources by baseline/build_reference.py (skipped when
that build is absent).  Checks that the side-by-side harness launches them
correctly -- the CUDA extension's ops agree bit for bit with crumpet_b200's on the
reference tests' shapes, and the Triton attention kernel, launched from its sm_100
cubin with Triton's parameter layout, matches the float64 oracle -- so the timings
in the bench line compare like with like."""

from __future__ import annotations

import numpy as np
import pytest
import torch

import bench
import crumpet_b200 as crumpet
import inputs as I
from oracle import attention as OA

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def ref(cuda_device):
    torch.zeros(1, device=cuda_device)  # the driver API calls need torch's context current
    kernels = bench.ReferenceGPUKernels.load()
    if kernels is None:
        pytest.skip("baseline/_ref not built")
    return kernels


@pytest.mark.parametrize("case", I.MECHANICS_CASES[:6], ids=[c[0] for c in I.MECHANICS_CASES[:6]])
def test_reference_mechanics_ops_agree_bit_for_bit(case, ref, cuda_device):
    _, shape, ws, ss, dtype, _ = case
    x = I.mechanics_input(case).to(cuda_device)
    ours = crumpet.fused_shift_partition_3d(x, ws, ss)
    theirs = torch.empty_like(ours)
    ref.ops.fused_shift_partition_3d(theirs, x, *ws, *ss)
    assert torch.equal(theirs, ours)
    back = torch.empty_like(x)
    ref.ops.fused_unshift_unpartition_3d(back, ours, *shape, *ws, *ss)
    assert torch.equal(back, x)
    D, H, W = shape[1:4]
    if ws[0] * ws[1] * ws[2] <= 1024:
        mask = crumpet.compute_attn_mask_3d(D, H, W, ws, ss, x.dtype, cuda_device)
        mask_r = torch.empty_like(mask)
        ref.ops.compute_attn_mask_3d(mask_r, D, H, W, *ws, *ss)
        assert torch.equal(mask_r, mask)


@pytest.mark.parametrize("B,H,N,masked", [(8, 3, 343, True), (4, 6, 343, False), (8, 24, 216, False)])
def test_reference_triton_attention_matches_oracle(B, H, N, masked, ref, cuda_device):
    g = torch.Generator().manual_seed(B * H + N)
    q, k, v = (torch.randn((B, H, N, 16), generator=g).half() for _ in range(3))
    bias = (torch.randn((H, N, N), generator=g) * 0.5).half()
    if masked:
        mask = crumpet.compute_attn_mask_3d(14, 14, 14, (7, 7, 7), (3, 3, 3), torch.float16,
                                            cuda_device).cpu()
        bnd = (mask.reshape(8, -1).abs().amax(1) > 0).to(torch.uint8)
    else:
        mask = torch.zeros((1, N, N), dtype=torch.float16)
        bnd = torch.zeros((B,), dtype=torch.uint8)
    dev = [t.to(cuda_device) for t in (q, k, v, bias, mask, bnd)]
    out = torch.empty_like(dev[0])
    ref.attention(out, *dev, 0.25)
    torch.cuda.synchronize()
    want = OA.window_attention(q.float().numpy(), k.float().numpy(), v.float().numpy(),
                               bias.float().numpy(), mask.float().numpy() if masked else None,
                               bnd.numpy() if masked else None, 0.25)
    assert np.abs(out.float().cpu().numpy() - want).max() <= 2e-3


def test_reference_launcher_refuses_other_specialisations(ref, cuda_device):
    q = torch.zeros((2, 3, 343, 32), dtype=torch.float16, device=cuda_device)  # head_dim 32
    bias = torch.zeros((3, 343, 343), dtype=torch.float16, device=cuda_device)
    mask = torch.zeros((1, 343, 343), dtype=torch.float16, device=cuda_device)
    bnd = torch.zeros((2,), dtype=torch.uint8, device=cuda_device)
    with pytest.raises(ValueError, match="specialisation"):
        ref.attention(torch.empty_like(q), q, q, q, bias, mask, bnd, 0.25)
