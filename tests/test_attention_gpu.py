"""Fused window attention on the GPU against the reference Triton kernel's
outputs (golden, from the Triton CPU interpreter) and the float64 oracle.

Tolerance: max abs error <= 2e-3 on fp16 outputs.  bf16
outputs are compared at 1.6e-2 (two bf16 ulps at 1.0): bf16 rounding of the
output alone is up to 3.9e-3."""

from __future__ import annotations

from pathlib import Path

import numpy as np
import pytest
import torch

import crumpet_b200 as crumpet
import inputs as I
from crumpet_b200 import _ops
from helpers import DTYPE_CODE, ptr, stream_ptr
from oracle import attention as OA

pytestmark = pytest.mark.gpu
GOLDEN = np.load(Path(__file__).resolve().parent / "golden" / "attention_ref_out.npz")
FP16_TOL = 2e-3
BF16_TOL = 1.6e-2


def tol_for(dtype):
    return BF16_TOL if dtype == torch.bfloat16 else FP16_TOL


def oracle_out(q, k, v, bias, mask, boundary, scale=None):
    f = lambda t: None if t is None else t.float().cpu().numpy()
    return OA.window_attention(f(q), f(k), f(v), f(bias), f(mask),
                               None if boundary is None else boundary.cpu().numpy(), scale)


def run(case, dev):
    q, k, v, bias, mask, boundary = I.attention_inputs(case)
    to = lambda t: None if t is None else t.to(dev)
    out = crumpet.fused_swin_attention(to(q), to(k), to(v), to(bias), to(mask), to(boundary))
    torch.cuda.synchronize()
    return out, (q, k, v, bias, mask, boundary)


@pytest.mark.parametrize("case", I.ATTENTION_CASES, ids=[c[0] for c in I.ATTENTION_CASES])
def test_attention_matches_reference_kernel(case, cuda_device):
    out, args = run(case, cuda_device)
    got = out.float().cpu().numpy()
    ref = GOLDEN[case[0]]
    assert np.abs(got - ref).max() <= FP16_TOL
    assert np.abs(got - oracle_out(*args)).max() <= FP16_TOL
    assert _ops.capi().crumpet_device_status(1) == 0


@pytest.mark.parametrize("case", I.ORACLE_ONLY_ATTENTION_CASES,
                         ids=[c[0] for c in I.ORACLE_ONLY_ATTENTION_CASES])
def test_attention_matches_oracle(case, cuda_device):
    out, args = run(case, cuda_device)
    err = np.abs(out.float().cpu().numpy() - oracle_out(*args)).max()
    assert err <= tol_for(out.dtype), err


def test_attention_capi_and_mask_broadcast(cuda_device):
    case = I.ATTENTION_CASES[0]
    q, k, v, bias, mask, boundary = (None if t is None else t.to(cuda_device)
                                     for t in I.attention_inputs(case))
    B, H, N, D = q.shape
    # mask with 2 windows reused for 8 batch entries (b % 2), no boundary flags
    m2 = mask[:2].contiguous()
    out = torch.empty_like(q)
    rc = _ops.capi().crumpet_fused_swin_attention(
        ptr(out), ptr(q), ptr(k), ptr(v), ptr(bias), ptr(m2), 2, ptr(None),
        DTYPE_CODE[q.dtype], B, H, N, D, 0.25, stream_ptr())
    assert rc == 0, _ops.last_error()
    torch.cuda.synchronize()
    want = oracle_out(q, k, v, bias, m2, None, 0.25)
    assert np.abs(out.float().cpu().numpy() - want).max() <= FP16_TOL


def test_boundary_flags_skip_the_mask(cuda_device):
    case = I.ATTENTION_CASES[0]
    q, k, v, bias, mask, boundary = (None if t is None else t.to(cuda_device)
                                     for t in I.attention_inputs(case))
    zero = torch.zeros_like(boundary)
    got = crumpet.fused_swin_attention(q, k, v, bias, mask, zero)
    want = crumpet.fused_swin_attention(q, k, v, bias, None)
    torch.cuda.synchronize()
    assert torch.equal(got, want)
    ones = torch.ones_like(boundary)
    full = crumpet.fused_swin_attention(q, k, v, bias, mask, ones)
    assert np.abs(full.float().cpu().numpy() - oracle_out(q, k, v, bias, mask, None)).max() <= FP16_TOL


def test_attention_large_batch_many_heads(cuda_device):
    # more (head, query tile) pairs than SMs exercises the multi-pair schedule
    g = torch.Generator(device="cpu").manual_seed(5)
    B, H, N = 3, 60, 343
    q, k, v = (torch.randn((B, H, N, 16), generator=g).half() for _ in range(3))
    bias = (torch.randn((H, N, N), generator=g) * 0.5).half()
    out = crumpet.fused_swin_attention(q.to(cuda_device), k.to(cuda_device), v.to(cuda_device),
                                       bias.to(cuda_device), None)
    err = np.abs(out.float().cpu().numpy() - oracle_out(q, k, v, bias, None, None)).max()
    assert err <= FP16_TOL


def test_attention_deterministic(cuda_device):
    case = I.ATTENTION_CASES[0]
    a, _ = run(case, cuda_device)
    b, _ = run(case, cuda_device)
    assert torch.equal(a, b)


@pytest.mark.parametrize("head_dim", [16, 32])
def test_many_windows_per_cta_stay_in_step(head_dim, cuda_device):
    """600 windows x 3 heads: every CTA walks hundreds of tiles through the shared
    stage ring with all three warpgroups (head_dim 32 has a 2-stage ring), so a
    warpgroup racing ahead of the ring would read another tile's K/V."""
    g = torch.Generator().manual_seed(11)
    B, H, N = 600, 3, 343
    q, k, v = (torch.randn((B, H, N, head_dim), generator=g).half() for _ in range(3))
    bias = (torch.randn((H, N, N), generator=g) * 0.1).half()
    out = crumpet.fused_swin_attention(q.to(cuda_device), k.to(cuda_device), v.to(cuda_device),
                                       bias.to(cuda_device), None)
    torch.cuda.synchronize()
    sel = [0, 1, 2, 149, 299, 450, 598, 599]
    want = OA.window_attention(q[sel].float().numpy(), k[sel].float().numpy(),
                               v[sel].float().numpy(), bias.float().numpy(), None)
    assert np.abs(out[sel].float().cpu().numpy() - want).max() <= FP16_TOL
    assert _ops.capi().crumpet_device_status(1) == 0
