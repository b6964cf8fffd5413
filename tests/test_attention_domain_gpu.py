"""The reference launcher's whole input domain (torch-ext/crumpet/fused_attention.py:149-226
takes any dtype tl.dot takes and any power-of-two head_dim >= 16, for any N): float32
q/k/v, head dims 64 / 128 / 256, and windows of more than 384 tokens, which run the fp32
SIMT kernel, against the float64 oracle.

Tolerances: float32 outputs within 2e-5 (the kernel computes in fp32 throughout);
float16 within the north star's 2e-3; bfloat16 within 1.6e-2 (two bf16 ulps at 1)."""

from __future__ import annotations

import numpy as np
import pytest
import torch

import crumpet_b200 as crumpet
from crumpet_b200 import _ops, profiling, swin_unetr
from crumpet_b200.fused_attention import swin_window_attention_qkv
from oracle import attention as OA
from oracle import mechanics as OM

pytestmark = pytest.mark.gpu
TOL = {torch.float32: 2e-5, torch.float16: 2e-3, torch.bfloat16: 1.6e-2}

# (name, B, H, window, head_dim, dtype, masked volume or None)
DENSE_CASES = [
    ("f32_d16_n343_mask", 8, 3, (7, 7, 7), 16, torch.float32, (14, 14, 14)),
    ("f32_d64_n343", 4, 2, (7, 7, 7), 64, torch.float32, None),
    ("f32_d128_n216", 3, 2, (6, 6, 6), 128, torch.float32, None),
    ("f16_d64_n343_mask", 8, 2, (7, 7, 7), 64, torch.float16, (14, 14, 14)),
    ("f16_d128_n343", 2, 2, (7, 7, 7), 128, torch.float16, None),
    ("f16_d64_n216", 4, 3, (6, 6, 6), 64, torch.float16, None),
    ("f16_d256_n64_mask", 8, 1, (4, 4, 4), 256, torch.float16, (8, 8, 8)),
    ("bf16_d64_n343", 2, 3, (7, 7, 7), 64, torch.bfloat16, None),
    ("f16_d16_n512_mask", 8, 2, (8, 8, 8), 16, torch.float16, (16, 16, 16)),
    ("f32_d32_n1000", 2, 1, (10, 10, 10), 32, torch.float32, None),
]


def _inputs(B, H, window, hd, dtype, mvol, seed):
    g = torch.Generator().manual_seed(seed)
    N = window[0] * window[1] * window[2]
    q, k, v = (torch.randn((B, H, N, hd), generator=g).to(dtype) for _ in range(3))
    bias = (torch.randn((H, N, N), generator=g) * 0.5).to(dtype)
    mask = None
    if mvol is not None:
        ss = tuple(w // 2 for w in window)
        mask = torch.from_numpy(OM.attn_mask(*mvol, window, ss, np.float32)).to(dtype)
    return q, k, v, bias, mask


@pytest.mark.parametrize("case", DENSE_CASES, ids=[c[0] for c in DENSE_CASES])
def test_dense_entry_domain_matches_oracle(case, cuda_device):
    name, B, H, window, hd, dtype, mvol = case
    q, k, v, bias, mask = _inputs(B, H, window, hd, dtype, mvol, seed=len(name) + hd)
    to = lambda t: None if t is None else t.to(cuda_device)
    out = crumpet.fused_swin_attention(to(q), to(k), to(v), to(bias), to(mask))
    torch.cuda.synchronize()
    assert out.dtype == dtype and out.shape == q.shape
    f = lambda t: None if t is None else t.float().numpy()
    want = OA.window_attention(f(q), f(k), f(v), f(bias), f(mask))
    err = np.abs(out.float().cpu().numpy() - want).max()
    assert err <= TOL[dtype], err
    assert _ops.capi().crumpet_device_status(1) == 0


@pytest.mark.parametrize("dtype,hd,dims,ws,ss", [
    (torch.float32, 16, (14, 14, 14), (7, 7, 7), (3, 3, 3)),
    (torch.float32, 32, (6, 6, 6), (6, 6, 6), (0, 0, 0)),
    (torch.float16, 64, (14, 14, 14), (7, 7, 7), (3, 3, 3)),
    (torch.bfloat16, 128, (14, 7, 7), (7, 7, 7), (3, 0, 2)),
], ids=["f32_d16_shift", "f32_d32_quirk216", "f16_d64_shift", "bf16_d128_mixed"])
def test_packed_entry_domain_matches_oracle(dtype, hd, dims, ws, ss, cuda_device):
    g = torch.Generator().manual_seed(hd)
    nw = tuple(d // w for d, w in zip(dims, ws))
    B, H, N = 2 * nw[0] * nw[1] * nw[2], 2, ws[0] * ws[1] * ws[2]
    qkv = torch.randn((B, N, 3, H, hd), generator=g).to(dtype)
    table = torch.randn((13 ** 3, H), generator=g) * 0.5
    index = torch.from_numpy(OA.relative_position_index((7, 7, 7))).long()
    out = swin_window_attention_qkv(qkv.to(cuda_device), table.to(cuda_device),
                                    index.to(cuda_device), nw, ws, ss, hd ** -0.5)
    torch.cuda.synchronize()
    bias = torch.from_numpy(OA.gather_bias(table.numpy(), index.numpy(), N)).to(dtype).float()
    mask = OM.attn_mask(*dims, ws, ss, np.float32) if any(ss) else None
    q, k, v = (qkv[:, :, i].permute(0, 2, 1, 3).float().numpy() for i in range(3))
    want = OA.window_attention(q, k, v, bias.numpy(), mask)
    got = out.float().cpu().numpy().reshape(B, N, H, hd).transpose(0, 2, 1, 3)
    err = np.abs(got - want).max()
    assert err <= TOL[dtype], err
    assert _ops.capi().crumpet_device_status(1) == 0


def test_unsupported_head_dims_are_rejected(cuda_device):
    q = torch.zeros((1, 1, 8, 24), dtype=torch.float16, device=cuda_device)
    bias = torch.zeros((1, 8, 8), dtype=torch.float16, device=cuda_device)
    with pytest.raises(ValueError, match="power-of-two head_dim"):
        crumpet.fused_swin_attention(q, q, q, bias, None)
    q = torch.zeros((1, 1, 8, 8), dtype=torch.float16, device=cuda_device)
    with pytest.raises(ValueError, match="power-of-two head_dim"):
        crumpet.fused_swin_attention(q, q, q, bias, None)


def test_fp32_stage_runs_the_fused_attention(cuda_device):
    """A float32 stage (no autocast) takes the fused attention, as the reference's patch
    does, and matches the eager stage."""
    torch.manual_seed(0)
    layer = swin_unetr.BasicLayer(48, 2, 3, (7, 7, 7)).to(cuda_device).eval()
    with torch.no_grad():
        for name, p in layer.named_parameters():
            if "norm" not in name:
                p.normal_(0, 0.02)
    x = torch.randn((1, 48, 14, 14, 14), device=cuda_device)
    with torch.no_grad():
        eager = layer(x)
        before = profiling.counters.get("swin_window_attention_qkv", 0)
        crumpet.patch_monai_swin_unetr(swin_unetr)
        try:
            patched = layer(x)
        finally:
            crumpet.unpatch_monai_swin_unetr()
    assert profiling.counters.get("swin_window_attention_qkv", 0) - before == 2
    assert patched.dtype == torch.float32
    assert (patched - eager).abs().max().item() < 1e-4
