"""Window attention at the deeper-stage shapes of BASELINE config 4, through both
attention entry points, against the float64 oracle.

Config 4: fp16, window 7 and shift 3 unless the dimension is at most the window
(then the window is the dimension and there is no shift), head_dim 16:
[1,28,28,28,96] with 6 heads, [1,14,14,14,192] with 12 heads, [1,7,7,7,384] with
24 heads (no shift), each also as a sliding-window batch of 4 and of 8 (the mask of
the volume's windows is reused by every batch entry: window b uses mask[b % nW]).
Inputs follow the config: tokens ~N(0,1) through qkv weights ~N(0,0.02), the bias
table ~N(0,0.02).  The kernels run the whole batch; the oracle checks a sample of
windows that includes the first, the last, interior and boundary windows.
Tolerance: max abs error <= 2e-3 (the north star's fp16 bound)."""

from __future__ import annotations

import numpy as np
import pytest
import torch

import crumpet_b200 as crumpet
from crumpet_b200 import _ops
from crumpet_b200.fused_attention import swin_window_attention_qkv
from oracle import attention as OA
from oracle import mechanics as OM

pytestmark = pytest.mark.gpu
TOL = 2e-3

# (name, volume edge, channels, heads, batch)
CFG4 = [
    ("28cube_c96_h6", 28, 96, 6, 1),
    ("28cube_c96_h6_b4", 28, 96, 6, 4),
    ("28cube_c96_h6_b8", 28, 96, 6, 8),
    ("14cube_c192_h12", 14, 192, 12, 1),
    ("14cube_c192_h12_b4", 14, 192, 12, 4),
    ("14cube_c192_h12_b8", 14, 192, 12, 8),
    ("7cube_c384_h24", 7, 384, 24, 1),
    ("7cube_c384_h24_b4", 7, 384, 24, 4),
    ("7cube_c384_h24_b8", 7, 384, 24, 8),
]


def geometry(edge):
    ws = (min(7, edge),) * 3
    ss = (3, 3, 3) if edge > 7 else (0, 0, 0)
    nw = tuple(edge // w for w in ws)
    return ws, ss, nw


def make_inputs(edge, C, H, batch, seed):
    """qkv [B, N, 3, H, 16] fp16 (B = batch x windows), table [13^3, H] fp32, index."""
    g = torch.Generator().manual_seed(seed)
    ws, ss, nw = geometry(edge)
    N = ws[0] * ws[1] * ws[2]
    B = batch * nw[0] * nw[1] * nw[2]
    x = torch.randn((B, N, C), generator=g)
    w_qkv = torch.randn((3 * C, C), generator=g) * 0.02
    qkv = (x @ w_qkv.T).half().reshape(B, N, 3, H, C // H)
    table = torch.randn((13 ** 3, H), generator=g) * 0.02
    index = torch.from_numpy(OA.relative_position_index((7, 7, 7))).long()
    return qkv, table, index, ws, ss, nw


def sample(B, nwin):
    picks = {0, 1, B - 1, B // 2, nwin - 1, min(B - 1, nwin), B - nwin}
    return sorted(p for p in picks if 0 <= p < B)


def oracle(qkv, table, index, ws, ss, nw, sel):
    B, N, _, H, hd = qkv.shape
    bias = torch.from_numpy(OA.gather_bias(table.numpy(), index.numpy(), N)).half().float()
    q, k, v = (qkv[sel, :, i].permute(0, 2, 1, 3).float().numpy() for i in range(3))
    mask = None
    if any(ss):
        full = OM.attn_mask(*(n * w for n, w in zip(nw, ws)), ws, ss, np.float32)
        mask = full[np.asarray(sel) % full.shape[0]]  # one row per sampled window
    return OA.window_attention(q, k, v, bias.numpy(), mask)  # [S, H, N, hd]


@pytest.mark.parametrize("case", CFG4, ids=[c[0] for c in CFG4])
def test_cfg4_dense_entry_matches_oracle(case, cuda_device):
    name, edge, C, H, batch = case
    qkv, table, index, ws, ss, nw = make_inputs(edge, C, H, batch, seed=len(name) * 7 + edge)
    B, N = qkv.shape[:2]
    nwin = nw[0] * nw[1] * nw[2]
    dev = cuda_device
    q, k, v = (qkv[:, :, i].permute(0, 2, 1, 3).contiguous().to(dev) for i in range(3))
    bias = torch.from_numpy(OA.gather_bias(table.numpy(), index.numpy(), N)).half().to(dev)
    mask = boundary = None
    if any(ss):
        mask = crumpet.compute_attn_mask_3d(edge, edge, edge, ws, ss, torch.float16, dev)
        flags = (mask.reshape(nwin, -1).abs().amax(1) > 0).to(torch.uint8)
        boundary = flags.repeat(batch)
    out = crumpet.fused_swin_attention(q, k, v, bias, mask, boundary)
    torch.cuda.synchronize()
    sel = sample(B, nwin)
    want = oracle(qkv, table, index, ws, ss, nw, sel)
    err = np.abs(out[sel].float().cpu().numpy() - want).max()
    assert err <= TOL, err
    assert torch.isfinite(out).all()
    assert _ops.capi().crumpet_device_status(1) == 0


@pytest.mark.parametrize("case", CFG4, ids=[c[0] for c in CFG4])
def test_cfg4_packed_entry_matches_oracle(case, cuda_device):
    name, edge, C, H, batch = case
    qkv, table, index, ws, ss, nw = make_inputs(edge, C, H, batch, seed=len(name) * 11 + edge)
    B, N, _, _, hd = qkv.shape
    nwin = nw[0] * nw[1] * nw[2]
    out = swin_window_attention_qkv(qkv.to(cuda_device), table.to(cuda_device),
                                    index.to(cuda_device), nw, ws, ss, hd ** -0.5)
    torch.cuda.synchronize()
    sel = sample(B, nwin)
    want = oracle(qkv, table, index, ws, ss, nw, sel)  # [S, H, N, hd]
    got = out[sel].float().cpu().numpy().reshape(len(sel), N, H, hd).transpose(0, 2, 1, 3)
    err = np.abs(got - want).max()
    assert err <= TOL, err
    assert torch.isfinite(out).all()
    assert _ops.capi().crumpet_device_status(1) == 0
