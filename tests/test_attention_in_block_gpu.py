"""The attention output inside the patched Swin block, at BASELINE config 1's
geometry ([1,28,28,28,48], window 7, shift 3, 3 heads, weights ~N(0,0.02)), under
fp16 autocast, checked at the north star's 2e-3 against the float64 oracle.

The block-level comparison with the eager network (tests/test_e2e_gpu.py) runs at
a looser tolerance because the two paths round LayerNorm, the Linears and the
residual adds at different points.  Here the attention kernel's own inputs and
output are recorded where the patched WindowAttention calls it (the module-level
names in crumpet_b200.monai_patch are wrapped for the duration of the run), and
the oracle recomputes the attention from exactly those inputs."""

from __future__ import annotations

import numpy as np
import pytest
import torch

import crumpet_b200 as crumpet
from crumpet_b200 import monai_patch, swin_unetr
from oracle import attention as OA
from oracle import mechanics as OM

pytestmark = pytest.mark.gpu
TOL = 2e-3


def _weights_like_config1(module, seed):
    g = torch.Generator().manual_seed(seed)
    with torch.no_grad():
        for name, p in module.named_parameters():
            if "norm" in name:
                continue
            p.copy_(torch.randn(p.shape, generator=g) * 0.02)


def _recorder(fn, calls):
    def wrapped(*args, **kwargs):
        out = fn(*args, **kwargs)
        calls.append((args, kwargs, out.detach().clone()))
        return out
    return wrapped


def test_dense_mask_attention_inside_block(cuda_device, monkeypatch):
    torch.manual_seed(0)
    blk = swin_unetr.SwinTransformerBlock(48, 3, (7, 7, 7), (3, 3, 3)).to(cuda_device).eval()
    _weights_like_config1(blk, 1)
    x = torch.randn((1, 28, 28, 28, 48), device=cuda_device)
    # a mask without recorded window geometry takes the dense-mask entry point
    mask = crumpet.compute_attn_mask_3d(28, 28, 28, (7, 7, 7), (3, 3, 3), torch.float16,
                                        cuda_device).clone()
    calls = []
    monkeypatch.setattr(monai_patch, "fused_swin_attention",
                        _recorder(monai_patch.fused_swin_attention, calls))
    crumpet.patch_monai_swin_unetr(swin_unetr)
    try:
        with torch.no_grad(), torch.autocast("cuda", dtype=torch.float16):
            blk(x, mask)
    finally:
        crumpet.unpatch_monai_swin_unetr()
    assert len(calls) == 1
    (q, k, v, bias, m, boundary), kwargs, out = calls[0]
    assert q.dtype == torch.float16 and q.shape == (64, 3, 343, 16)
    f = lambda t: None if t is None else t.float().cpu().numpy()
    want = OA.window_attention(f(q), f(k), f(v), f(bias), f(m),
                               None if boundary is None else boundary.cpu().numpy(),
                               kwargs.get("scale"))
    err = np.abs(out.float().cpu().numpy() - want).max()
    assert err <= TOL, err


def test_packed_attention_inside_stage(cuda_device, monkeypatch):
    """A whole stage (unshifted then shifted block): the patched BasicLayer records the
    mask's window geometry, so both blocks take the packed entry with the on-chip mask."""
    torch.manual_seed(0)
    layer = swin_unetr.BasicLayer(48, 2, 3, (7, 7, 7)).to(cuda_device).eval()
    _weights_like_config1(layer, 2)
    x = torch.randn((1, 48, 28, 28, 28), device=cuda_device)
    calls = []
    monkeypatch.setattr(monai_patch, "swin_window_attention_qkv",
                        _recorder(monai_patch.swin_window_attention_qkv, calls))
    crumpet.patch_monai_swin_unetr(swin_unetr)
    try:
        with torch.no_grad(), torch.autocast("cuda", dtype=torch.float16):
            layer(x)
    finally:
        crumpet.unpatch_monai_swin_unetr()
    assert len(calls) == 2
    shifts = []
    for (qkv, table, index, nw, ws, ss, scale), _, out in calls:
        shifts.append(tuple(ss))
        B, N, _, H, hd = qkv.shape
        assert qkv.dtype == torch.float16 and (B, N, H, hd) == (64, 343, 3, 16)
        bias = OA.gather_bias(table.detach().float().cpu().numpy(), index.cpu().numpy(), N)
        bias = torch.from_numpy(bias).half().float().numpy()  # rounded as the reference does
        q, k, v = (qkv[:, :, i].permute(0, 2, 1, 3).float().cpu().numpy() for i in range(3))
        mask = None
        if any(ss):
            mask = OM.attn_mask(*(n * w for n, w in zip(nw, ws)), tuple(ws), tuple(ss), np.float32)
        want = OA.window_attention(q, k, v, bias, mask, None, scale)
        got = out.float().cpu().numpy().reshape(B, N, H, hd).transpose(0, 2, 1, 3)
        err = np.abs(got - want).max()
        assert err <= TOL, (ss, err)
    assert shifts == [(0, 0, 0), (3, 3, 3)]
