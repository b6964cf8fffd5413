"""Bounded-wait error path of the attention kernel on the GPU, without faulting it.

The kernel's waits (on TMA loads, tensor-core results and the other warps) give up
after 2 s, record a device error word, drain and free their tensor memory.  The
test hook `crumpet_test_stall_attention` makes the producer issue nothing, so every
wait runs out; the test checks that the launch returns, that the error word is set,
and that the context stays usable (the next launch is correct)."""

from __future__ import annotations

import time

import numpy as np
import pytest
import torch

import crumpet_b200 as crumpet
from crumpet_b200 import _ops
from oracle import attention as OA

pytestmark = pytest.mark.gpu


def _case(device):
    g = torch.Generator().manual_seed(7)
    q, k, v = (torch.randn((4, 2, 64, 16), generator=g).half() for _ in range(3))
    bias = (torch.randn((2, 64, 64), generator=g) * 0.5).half()
    return q, k, v, bias


def test_attention_wait_timeout_sets_device_error_and_context_survives(cuda_device):
    lib = _ops.capi()
    lib.crumpet_device_status(1)
    q, k, v, bias = _case(cuda_device)
    dq, dk, dv, db = (t.to(cuda_device) for t in (q, k, v, bias))
    prev = lib.crumpet_test_stall_attention(1)
    try:
        t0 = time.time()
        crumpet.fused_swin_attention(dq, dk, dv, db, None)
        torch.cuda.synchronize()
        waited = time.time() - t0
    finally:
        lib.crumpet_test_stall_attention(prev)
    assert lib.crumpet_device_status(1) == 1  # the kernel reported its expired waits
    assert 1.0 < waited < 30.0
    out = crumpet.fused_swin_attention(dq, dk, dv, db, None)
    torch.cuda.synchronize()
    want = OA.window_attention(q.float().numpy(), k.float().numpy(), v.float().numpy(),
                               bias.float().numpy(), None)
    assert np.abs(out.float().cpu().numpy() - want).max() <= 2e-3
    assert lib.crumpet_device_status(0) == 0
