"""Roll+partition, unpartition+reverse-roll and mask kernels on the GPU:
bit-exact against the reference's golden digests (tests/golden/manifest.json)
and the oracle, through the torch ops and through the C ABI.  Ports the
reference's tests/test_correctness.py, test_dtype.py, test_backward.py and
test_compile.py."""

from __future__ import annotations

import json
from pathlib import Path

import numpy as np
import pytest
import torch

import crumpet_b200 as crumpet
import inputs as I
from crumpet_b200 import _ops
from helpers import DTYPE_CODE, ptr, sha, stream_ptr
from oracle import mechanics as OM

pytestmark = pytest.mark.gpu
MANIFEST = json.loads((Path(__file__).resolve().parent / "golden" / "manifest.json").read_text())
MECH_IDS = [c[0] for c in I.MECHANICS_CASES]
MASK_IDS = [c[0] for c in I.MASK_CASES]


@pytest.mark.parametrize("case", I.MECHANICS_CASES, ids=MECH_IDS)
def test_partition_unpartition_match_reference(case, cuda_device):
    name, shape, ws, ss, dtype, seed = case
    B, D, H, W, C = shape
    x = I.mechanics_input(case).to(cuda_device)
    golden = MANIFEST["mechanics"][name]
    win = crumpet.fused_shift_partition_3d(x, ws, ss)
    assert list(win.shape) == golden["partition_shape"]
    assert sha(win) == golden["partition_sha256"]
    back = crumpet.fused_unshift_unpartition_3d(win, B, D, H, W, C, ws, ss)
    assert torch.equal(back, x)


@pytest.mark.parametrize("case", I.MECHANICS_CASES[:8], ids=MECH_IDS[:8])
def test_partition_matches_oracle_and_capi(case, cuda_device):
    name, shape, ws, ss, dtype, seed = case
    B, D, H, W, C = shape
    x = I.mechanics_input(case)
    raw = x.view(torch.int16) if x.dtype == torch.bfloat16 else x
    want = torch.from_numpy(OM.shift_partition(raw.numpy(), ws, ss))
    if x.dtype == torch.bfloat16:
        want = want.view(torch.bfloat16)
    xd = x.to(cuda_device)
    out = torch.empty(want.shape, dtype=x.dtype, device=cuda_device)
    lib = _ops.capi()
    rc = lib.crumpet_fused_shift_partition_3d(ptr(out), ptr(xd), DTYPE_CODE[x.dtype], B, D, H, W, C,
                                              *ws, *ss, stream_ptr())
    assert rc == 0, _ops.last_error()
    assert torch.equal(out.cpu(), want)
    back = torch.empty_like(xd)
    rc = lib.crumpet_fused_unshift_unpartition_3d(ptr(back), ptr(out), DTYPE_CODE[x.dtype], B, D, H,
                                                  W, C, *ws, *ss, stream_ptr())
    assert rc == 0, _ops.last_error()
    assert torch.equal(back, xd)


@pytest.mark.parametrize("case", I.MASK_CASES, ids=MASK_IDS)
def test_mask_matches_reference(case, cuda_device):
    name, dims, ws, ss, dtype = case
    crumpet.clear_mask_cache()
    m = crumpet.compute_attn_mask_3d(*dims, ws, ss, getattr(torch, dtype), cuda_device)
    golden = MANIFEST["mask"][name]
    assert list(m.shape) == golden["shape"]
    assert int((m != 0).sum()) == golden["neg_count"]
    assert sha(m) == golden["sha256"]
    crumpet.clear_mask_cache()


def test_mask_capi_unaligned_output(cuda_device):
    # an output that is only element-aligned exercises the scalar store path
    want = torch.from_numpy(OM.attn_mask(14, 14, 14, (7, 7, 7), (3, 3, 3), np.float32)).half()
    buf = torch.full((want.numel() + 1,), 7.0, dtype=torch.float16, device=cuda_device)
    out = buf[1:]
    rc = _ops.capi().crumpet_compute_attn_mask_3d(ptr(out), 1, 14, 14, 14, 7, 7, 7, 3, 3, 3, stream_ptr())
    assert rc == 0, _ops.last_error()
    assert torch.equal(out.view(want.shape).cpu(), want)
    assert buf[0].item() == 7.0


def test_shift_size_zero_mask_is_zero(cuda_device):
    mask = crumpet.compute_attn_mask_3d(14, 14, 14, (7, 7, 7), (0, 0, 0), torch.float16, cuda_device)
    assert torch.count_nonzero(mask).item() == 0


def test_partition_unaligned_pointers(cuda_device):
    # views that start one element in force the 2-byte vector path
    shape = (1, 8, 8, 8, 32)
    n = int(np.prod(shape))
    base = torch.randn((n + 1,), device=cuda_device, dtype=torch.float16)
    xv = base[1:].view(shape)
    out_base = torch.empty((n + 1,), device=cuda_device, dtype=torch.float16)
    out = out_base[1:].view(8, 64, 32)
    rc = _ops.capi().crumpet_fused_shift_partition_3d(ptr(out), ptr(xv), 1, *shape, 4, 4, 4, 2, 2, 2,
                                                      stream_ptr())
    assert rc == 0, _ops.last_error()
    want = OM.shift_partition(xv.cpu().numpy(), (4, 4, 4), (2, 2, 2))
    assert np.array_equal(out.cpu().numpy(), want)


@pytest.mark.parametrize("dtype", [torch.float32, torch.float16, torch.bfloat16])
def test_supported_dtypes(dtype, cuda_device):
    x = torch.randn((1, 8, 8, 8, 4), device=cuda_device, dtype=dtype)
    y = crumpet.fused_shift_partition_3d(x, (4, 4, 4), (2, 2, 2))
    z = crumpet.fused_unshift_unpartition_3d(y, 1, 8, 8, 8, 4, (4, 4, 4), (2, 2, 2))
    assert y.dtype == dtype and z.dtype == dtype
    assert torch.equal(z, x)
    mask = crumpet.compute_attn_mask_3d(8, 8, 8, (4, 4, 4), (2, 2, 2), dtype, cuda_device)
    assert mask.dtype == dtype


@pytest.mark.parametrize("shift_size", [(3, 3, 3), (0, 0, 0)])
def test_backward_matches_reference(shift_size, cuda_device):
    x = torch.randn((1, 14, 14, 14, 5), device=cuda_device, requires_grad=True)
    x_ref = x.detach().clone().requires_grad_(True)
    y = crumpet.fused_shift_partition_3d(x, (7, 7, 7), shift_size)
    y_ref = crumpet.unfused_shift_partition_3d_reference(x_ref, (7, 7, 7), shift_size)
    grad = torch.randn_like(y)
    y.backward(grad)
    y_ref.backward(grad)
    assert torch.equal(x.grad, x_ref.grad)

    w = y.detach().clone().requires_grad_(True)
    w_ref = w.detach().clone().requires_grad_(True)
    z = crumpet.fused_unshift_unpartition_3d(w, 1, 14, 14, 14, 5, (7, 7, 7), shift_size)
    z_ref = crumpet.unfused_unshift_unpartition_3d_reference(w_ref, 1, 14, 14, 14, 5, (7, 7, 7), shift_size)
    g2 = torch.randn_like(z)
    z.backward(g2)
    z_ref.backward(g2)
    assert torch.equal(w.grad, w_ref.grad)


def test_torch_compile_fullgraph_round_trip(cuda_device):
    class Module(torch.nn.Module):
        def forward(self, x):
            w = crumpet.fused_shift_partition_3d(x, (2, 2, 2), (1, 1, 1))
            return crumpet.fused_unshift_unpartition_3d(w, x.shape[0], 4, 4, 4, x.shape[-1], (2, 2, 2), (1, 1, 1))

    x = torch.randn((1, 4, 4, 4, 3), device=cuda_device)
    try:
        compiled = torch.compile(Module(), fullgraph=True)
        out = compiled(x)
    except Exception as exc:  # inductor toolchain problems are environment faults
        if "Inductor" in type(exc).__name__ or "CppCompileError" in repr(exc):
            pytest.skip(f"torch.compile toolchain unavailable: {exc!r}"[:200])
        raise
    assert torch.equal(out, x)


def test_empty_batch(cuda_device):
    x = torch.empty((0, 8, 8, 8, 4), device=cuda_device)
    y = crumpet.fused_shift_partition_3d(x, (4, 4, 4), (2, 2, 2))
    assert y.shape == (0, 64, 4)
