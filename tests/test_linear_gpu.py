"""The qkv / proj Linears of the window attention on the tensor cores (tcgen05 GEMM with a
fused bias epilogue), against a float64 reference and against torch's own F.linear (cuBLAS)
on the same fp16 / bf16 operands: within one rounding of the output."""

from __future__ import annotations

import pytest
import torch

import crumpet_b200 as crumpet
from crumpet_b200 import _ops
from helpers import DTYPE_CODE, ptr, stream_ptr

pytestmark = pytest.mark.gpu

# (M, K, N): stage-1 qkv and proj at full size (2744 windows x 343 tokens of an 8-ROI batch),
# stage-1 proj with a partial last tile, a single partial tile, stage-2 proj, the largest
# supported N, K = 96 at its largest N
CASES = [(941192, 48, 144), (941192, 48, 48), (1000, 48, 48), (77, 48, 144), (5000, 96, 96),
         (3000, 48, 256), (2048, 96, 160)]
IDS = [f"M{m}_K{k}_N{n}" for m, k, n in CASES]


def _ref(x, w, b):
    y = x.double() @ w.double().t()
    return y if b is None else y + b.double()


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16], ids=["f16", "bf16"])
@pytest.mark.parametrize("case", CASES, ids=IDS)
def test_window_linear_matches_float64_and_cublas(case, dtype, cuda_device):
    M, K, N = case
    g = torch.Generator(device=cuda_device).manual_seed(M + N)
    x = torch.randn((M, K), device=cuda_device, generator=g).to(dtype)
    w = (torch.randn((N, K), device=cuda_device, generator=g) * K ** -0.5).to(dtype)
    b = (0.1 * torch.randn((N,), device=cuda_device, generator=g)).to(dtype)
    got = crumpet.window_linear(x, w, b)
    torch.cuda.synchronize()
    assert _ops.capi().crumpet_device_status(1) == 0
    assert got.shape == (M, N) and got.dtype == dtype
    ref = _ref(x, w, b)
    ulp = 2.0 ** -10 if dtype == torch.float16 else 2.0 ** -7
    err = (got.double() - ref).abs()
    assert (err <= ref.abs() * ulp + 1e-3).all(), err.max().item()
    cublas = torch.nn.functional.linear(x, w, b)
    assert ((got.double() - cublas.double()).abs() <= cublas.double().abs() * 2 * ulp + 2e-3).all()


def test_window_linear_no_bias_views_and_c_abi(cuda_device):
    g = torch.Generator(device=cuda_device).manual_seed(3)
    x = torch.randn((4, 343, 48), device=cuda_device, generator=g).half()
    w = torch.randn((144, 48), device=cuda_device, generator=g).half() * 0.1
    got = crumpet.window_linear(x, w)  # [..., K] input, no bias
    assert got.shape == (4, 343, 144)
    ref = _ref(x.reshape(-1, 48), w, None).reshape(4, 343, 144)
    assert ((got.double() - ref).abs() <= ref.abs() * 2.0 ** -10 + 1e-3).all()
    xt = torch.randn((48, 500), device=cuda_device, generator=g).half().t()  # a strided view
    assert torch.equal(crumpet.window_linear(xt, w), crumpet.window_linear(xt.contiguous(), w))
    out = torch.empty((1372, 144), dtype=torch.float16, device=cuda_device)
    x2 = x.reshape(-1, 48)
    bias = torch.zeros(144, device=cuda_device)
    rc = _ops.capi().crumpet_window_linear(ptr(out), ptr(x2), ptr(w), ptr(bias),
                                           DTYPE_CODE[torch.float16], 1372, 48, 144, stream_ptr())
    assert rc == 0, _ops.last_error()
    assert torch.equal(out, got.reshape(-1, 144))
