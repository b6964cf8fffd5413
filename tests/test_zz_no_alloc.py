"""crumpet_swin_window_attention_qkv_static_tiles: the packed-qkv window attention for
callers that cannot allocate device memory (the bias tiles live in a fixed buffer of the
library instead of one the caller allocates), checked through the C ABI against the
entry point that takes caller-allocated tiles, on calls in a row that reuse the buffer
with different shapes and inputs.  Named so that pytest collects it last."""

from __future__ import annotations

import pytest
import torch

from crumpet_b200 import _ops
from helpers import DTYPE_CODE, ptr, stream_ptr

pytestmark = pytest.mark.gpu

TOL = 2e-3  # the attention tests' tolerance on fp16 outputs
STATIC_BYTES = 4 << 20


def _rel_index(w: int) -> torch.Tensor:
    c = torch.stack(torch.meshgrid(*(torch.arange(w),) * 3, indexing="ij")).flatten(1)
    rel = (c[:, :, None] - c[:, None, :]) + (w - 1)
    m = 2 * w - 1
    return (rel[0] * m * m + rel[1] * m + rel[2]).long()


def _case(seed, dev, windows, ws, ss, H, cfg=7, dtype=torch.float16):
    """qkv, table and index of one call: `windows` windows per axis of window `ws`,
    shift `ss`, H heads of 16 channels, relative-position index of the configured
    cfg^3 window sliced to the runtime N (as MONAI's module does for the 6^3 stage)."""
    g = torch.Generator().manual_seed(seed)
    N = ws ** 3
    B = windows ** 3
    qkv = torch.randn((B, N, 3, H, 16), generator=g).to(dtype).to(dev)
    table = (torch.randn(((2 * cfg - 1) ** 3, H), generator=g) * 0.5).to(dev)
    index = _rel_index(cfg).to(dev)
    return dict(qkv=qkv, table=table, index=index, windows=windows, ws=ws, ss=ss, H=H, N=N,
                B=B, dtype=dtype)


def _geometry(c):
    w, ws, ss = c["windows"], c["ws"], c["ss"]
    return [w, w, w, ws, ws, ws, ss, ss, ss, DTYPE_CODE[c["dtype"]], c["B"], c["H"], c["N"], 16]


def _with_caller_tiles(lib, c):
    """The existing path: tiles in a buffer the caller allocated, then the attention."""
    nbytes = lib.crumpet_attention_bias_tiles_bytes(c["H"], c["N"])
    tiles = torch.empty(nbytes, dtype=torch.uint8, device=c["qkv"].device)
    rc = lib.crumpet_attention_bias_tiles(ptr(tiles), ptr(c["table"]), 1, c["table"].shape[0],
                                          ptr(c["index"]), c["index"].shape[1],
                                          DTYPE_CODE[c["dtype"]], c["H"], c["N"], 0.25,
                                          stream_ptr())
    assert rc == 0, _ops.last_error()
    out = torch.empty((c["B"], c["N"], c["H"] * 16), dtype=c["dtype"], device=c["qkv"].device)
    rc = lib.crumpet_swin_window_attention_qkv_tiles(ptr(out), ptr(c["qkv"]), ptr(tiles),
                                                     *_geometry(c), 0.25, stream_ptr())
    assert rc == 0, _ops.last_error()
    return out


def _static(lib, c):
    out = torch.full((c["B"], c["N"], c["H"] * 16), float("nan"), dtype=c["dtype"],
                     device=c["qkv"].device)
    rc = lib.crumpet_swin_window_attention_qkv_static_tiles(
        ptr(out), ptr(c["qkv"]), ptr(c["table"]), 1, c["table"].shape[0], ptr(c["index"]),
        c["index"].shape[1], *_geometry(c), 0.25, stream_ptr())
    assert rc == 0, _ops.last_error()
    return out


def test_static_tiles_match_caller_tiles_on_calls_in_a_row(cuda_device):
    lib = _ops.capi()
    cases = [
        # 12 heads x 3 query tiles at N = 343, shifted: 3.2 MiB of tiles, near the limit
        _case(1, cuda_device, 2, 7, 3, 12),
        # 24 heads x 2 query tiles at N = 216 (the 6^3 stage): another tile size over the
        # same buffer
        _case(2, cuda_device, 1, 6, 0, 24),
        # the first shape again with a new table and new inputs: nothing of the earlier
        # calls may show through
        _case(3, cuda_device, 2, 7, 3, 12),
        _case(4, cuda_device, 2, 7, 0, 3, dtype=torch.bfloat16),
    ]
    for c in cases:
        assert lib.crumpet_attention_bias_tiles_bytes(c["H"], c["N"]) <= STATIC_BYTES
        got = _static(lib, c)
        want = _with_caller_tiles(lib, c)
        torch.cuda.synchronize()
        assert torch.isfinite(got.float()).all()
        err = (got.float() - want.float()).abs().max().item()
        assert err <= TOL, (c["H"], c["N"], err)
    assert lib.crumpet_device_status(1) == 0


def test_static_tiles_reject_more_than_the_buffer_holds(cuda_device):
    lib = _ops.capi()
    c = _case(5, cuda_device, 1, 7, 0, 24)  # 24 heads x 3 tiles at N = 343: 6.2 MiB
    assert lib.crumpet_attention_bias_tiles_bytes(24, 343) > STATIC_BYTES
    out = torch.empty((c["B"], c["N"], 24 * 16), dtype=torch.float16, device=cuda_device)
    rc = lib.crumpet_swin_window_attention_qkv_static_tiles(
        ptr(out), ptr(c["qkv"]), ptr(c["table"]), 1, c["table"].shape[0], ptr(c["index"]),
        c["index"].shape[1], *_geometry(c), 0.25, stream_ptr())
    assert rc == 3 and "4 MiB" in _ops.last_error()
