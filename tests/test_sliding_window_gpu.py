"""Sliding-window ROI kernels on the GPU, bit-exact against the eager torch passes
they replace (MONAI sliding_window_inference, mode "constant", as driven by the
reference at torch-ext/crumpet/demo_btcv.py:98-129): the ROI crop + torch.cat, the
per-ROI fp32 accumulation loop, and the count division + arg-max."""

from __future__ import annotations

import pytest
import torch

from crumpet_b200 import _ops
from crumpet_b200.inferer import SlidingWindowInferer, axis_counts, roi_grid
from helpers import DTYPE_CODE, ptr, stream_ptr

pytestmark = pytest.mark.gpu


def _eager_accumulate(model, volume, roi, sw_batch, overlap, classes, autocast):
    rd, rh, rw = roi
    spatial = tuple(volume.shape[2:])
    acc = torch.zeros((1, classes, *spatial), dtype=torch.float32, device=volume.device)
    starts = roi_grid(spatial, roi, overlap)
    for b0 in range(0, len(starts), sw_batch):
        batch = starts[b0:b0 + sw_batch]
        window = torch.cat([volume[..., z:z + rd, y:y + rh, x:x + rw] for z, y, x in batch])
        with torch.autocast("cuda", dtype=torch.float16, enabled=autocast):
            pred = model(window)
        for i, (z, y, x) in enumerate(batch):
            acc[0, :, z:z + rd, y:y + rh, x:x + rw] += pred[i].float()
    cnt = torch.zeros((1, 1, *spatial), dtype=torch.float32, device=volume.device)
    for z, y, x in starts:
        cnt[..., z:z + rd, y:y + rh, x:x + rw] += 1.0
    return acc, acc / cnt


GATHER_LAYOUTS = {
    # W = 53 and x starts 17 / 21: one element per thread
    "scalar_x": (53, [(0, 0, 0), (30, 5, 17), (38, 29, 21), (7, 13, 0)]),
    # W = 64 and every x start a multiple of 8: eight x voxels per thread
    "vec8_x": (64, [(0, 0, 0), (30, 5, 16), (38, 29, 32), (7, 13, 8)]),
}


@pytest.mark.parametrize("layout", list(GATHER_LAYOUTS))
@pytest.mark.parametrize("in_dtype", [torch.float32, torch.float16])
@pytest.mark.parametrize("out_dtype", [torch.float32, torch.float16, torch.bfloat16])
def test_roi_gather_matches_slicing(out_dtype, in_dtype, layout, cuda_device):
    g = torch.Generator(device=cuda_device).manual_seed(0)
    width, starts = GATHER_LAYOUTS[layout]
    vol = torch.rand((2, 70, 61, width), device=cuda_device, generator=g).to(in_dtype)
    roi = (32, 32, 32)
    out = torch.empty((4, 2, *roi), dtype=out_dtype, device=cuda_device)
    _ops.require().roi_gather(out, vol, [v for s in starts for v in s], list(roi))
    want = torch.stack([vol[:, z:z + 32, y:y + 32, x:x + 32] for z, y, x in starts]).to(out_dtype)
    assert torch.equal(out, want)


@pytest.mark.parametrize("width,rw", [(61, 24), (64, 24), (80, 32)],
                         ids=["scalar_x", "vec4_x", "vec8_x"])
@pytest.mark.parametrize("pred_dtype", [torch.float16, torch.bfloat16, torch.float32])
def test_roi_accumulate_bit_exact_with_overlaps(pred_dtype, width, rw, cuda_device):
    # W = 64 puts every ROI x start on a multiple of 4 (4-voxel vector path); W = 80
    # with 32-wide ROIs on multiples of 8 (8-voxel path); W = 61 clamps the last ROI to
    # x = 37 (one voxel per thread)
    g = torch.Generator(device=cuda_device).manual_seed(1)
    classes, spatial, roi = 5, (50, 47, width), (24, 24, rw)
    starts = roi_grid(spatial, roi, 0.5)
    acc = torch.randn((classes, *spatial), device=cuda_device, generator=g)
    want = acc.clone()
    for b0 in range(0, len(starts), 8):
        batch = starts[b0:b0 + 8]
        pred = torch.randn((len(batch), classes, *roi), device=cuda_device, generator=g).to(pred_dtype)
        _ops.require().roi_accumulate(acc, pred, [v for s in batch for v in s], list(roi))
        for i, (z, y, x) in enumerate(batch):
            want[:, z:z + 24, y:y + 24, x:x + rw] += pred[i].float()
    assert torch.equal(acc, want)


@pytest.mark.parametrize("width", [29, 32], ids=["scalar_x", "vec4_x"])
@pytest.mark.parametrize("classes", [14, 5])
def test_roi_argmax_and_normalize_bit_exact(classes, width, cuda_device):
    # W = 32: four voxels per thread (classes loaded four planes at a time, 5 leaves a
    # ragged last group); W = 29: one voxel per thread
    g = torch.Generator(device=cuda_device).manual_seed(2)
    spatial, roi = (40, 33, width), (16, 16, 16)
    acc = torch.randn((classes, *spatial), device=cuda_device, generator=g)
    acc[3, :5] = acc[classes - 1, :5]    # exact ties: the first index wins
    acc[2, 10:12, :4] = float("nan")     # NaN is the maximum
    counts = [torch.tensor(axis_counts(s, r, 0.5), device=cuda_device)
              for s, r in zip(spatial, roi)]
    cnt = counts[0][:, None, None] * counts[1][None, :, None] * counts[2][None, None, :]
    logits = torch.empty_like(acc)
    labels = torch.empty(spatial, dtype=torch.uint8, device=cuda_device)
    _ops.require().roi_normalize(logits, acc, *counts)
    _ops.require().roi_argmax(labels, acc, *counts)
    want = acc / cnt
    assert torch.equal(logits.nan_to_num(123.0), want.nan_to_num(123.0))
    assert torch.equal(labels, want.argmax(0).to(torch.uint8))


def test_roi_kernels_through_the_c_abi(cuda_device):
    vol = torch.rand((1, 40, 40, 40), device=cuda_device)
    starts = (torch.tensor([[0, 0, 0], [20, 20, 20]], dtype=torch.int64))
    import ctypes

    host = (ctypes.c_int64 * 6)(*starts.flatten().tolist())
    out = torch.empty((2, 1, 20, 20, 20), dtype=torch.float16, device=cuda_device)
    lib = _ops.capi()
    rc = lib.crumpet_roi_gather(ptr(out), DTYPE_CODE[torch.float16], ptr(vol),
                                DTYPE_CODE[torch.float32], 1, 40, 40, 40, host, 2, 20, 20, 20,
                                stream_ptr())
    assert rc == 0, _ops.last_error()
    assert torch.equal(out[1, 0], vol[0, 20:, 20:, 20:].half())
    acc = torch.zeros((1, 40, 40, 40), device=cuda_device)
    rc = lib.crumpet_roi_accumulate(ptr(acc), ptr(out), DTYPE_CODE[torch.float16], 1, 40, 40, 40,
                                    host, 2, 20, 20, 20, stream_ptr())
    assert rc == 0, _ops.last_error()
    assert torch.equal(acc[0, :20, :20, :20], out[0, 0].float())


@pytest.mark.parametrize("autocast", [True, False], ids=["fp16_autocast", "fp32"])
def test_inferer_matches_eager_sliding_window(autocast, cuda_device):
    """The whole ROI driver with a deterministic stand-in network: crop, forward,
    accumulate, normalise and arg-max are bit-identical to the eager passes."""
    torch.manual_seed(0)
    model = torch.nn.Conv3d(1, 6, 3, padding=1).to(cuda_device).eval()
    vol = torch.rand((1, 1, 70, 64, 58), device=cuda_device)
    inf = SlidingWindowInferer(model, (32, 32, 32), 4, 0.5, 6,
                               torch.float16 if autocast else None)
    with torch.no_grad():
        acc, _ = inf.accumulate(vol)
        logits = inf.logits(vol)
        labels = inf.segment(vol)
        want_acc, want_logits = _eager_accumulate(model, vol, (32, 32, 32), 4, 0.5, 6, autocast)
    assert torch.equal(acc, want_acc)
    assert torch.equal(logits, want_logits)
    assert torch.equal(labels, want_logits[0].argmax(0).to(torch.uint8))
