"""ROI sharding over two GPUs with NCCL (skipped with fewer than two): the slab
accumulators, the halo exchange and the label gather give rank 0 the single-process
result.  The host-side logic is covered on the CPU with gloo ranks
(tests/test_multirank.py); this runs the same path with the CUDA kernels and NCCL."""

from __future__ import annotations

import datetime
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu

SHAPE = (1, 1, 288, 192, 96)  # 5 x 3 x 1 ROIs of 96^3


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _model(device):
    from crumpet_b200 import swin_unetr

    torch.manual_seed(0)
    return swin_unetr.SwinUNETR(1, 14, 48).to(device).eval()


def _worker(rank, world, port, queue):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    import crumpet_b200 as crumpet
    from crumpet_b200 import swin_unetr
    from crumpet_b200.inferer import SlidingWindowInferer, synthetic_volume

    device = torch.device("cuda", rank)
    torch.cuda.set_device(device)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=device,
                            timeout=datetime.timedelta(seconds=60))
    try:
        crumpet.patch_monai_swin_unetr(swin_unetr)
        host = synthetic_volume(SHAPE).pin_memory()
        inf = SlidingWindowInferer(_model(device), (96, 96, 96), 4, 0.5, 14, torch.float16,
                                   rank, world, device=device)
        labels = inf.segment(host)  # host volume: each rank copies its own slab
        logits = inf.logits(host.to(device))
        torch.cuda.synchronize()
        queue.put((rank, "ok", None if labels is None else
                   (labels.cpu(), logits.cpu(), inf.exchanged_bytes)))
    except Exception as exc:
        queue.put((rank, "error", repr(exc)[:300]))
    finally:
        crumpet.unpatch_monai_swin_unetr()
        dist.destroy_process_group()


def test_two_gpu_slabs_match_single_gpu():
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    import crumpet_b200 as crumpet
    from crumpet_b200 import swin_unetr
    from crumpet_b200.inferer import SlidingWindowInferer, synthetic_volume

    ctx = mp.get_context("spawn")
    queue = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, queue)) for r in range(2)]
    for p in procs:
        p.start()
    results = dict((r, (s, payload)) for r, s, payload in (queue.get(timeout=300) for _ in range(2)))
    for p in procs:
        p.join(timeout=60)
    assert results[0][0] == "ok" and results[1][0] == "ok", results
    labels, logits, exchanged = results[0][1]

    device = torch.device("cuda", 0)
    crumpet.patch_monai_swin_unetr(swin_unetr)
    try:
        single = SlidingWindowInferer(_model(device), (96, 96, 96), 4, 0.5, 14, torch.float16)
        vol = synthetic_volume(SHAPE).to(device)
        want_logits = single.logits(vol).cpu()
        want_labels = single.segment(vol).cpu()
    finally:
        crumpet.unpatch_monai_swin_unetr()
    # the sums meet in another order across ranks: equal to fp32 rounding
    assert torch.allclose(logits, want_logits, atol=1e-5, rtol=1e-5)
    assert (labels == want_labels).float().mean().item() >= 0.9999
    assert 0 < exchanged < 14 * 288 * 192 * 96 * 4
