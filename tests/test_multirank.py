"""ROI-sharded sliding-window inference over gloo ranks on the CPU (world size 2):
the reduced result equals the single-process result, and a failing rank surfaces as
an error on rank 0 within the process-group timeout instead of hanging it."""

from __future__ import annotations

import datetime
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from crumpet_b200 import swin_unetr
from crumpet_b200.inferer import SlidingWindowInferer, roi_grid, shard_plan

VOLUME = (1, 1, 96, 64, 64)
TALL = (1, 1, 160, 64, 64)  # four ROI rows along z: three ranks exchange two halos


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _model():
    torch.manual_seed(0)
    return swin_unetr.SwinUNETR(1, 3, 12, depths=(1, 1, 1, 1)).eval()


def _volume(shape=VOLUME):
    g = torch.Generator().manual_seed(1)
    return torch.rand(shape, generator=g)


def _worker(rank, world, port, fail_rank, queue, shape=VOLUME):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.set_num_threads(1)
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=5))
    try:
        inf = SlidingWindowInferer(_model(), (64, 64, 64), 1, 0.5, num_classes=3,
                                   autocast_dtype=None, rank=rank, world=world)
        if rank == fail_rank:
            raise RuntimeError("injected failure on this rank")
        vol = _volume(shape)
        logits = inf.logits(vol)
        labels = inf.segment(vol)
        queue.put((rank, "ok", None if logits is None else (logits.numpy(), labels.numpy(),
                                                            inf.exchanged_bytes)))
    except Exception as exc:  # reported to the parent, never swallowed
        queue.put((rank, "error", repr(exc)[:200]))
    finally:
        try:
            dist.destroy_process_group()
        except Exception:
            pass


def _run(world, fail_rank=-1, shape=VOLUME):
    ctx = mp.get_context("spawn")
    queue = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, fail_rank, queue, shape))
             for r in range(world)]
    for p in procs:
        p.start()
    results = {}
    for _ in range(world):
        rank, status, payload = queue.get(timeout=120)
        results[rank] = (status, payload)
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    return results


def _single(shape):
    single = SlidingWindowInferer(_model(), (64, 64, 64), 1, 0.5, num_classes=3,
                                  autocast_dtype=None)
    with torch.no_grad():
        return single.logits(_volume(shape)).numpy(), single.segment(_volume(shape)).numpy()


@pytest.mark.parametrize("world,shape", [(2, VOLUME), (3, TALL)], ids=["w2", "w3_tall"])
def test_roi_sharded_slabs_match_single_process(world, shape):
    want_logits, want_labels = _single(shape)
    results = _run(world, shape=shape)
    assert all(results[r][0] == "ok" for r in range(world)), results
    assert all(results[r][1] is None for r in range(1, world))  # rank 0 alone holds the result
    logits, labels, exchanged = results[0][1]
    assert abs(logits - want_logits).max() < 1e-5
    assert (labels == want_labels).all()
    # only halo planes crossed ranks: less than one whole accumulator
    assert 0 < exchanged < 3 * shape[2] * shape[3] * shape[4] * 4


@pytest.mark.parametrize("world", range(1, 9))
def test_shard_plan_partitions_the_volume(world):
    """The cfg5 grid (512 x 512 x 224 volume, 96^3 ROIs at 0.5 overlap): the ROI ranges
    partition the grid, the owned ranges partition [0, 512), each owned range lies in its
    owner's slab, and every slab is much smaller than the volume for world >= 4."""
    starts = roi_grid((512, 512, 224), (96, 96, 96), 0.5)
    plan = shard_plan(starts, world, 512, 96)
    assert [roi for sh in plan for roi in sh.rois] == starts
    edges = [sh.own for sh in plan]
    assert edges[0][0] == 0 and edges[-1][1] == 512
    assert all(edges[r][1] == edges[r + 1][0] for r in range(world - 1))
    for sh in plan:
        assert sh.slab[0] <= sh.own[0] and sh.own[1] <= sh.slab[1]
        for z, _, _ in sh.rois:
            assert sh.slab[0] <= z and z + 96 <= sh.slab[1]
    if world >= 4:
        assert max(sh.slab[1] - sh.slab[0] for sh in plan) <= 240


def test_failing_rank_surfaces_on_rank0():
    results = _run(2, fail_rank=1)
    assert results[1][0] == "error" and "injected" in results[1][1]
    # rank 0's reduce cannot complete: it must end with an error, not hang
    assert results[0][0] == "error"
