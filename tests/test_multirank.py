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
from crumpet_b200.inferer import SlidingWindowInferer

VOLUME = (1, 1, 96, 64, 64)


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _model():
    torch.manual_seed(0)
    return swin_unetr.SwinUNETR(1, 3, 12, depths=(1, 1, 1, 1)).eval()


def _volume():
    g = torch.Generator().manual_seed(1)
    return torch.rand(VOLUME, generator=g)


def _worker(rank, world, port, fail_rank, queue):
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
        logits = inf.logits(_volume())
        queue.put((rank, "ok", None if logits is None else logits.numpy()))
    except Exception as exc:  # reported to the parent, never swallowed
        queue.put((rank, "error", repr(exc)[:200]))
    finally:
        try:
            dist.destroy_process_group()
        except Exception:
            pass


def _run(world, fail_rank=-1):
    ctx = mp.get_context("spawn")
    queue = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, fail_rank, queue)) for r in range(world)]
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


def test_roi_sharded_reduce_matches_single_process():
    single = SlidingWindowInferer(_model(), (64, 64, 64), 1, 0.5, num_classes=3,
                                  autocast_dtype=None)
    with torch.no_grad():
        want = single.logits(_volume()).numpy()
    results = _run(2)
    assert results[0][0] == "ok" and results[1][0] == "ok"
    assert results[1][1] is None  # only rank 0 holds the merged logits
    assert abs(results[0][1] - want).max() < 1e-5


def test_failing_rank_surfaces_on_rank0():
    results = _run(2, fail_rank=1)
    assert results[1][0] == "error" and "injected" in results[1][1]
    # rank 0's reduce cannot complete: it must end with an error, not hang
    assert results[0][0] == "error"
