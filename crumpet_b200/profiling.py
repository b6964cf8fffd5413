"""Launch accounting and live per-kernel timing for the benchmark.

``counters`` counts crumpet_b200 kernel launches per op.  ``KernelTimer``
(enabled with ``with KernelTimer() as t:``) brackets every fused window
attention launch with CUDA events on the launching stream and records the
algorithmic work of that launch, so the benchmark can report the attention
kernel's achieved bandwidth / FLOP rate inside the timed end-to-end region.
"""

from __future__ import annotations

import collections

import torch

counters: "collections.Counter[str]" = collections.Counter()
_active: list["KernelTimer"] = []


def count(op: str, n: int = 1) -> None:
    counters[op] += n


def total_launches() -> int:
    return sum(counters.values())


class KernelTimer:
    def __init__(self) -> None:
        self.records: list[tuple[torch.cuda.Event, torch.cuda.Event, dict]] = []

    def __enter__(self) -> "KernelTimer":
        _active.append(self)
        return self

    def __exit__(self, *exc) -> None:
        _active.remove(self)

    def summary(self) -> dict:
        torch.cuda.synchronize()
        n = len(self.records)
        if n == 0:
            return {"launches": 0}
        ms = sum(s.elapsed_time(e) for s, e, _ in self.records)
        tot = collections.Counter()
        for _, _, work in self.records:
            work = dict(work)
            masked, per_window = work.pop("mask_bytes", (0, 0))
            if isinstance(masked, torch.Tensor):
                masked = int(masked.sum())
            work["bytes"] = work.get("bytes", 0) + masked * per_window
            tot.update(work)
        out = {"launches": n, "total_ms": ms, "avg_ms": ms / n}
        out.update({k: v / n for k, v in tot.items()})  # per-launch averages
        return out


def attention_begin(work: dict):
    """Start-of-launch hook for fused attention; returns a token for attention_end."""
    if not _active:
        return None
    start = torch.cuda.Event(enable_timing=True)
    start.record()
    return (start, work)


def attention_end(token) -> None:
    if token is None:
        return
    start, work = token
    end = torch.cuda.Event(enable_timing=True)
    end.record()
    for t in _active:
        t.records.append((start, end, work))
