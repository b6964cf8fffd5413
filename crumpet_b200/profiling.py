"""Launch accounting and live per-kernel timing for the benchmark.

``counters`` counts crumpet_b200 kernel launches per op.  ``KernelTimer``
(enabled with ``with KernelTimer() as t:``) brackets every crumpet_b200 launch
with CUDA events on the launching stream and records the algorithmic work of
that launch, so the benchmark can report, inside the timed end-to-end region,
the attention kernel's achieved rates and every kernel's time against its ideal.
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


# the attention ops (their launches also feed the bench's attention roofline)
ATTENTION_OPS = ("fused_swin_attention", "swin_window_attention_qkv")


def _resolve(work: dict) -> dict:
    work = dict(work)
    masked, per_window = work.pop("mask_bytes", (0, 0))
    if isinstance(masked, torch.Tensor):
        masked = int(masked.sum())
    work["bytes"] = work.get("bytes", 0) + masked * per_window
    return work


class KernelTimer:
    """CUDA events around every crumpet_b200 launch while active, with the launch's
    algorithmic work ("bytes" moved, plus "flops" / "exps" for the attention)."""

    def __init__(self) -> None:
        self.records: list[tuple[torch.cuda.Event, torch.cuda.Event, str, dict]] = []

    def __enter__(self) -> "KernelTimer":
        _active.append(self)
        return self

    def __exit__(self, *exc) -> None:
        _active.remove(self)

    def summary(self, ops=ATTENTION_OPS) -> dict:
        """Launch count, total / average ms and per-launch average work of `ops`."""
        torch.cuda.synchronize()
        recs = [r for r in self.records if r[2] in ops]
        n = len(recs)
        if n == 0:
            return {"launches": 0}
        ms = sum(s.elapsed_time(e) for s, e, _, _ in recs)
        tot = collections.Counter()
        for _, _, _, work in recs:
            tot.update(_resolve(work))
        out = {"launches": n, "total_ms": ms, "avg_ms": ms / n}
        out.update({k: v / n for k, v in tot.items()})  # per-launch averages
        return out

    def by_op(self) -> dict:
        """Per op: launches, total ms and total work; "sizes" splits the same totals by
        the launch's algorithmic bytes (one entry per distinct launch shape, e.g. per
        Swin stage)."""
        torch.cuda.synchronize()
        res: dict = {}
        for s, e, op, work in self.records:
            d = res.setdefault(op, {"launches": 0, "ms": 0.0, "bytes": 0, "exps": 0,
                                    "sizes": {}})
            ms = s.elapsed_time(e)
            w = _resolve(work)
            for tgt in (d, d["sizes"].setdefault(int(w.get("bytes", 0)),
                                                 {"launches": 0, "ms": 0.0, "bytes": 0,
                                                  "exps": 0})):
                tgt["launches"] += 1
                tgt["ms"] += ms
                tgt["bytes"] += w.get("bytes", 0)
                tgt["exps"] += w.get("exps", 0)
        return res


class suspended:
    """Within this context no timer records launches, and the launch counts it adds are
    handed back as ``delta`` and removed from ``counters``: used while a CUDA graph is
    captured, where nothing runs yet (each replay adds ``delta`` with ``count_replay``)."""

    def __enter__(self) -> "suspended":
        self._timers = list(_active)
        _active.clear()
        self._before = collections.Counter(counters)
        self.delta: "collections.Counter[str]" = collections.Counter()
        return self

    def __exit__(self, *exc) -> None:
        self.delta = counters - self._before
        counters.clear()
        counters.update(self._before)
        _active.extend(self._timers)


def count_replay(delta: "collections.Counter[str]") -> None:
    counters.update(delta)


def kernel_begin(op: str, work):
    """Start-of-launch hook; `work` is a dict or a callable returning one (evaluated only
    while a timer is active).  Returns a token for kernel_end."""
    if not _active:
        return None
    start = torch.cuda.Event(enable_timing=True)
    start.record()
    return (start, op, work() if callable(work) else work)


def kernel_end(token) -> None:
    if token is None:
        return
    start, op, work = token
    end = torch.cuda.Event(enable_timing=True)
    end.record()
    for t in _active:
        t.records.append((start, end, op, work))
