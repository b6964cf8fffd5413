"""Sliding-window ROI inference for Swin UNETR, sharded by ROI across GPUs.

Semantics of MONAI's ``sliding_window_inference`` with ``mode="constant"``
(the driver of the reference's end-to-end runs, torch-ext/crumpet/demo_btcv.py:98-129):
ROIs of ``roi_size`` at a stride of ``int(roi * (1 - overlap))`` per axis, the
last ROI of every axis clamped to end at the volume edge, ``sw_batch_size``
ROIs per forward, predictions summed into a float32 accumulator and divided
by the per-voxel ROI count.

On CUDA the crop, accumulate and normalise/arg-max passes run as crumpet_b200
kernels (``roi_gather``, ``roi_accumulate``, ``roi_argmax`` / ``roi_normalize``):
one launch per ROI batch instead of a copy, a cast and an add per ROI, with the
same fp32 additions in the same order, so the results are bit-identical to the
eager loop; CPU tensors take the eager torch path.

With ``cuda_graphs=True`` each ROI batch's network forward is a CUDA graph
replay: one graph per batch size, captured on first use (after two warm-up
forwards on a side stream) with the crop kernel writing straight into the
graph's input buffer and the accumulate kernel reading its output buffer.  The
crop and accumulate launches stay outside the graph (their ROI starts change
from batch to batch).  Replays run the same kernels on the same data as the eager
forward, so the results are identical; what goes away is the host's per-launch
work between the GPU's kernels.  The model must be fixed (weights are read
in place by the replays) and its forward free of host synchronisation.  A graph
holds the forward as it was captured -- including whether crumpet_b200's patch
was applied -- so after changing the model (patching or unpatching it, replacing
modules or parameter tensors) call ``reset_graphs()``.

Multi-GPU: one process per GPU, nothing exchanged inside the model.  Rank r runs the
r-th contiguous 1/world of the ROI grid (balanced to one ROI), cut into batches.  The
grid is ordered with z outermost, so a rank's ROIs cover a z-slab of the volume: the
rank accumulates into a slab-sized buffer only.  The output z-axis is cut into
disjoint ranges, one owned by each rank (from the z of its first ROI to that of the
next rank's first ROI), each inside its owner's slab.  After accumulation every rank
sends the parts of its slab that lie in other ranks' ranges to their owners (NCCL
point-to-point: only the halo planes where neighbouring slabs overlap), each owner
adds them into its range in rank order, normalises it and takes its arg-max, and
rank 0 gathers the uint8 labels.  With a host (CPU) volume and a CUDA ``device``,
each rank copies only its slab of the volume to its GPU.
"""

from __future__ import annotations

import itertools
from dataclasses import dataclass
from typing import Sequence

import torch
import torch.distributed as dist

from . import _ops
from . import cache as _mask_cache
from . import profiling as _prof


def axis_starts(size: int, roi: int, overlap: float) -> list[int]:
    """Start offsets of the ROIs along one axis."""
    if size <= roi:
        return [0]
    interval = max(int(roi * (1.0 - overlap)), 1)
    count = -(-(size - roi) // interval) + 1
    return [min(i * interval, size - roi) for i in range(count)]


def roi_grid(spatial: Sequence[int], roi: Sequence[int], overlap: float) -> list[tuple[int, int, int]]:
    starts = [axis_starts(s, r, overlap) for s, r in zip(spatial, roi)]
    return list(itertools.product(*starts))


def axis_counts(size: int, roi: int, overlap: float) -> list[float]:
    """Number of ROIs covering each coordinate of one axis (the count map factorises)."""
    counts = [0.0] * size
    for s in axis_starts(size, roi, overlap):
        for i in range(s, min(s + roi, size)):
            counts[i] += 1.0
    return counts


@dataclass(frozen=True)
class RankShard:
    """One rank's share of a sliding-window pass along z (the grid's outer axis)."""

    rois: tuple  # its ROI starts (absolute (z, y, x))
    slab: tuple  # [z0, z1): the planes its ROIs read and write
    own: tuple   # [a, b): the planes whose normalised logits / labels it produces


def shard_plan(starts, world: int, depth: int, roi_d: int) -> list[RankShard]:
    """Contiguous balanced ROI ranges per rank, their z-slabs, and a partition of
    [0, depth) into owned ranges with each range inside its owner's slab."""
    n = len(starts)
    bounds = [r * n // world for r in range(world + 1)]
    first_z = [starts[bounds[r]][0] if bounds[r] < n else depth for r in range(world)]
    plan = []
    for r in range(world):
        mine = tuple(starts[bounds[r]:bounds[r + 1]])
        a = 0 if r == 0 else first_z[r]
        b = depth if r == world - 1 else first_z[r + 1]
        if mine:
            z0 = min(st[0] for st in mine)
            z1 = min(depth, max(st[0] for st in mine) + roi_d)
        else:
            z0 = z1 = a
        # the buffer must also cover the owned range (it does whenever consecutive ROI
        # z-starts are at most a ROI apart, which every overlap >= 0 grid satisfies)
        plan.append(RankShard(mine, (min(z0, a), max(z1, b)) if b > a else (z0, z1), (a, b)))
    return plan


def _intersect(p, q):
    lo, hi = max(p[0], q[0]), min(p[1], q[1])
    return (lo, hi) if hi > lo else None


class SlidingWindowInferer:
    """Runs ``model`` over a ``[1, C_in, D, H, W]`` volume in ROI batches.

    ``rank``/``world`` select this process's share of the ROI batches (a
    single-process run is rank 0 of 1).  ``autocast_dtype`` wraps every
    forward in ``torch.autocast`` (fp16 in the benchmark, as in the
    reference's runs).  ``cuda_graphs`` replays each batch's forward from a
    captured CUDA graph (CUDA volumes only; see the module docstring).
    """

    def __init__(self, model: torch.nn.Module, roi_size=(96, 96, 96), sw_batch_size: int = 4,
                 overlap: float = 0.5, num_classes: int = 14,
                 autocast_dtype: torch.dtype | None = torch.float16, rank: int = 0, world: int = 1,
                 group=None, cuda_graphs: bool = False, device: torch.device | str | None = None):
        self.model = model
        self.device = None if device is None else torch.device(device)
        self.roi = tuple(int(r) for r in roi_size)
        self.sw_batch = int(sw_batch_size)
        self.overlap = float(overlap)
        self.num_classes = int(num_classes)
        self.autocast_dtype = autocast_dtype
        self.rank = rank
        self.world = world
        self.group = group
        self.cuda_graphs = bool(cuda_graphs)
        self._count_cache: dict = {}
        self._graphs: dict = {}
        self._staging: dict = {}

    def rois(self, spatial) -> list[tuple[int, int, int]]:
        return roi_grid(spatial, self.roi, self.overlap)

    def plan(self, spatial) -> list[RankShard]:
        """Every rank's ROIs, z-slab and owned z-range (see :func:`shard_plan`)."""
        key = ("plan", tuple(spatial))
        if key not in self._count_cache:
            self._count_cache[key] = shard_plan(self.rois(spatial), self.world,
                                                int(spatial[0]), self.roi[0])
        return self._count_cache[key]

    def my_batches(self, spatial) -> list[list[tuple[int, int, int]]]:
        """This rank's ROI batches: a contiguous range of the ROI grid (ranks differ by at
        most one ROI, and a batch's ROIs stay spatially adjacent), cut into the fewest
        batches of at most sw_batch ROIs, as equal in size as possible (50 ROIs in batches
        of 8 run as 8 + 6 x 7 rather than 6 x 8 + 2: a two-ROI batch leaves the GPU idle
        for much of its forward).  The ROI order, and so the order of the additions into
        each voxel, does not depend on where the batches are cut."""
        mine = list(self.plan(spatial)[self.rank].rois)
        if not mine:
            return []
        count = -(-len(mine) // self.sw_batch)
        small, extra = divmod(len(mine), count)
        out, i = [], 0
        for k in range(count):
            size = small + (1 if k < extra else 0)
            out.append(mine[i:i + size])
            i += size
        return out

    def _count_map(self, spatial, device) -> torch.Tensor:
        key = (tuple(spatial), device)
        if key not in self._count_cache:
            cnt = torch.zeros((1, 1, *spatial), dtype=torch.float32, device=device)
            rd, rh, rw = self.roi
            for z, y, x in self.rois(spatial):
                cnt[..., z:z + rd, y:y + rh, x:x + rw] += 1.0
            self._count_cache[key] = cnt
        return self._count_cache[key]

    def _axis_counts(self, spatial, device) -> list[torch.Tensor]:
        key = ("axes", tuple(spatial), device)
        if key not in self._count_cache:
            self._count_cache[key] = [
                torch.tensor(axis_counts(s, r, self.overlap), dtype=torch.float32, device=device)
                for s, r in zip(spatial, self.roi)]
        return self._count_cache[key]

    def _window_dtype(self, volume: torch.Tensor) -> torch.dtype:
        # under autocast the first convolutions cast their input to the autocast
        # dtype; the crop writes that dtype directly (same rounding)
        return self.autocast_dtype if self.autocast_dtype is not None else volume.dtype

    def _gather(self, volume: torch.Tensor, batch, out: torch.Tensor | None = None) -> torch.Tensor:
        rd, rh, rw = self.roi
        if not volume.is_cuda:
            return torch.cat([volume[..., z:z + rd, y:y + rh, x:x + rw] for z, y, x in batch])
        if out is None:
            out = torch.empty((len(batch), volume.shape[1], rd, rh, rw),
                              dtype=self._window_dtype(volume), device=volume.device)
        token = _prof.kernel_begin("roi_gather", lambda: {
            "bytes": out.numel() * (out.element_size() + volume.element_size())})
        _ops.require().roi_gather(out, volume[0].contiguous(), [v for st in batch for v in st],
                                  list(self.roi))
        _prof.count("roi_gather")
        _prof.kernel_end(token)
        return out

    def _forward(self, window: torch.Tensor, cache: bool = True) -> torch.Tensor:
        if self.autocast_dtype is None:
            return self.model(window)
        with torch.autocast("cuda", dtype=self.autocast_dtype, cache_enabled=cache):
            return self.model(window)

    def reset_graphs(self) -> None:
        """Drop the captured graphs (and their memory pool); the next batches capture anew."""
        self._graphs.clear()

    def _graph(self, n: int, volume: torch.Tensor):
        """(graph, input buffer, output buffer, launch counts of one replay) for batches
        of n ROIs, captured on first use."""
        dtype = self._window_dtype(volume)
        key = (n, int(volume.shape[1]), dtype, volume.device)
        if key not in self._graphs:
            static_in = torch.zeros((n, volume.shape[1], *self.roi), dtype=dtype,
                                    device=volume.device)
            # warm-up on a side stream (library handles, workspaces, the mask cache)
            side = torch.cuda.Stream(volume.device)
            side.wait_stream(torch.cuda.current_stream(volume.device))
            with torch.cuda.stream(side), _prof.suspended():
                for _ in range(2):
                    self._forward(static_in, cache=False)
            torch.cuda.current_stream(volume.device).wait_stream(side)
            graph = torch.cuda.CUDAGraph()
            with _prof.suspended() as launches, torch.cuda.graph(graph):
                static_out = self._forward(static_in, cache=False)
            # The replays read every tensor the capture read, by address.  Masks taken
            # from the mask cache (the dense-mask and unpatched paths) could be evicted
            # or cleared later and their memory reused, so the graph entry holds them.
            held = _mask_cache.cached_masks()
            self._graphs[key] = (graph, static_in, static_out, launches.delta, held)
        return self._graphs[key][:4]

    def _stage(self, volume: torch.Tensor, shard: RankShard) -> tuple[torch.Tensor, int]:
        """The tensor the ROI crops read and the z of its first plane: the volume itself
        when it is already on the compute device; a host volume with a CUDA ``device``
        has this rank's slab copied (asynchronously from pinned memory) into a device
        buffer that later calls reuse."""
        dev = self.device if self.device is not None else volume.device
        if dev.type != "cuda" or volume.device == dev:
            return volume, 0
        z0, z1 = shard.slab
        shape = (*volume.shape[:2], z1 - z0, *volume.shape[3:])
        key = (shape, volume.dtype, dev)
        buf = self._staging.get(key)
        if buf is None:
            buf = self._staging[key] = torch.empty(shape, dtype=volume.dtype, device=dev)
        buf.copy_(volume[:, :, z0:z1], non_blocking=True)
        return buf, z0

    def staged_bytes(self, spatial, channels: int = 1, itemsize: int = 4) -> int:
        """Host-to-device bytes one call copies on this rank for a host volume."""
        z0, z1 = self.plan(spatial)[self.rank].slab
        return channels * (z1 - z0) * int(spatial[1]) * int(spatial[2]) * itemsize

    @torch.no_grad()
    def accumulate(self, volume: torch.Tensor) -> tuple[torch.Tensor, int]:
        """This rank's summed predictions over its z-slab, fp32 [1, classes, z1 - z0, H, W]
        (the whole volume when one process covers every ROI), and its ROI count."""
        spatial = tuple(int(s) for s in volume.shape[2:])
        shard = self.plan(spatial)[self.rank]
        src, src_z = self._stage(volume, shard)
        base = shard.slab[0]
        rd, rh, rw = self.roi
        acc = torch.zeros((1, self.num_classes, shard.slab[1] - base, *spatial[1:]),
                          dtype=torch.float32, device=src.device)
        done = 0
        for batch in self.my_batches(spatial):
            crops = [(z - src_z, y, x) for z, y, x in batch]
            if self.cuda_graphs and src.is_cuda:
                # capture and replay on the volume's device and its current stream
                with torch.cuda.device(src.device):
                    graph, static_in, pred, launches = self._graph(len(batch), src)
                    self._gather(src, crops, out=static_in)
                    graph.replay()
                _prof.count_replay(launches)
            else:
                pred = self._forward(self._gather(src, crops))
            into = [(z - base, y, x) for z, y, x in batch]
            if src.is_cuda:
                token = _prof.kernel_begin(
                    "roi_accumulate", lambda: {"bytes": _accumulate_bytes(pred, into, self.roi)})
                _ops.require().roi_accumulate(acc[0], pred.contiguous(),
                                              [v for st in into for v in st], list(self.roi))
                _prof.count("roi_accumulate")
                _prof.kernel_end(token)
            else:
                for i, (z, y, x) in enumerate(into):
                    acc[0, :, z:z + rd, y:y + rh, x:x + rw] += pred[i].float()
            done += len(batch)
        return acc, done

    def _check_kernels(self, device: torch.device) -> None:
        """Raise when a crumpet_b200 kernel gave up on a bounded wait while this volume ran
        (its output is then incomplete).  With several ranks every rank learns of a
        failure on any of them through one small all-reduce, so all of them raise
        together instead of leaving the others waiting in the next collective."""
        bad = device_error(device)
        if self.world > 1:
            flag = torch.tensor([bad], dtype=torch.int32, device=device)
            dist.all_reduce(flag, op=dist.ReduceOp.MAX, group=self.group)
            bad = int(flag.item())
        if bad:
            raise RuntimeError(
                f"crumpet_b200 kernel reported device error {bad} during sliding-window "
                "inference (a bounded wait expired or an input was out of range); the "
                "accumulated predictions are incomplete")

    def _peer(self, r: int) -> int:
        return r if self.group is None else dist.get_global_rank(self.group, r)

    def _exchange(self, acc: torch.Tensor, plan: list[RankShard]) -> None:
        """Send this rank's slab planes that other ranks own to them, and add the planes of
        its own range that other ranks' slabs produced (in rank order)."""
        me = plan[self.rank]
        base = me.slab[0]
        ops, incoming = [], []
        for r, sh in enumerate(plan):
            ov = _intersect(sh.own, me.slab) if r != self.rank else None
            if ov is not None:
                part = acc[0, :, ov[0] - base:ov[1] - base].contiguous()
                ops.append(dist.P2POp(dist.isend, part, self._peer(r), self.group))
        for q, sh in enumerate(plan):
            ov = _intersect(me.own, sh.slab) if q != self.rank else None
            if ov is not None:
                buf = torch.empty((acc.shape[1], ov[1] - ov[0], *acc.shape[3:]),
                                  dtype=acc.dtype, device=acc.device)
                ops.append(dist.P2POp(dist.irecv, buf, self._peer(q), self.group))
                incoming.append((ov, buf))
        if ops:
            for req in dist.batch_isend_irecv(ops):
                req.wait()
        for ov, buf in incoming:
            acc[0, :, ov[0] - base:ov[1] - base] += buf
        # bytes this rank moved over the interconnect for this volume (sent + received)
        self.exchanged_bytes = sum(op.tensor.numel() * op.tensor.element_size() for op in ops)

    def _merged(self, volume: torch.Tensor):
        """(this rank's owned z-range, the summed predictions over it [1, classes, b - a,
        H, W]) with every rank's contributions added."""
        spatial = tuple(int(s) for s in volume.shape[2:])
        acc, _ = self.accumulate(volume)
        self._check_kernels(acc.device)
        plan = self.plan(spatial)
        self.exchanged_bytes = 0
        if self.world > 1:
            self._exchange(acc, plan)
        me = plan[self.rank]
        a, b = me.own
        base = me.slab[0]
        if (a, b) == (base, base + acc.shape[2]):
            return (a, b), acc
        return (a, b), acc[:, :, a - base:b - base].contiguous()

    def _to_rank0(self, part: torch.Tensor, spatial, zdim: int):
        """Assemble the owned ranges of every rank along ``zdim`` on rank 0 (None elsewhere)."""
        if self.world == 1:
            return part
        plan = self.plan(spatial)
        if self.rank != 0:
            if plan[self.rank].own[1] > plan[self.rank].own[0]:
                # batched, so NCCL does not serialise it with the other ranks' sends
                op = dist.P2POp(dist.isend, part.contiguous(), self._peer(0), self.group)
                for req in dist.batch_isend_irecv([op]):
                    req.wait()
            return None
        shape = list(part.shape)
        shape[zdim] = int(spatial[0])
        full = torch.empty(shape, dtype=part.dtype, device=part.device)
        a, b = plan[0].own
        full.narrow(zdim, a, b - a).copy_(part)
        ops, bufs = [], []
        for q in range(1, self.world):
            aq, bq = plan[q].own
            if bq > aq:
                shp = list(part.shape)
                shp[zdim] = bq - aq
                buf = torch.empty(shp, dtype=part.dtype, device=part.device)
                ops.append(dist.P2POp(dist.irecv, buf, self._peer(q), self.group))
                bufs.append((aq, bq, buf))
        if ops:
            for req in dist.batch_isend_irecv(ops):
                req.wait()
        for aq, bq, buf in bufs:
            full.narrow(zdim, aq, bq - aq).copy_(buf)
        return full

    @torch.no_grad()
    def logits(self, volume: torch.Tensor) -> torch.Tensor | None:
        """Averaged logits [1, classes, D, H, W] on rank 0 (None on other ranks)."""
        spatial = tuple(int(s) for s in volume.shape[2:])
        (a, b), acc = self._merged(volume)
        if b == a:  # this rank owns no planes (more ranks than ROI rows)
            out = acc[:, :, :0]
        elif not acc.is_cuda:
            out = acc / self._count_map(spatial, acc.device)[:, :, a:b]
        else:
            out = torch.empty_like(acc)
            count_d, count_h, count_w = self._axis_counts(spatial, acc.device)
            token = _prof.kernel_begin("roi_normalize",
                                       lambda: {"bytes": 2 * acc.numel() * acc.element_size()})
            _ops.require().roi_normalize(out[0], acc[0], count_d[a:b], count_h, count_w)
            _prof.count("roi_normalize")
            _prof.kernel_end(token)
        return self._to_rank0(out, spatial, 2)

    @torch.no_grad()
    def segment(self, volume: torch.Tensor) -> torch.Tensor | None:
        """uint8 label map [D, H, W] on rank 0 (None on other ranks): the arg-max of
        the averaged logits."""
        spatial = tuple(int(s) for s in volume.shape[2:])
        (a, b), acc = self._merged(volume)
        if b == a:  # this rank owns no planes (more ranks than ROI rows)
            labels = torch.empty((0, *spatial[1:]), dtype=torch.uint8, device=acc.device)
        elif not acc.is_cuda:
            logits = acc / self._count_map(spatial, acc.device)[:, :, a:b]
            labels = logits[0].argmax(dim=0).to(torch.uint8)
        else:
            labels = torch.empty((b - a, *spatial[1:]), dtype=torch.uint8, device=acc.device)
            count_d, count_h, count_w = self._axis_counts(spatial, acc.device)
            token = _prof.kernel_begin("roi_argmax", lambda: {
                "bytes": acc.numel() * acc.element_size() + labels.numel()})
            _ops.require().roi_argmax(labels, acc[0], count_d[a:b], count_h, count_w)
            _prof.count("roi_argmax")
            _prof.kernel_end(token)
        return self._to_rank0(labels, spatial, 0)


def device_error(device: torch.device) -> int:
    """The crumpet_b200 device error word for CUDA work (0 = healthy), cleared after the
    read; 0 for CPU devices.  Reading it waits for the device."""
    if device.type != "cuda":
        return 0
    from . import device_status

    return device_status(clear=True)


def _accumulate_bytes(pred: torch.Tensor, batch, roi) -> int:
    """Algorithmic bytes of one accumulate launch: the predictions once, and a read and
    a write of the fp32 accumulator over the batch's bounding box."""
    box = 1
    for a in range(3):
        lo = min(st[a] for st in batch)
        hi = max(st[a] for st in batch) + roi[a]
        box *= hi - lo
    return pred.numel() * pred.element_size() + 8 * int(pred.shape[1]) * box


def synthetic_volume(shape=(1, 1, 512, 512, 224), seed: int = 0) -> torch.Tensor:
    """Uniform [-1000, 1000] intensities clipped and scaled to [0, 1] (CPU, fp32)."""
    g = torch.Generator().manual_seed(seed)
    x = torch.rand(shape, generator=g) * 2000.0 - 1000.0
    return ((x.clamp(-1000.0, 1000.0) + 1000.0) / 2000.0).contiguous()
