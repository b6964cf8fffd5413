#!/usr/bin/env python
"""End-to-end benchmark: Swin UNETR 96^3 sliding-window inference, ROIs/s.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Workload: MONAI-architecture Swin UNETR (in 1, out 14,
feature 48, depths 2,2,2,2, heads 3,6,12,24, window 7, patch 2), random init
(seed 0), fp16 autocast, sliding-window inference with 96^3 ROIs at 0.5
overlap over a synthetic 1x1x512x512x224 volume of uniform[-1000, 1000]
intensities scaled to [0, 1]: 400 ROIs per step, batches of 8, arg-max
segmentation.  A step is one full volume.  With N GPUs (torchrun, one process
per GPU) each rank takes a contiguous, balanced 1/N of the ROI grid, accumulates
over the z-slab its ROIs cover, exchanges only the overlapping halo planes with
its neighbours (NCCL point-to-point), takes the arg-max of the z-range it owns, and
rank 0 gathers the uint8 labels (total work fixed: strong scaling).

``value``: ROIs/s with the volume resident in HBM and the segmentation left
on the device, CUDA-event timed, max over ranks.  ``e2e``: the same through
``segment(host_volume)`` -- each rank copies its slab from pinned host memory --
with the segmentation copied back inside every step.  Both run each ROI batch's network forward as a CUDA graph replay
(``--eager``: without graphs).  The 3.3 GB accumulator and 235 MB volume exceed
L2, so no flush is needed between steps.  Also reported: the same steps on the
eager forward with CUDA events around every crumpet_b200 launch (``eager``), and
from that pass the fused attention kernel's rates (roofline) and every
crumpet_b200 kernel against its roofline (crumpet_kernels: event time vs
algorithmic bytes at the measured HBM rate, or the SFU rate for the attention's
exponentials),
stand-alone per-kernel HBM GB/s at the BASELINE stage-0 sizes, clocks sampled
during the timed region, and the CPU eager baseline (the unpatched network on
the host cores).

``--impl reference``: times the reference path on the CPU -- the eager,
unpatched network (torch.roll / window partition / eager attention, i.e. the
MONAI code path crumpet patches) on one ROI per step with all host threads.
"""

from __future__ import annotations

import argparse
import datetime
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "Swin UNETR 96³ ROIs/s (fp16, 1/2/4/8 B200); per-kernel HBM GB/s vs peak"
UNIT = "ROIs/s"
PER_KERNEL_PASS = ("per-kernel pass: the timed steps repeated on the eager forward with CUDA "
                   "events around every crumpet_b200 launch on its stream (the timed steps "
                   "replay CUDA graphs of the same kernels, which cannot be bracketed per kernel)")
FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0,
                  "source": "fallback"}


def parse_args():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=3)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=("ours", "reference"), default="ours")
    ap.add_argument("--sw-batch", type=int, default=8)
    ap.add_argument("--volume", type=int, nargs=3, default=(512, 512, 224))
    ap.add_argument("--roi", type=int, default=96)
    ap.add_argument("--overlap", type=float, default=0.5)
    ap.add_argument("--skip-kernels", action="store_true", help="omit stand-alone kernel timings")
    ap.add_argument("--skip-cpu", action="store_true", help="omit the CPU baseline")
    ap.add_argument("--eager", action="store_true",
                    help="run the timed steps without CUDA graphs (the eager forward)")
    ap.add_argument("--only-kernels", action="store_true",
                    help="print only the stand-alone kernel timings (profiling target)")
    return ap.parse_args()


def load_peaks() -> dict:
    path = ROOT / "MEASURED_PEAKS.json"
    if path.exists():
        data = json.loads(path.read_text())
        data["source"] = "measured"
        return data
    return dict(FALLBACK_PEAKS)


def build_model(device):
    import torch

    from crumpet_b200.swin_unetr import SwinUNETR

    torch.manual_seed(0)
    model = SwinUNETR(in_channels=1, out_channels=14, feature_size=48, depths=(2, 2, 2, 2),
                      num_heads=(3, 6, 12, 24))
    return model.to(device).eval()


class ClockSampler:
    """nvidia-smi clock / throttle-reason samples during the timed region, every 200 ms.

    On two B200s the same steps ran 882-885 ms with and without a sampler (every GPU from
    one process, each rank its own GPU, NVML from a thread, 500 or 2000 ms): sampling does
    not slow the timed work."""

    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_ids):
        self.gpu_ids = gpu_ids
        self.proc = None
        self.tmp = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)

    def __enter__(self):
        if not self.gpu_ids:
            return self
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={','.join(str(i) for i in self.gpu_ids)}",
                 f"--query-gpu={self.QUERY}", "--format=csv,noheader,nounits", "-lms", "200"],
                stdout=self.tmp, stderr=subprocess.DEVNULL)
        except OSError:
            self.proc = None
            return self
        # nvidia-smi takes a moment to start: a timed region shorter than a second (a few
        # multi-GPU steps) would otherwise end before its first sample
        deadline = time.time() + 5.0
        while time.time() < deadline and self.proc.poll() is None:
            self.tmp.flush()
            if Path(self.tmp.name).stat().st_size > 0:
                break
            time.sleep(0.05)
        return self

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self) -> dict:
        self.tmp.flush()
        rows = []
        for line in Path(self.tmp.name).read_text().splitlines():
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                rows.append((float(parts[1]), float(parts[2]), parts[5:9]))
            except ValueError:
                continue
        os.unlink(self.tmp.name)
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"], "samples": 0}
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for _, _, flags in rows for i, f in enumerate(flags)
                          if f.lower() == "active"})
        return {"sm_mhz": statistics.median(r[0] for r in rows), "sm_max_mhz": max(r[1] for r in rows),
                "reasons": reasons, "samples": len(rows)}


def visible_gpu_ids(world: int) -> list[int]:
    env = os.environ.get("CUDA_VISIBLE_DEVICES")
    if env:
        ids = [int(x) for x in env.split(",") if x.strip().isdigit()]
        if ids:
            return ids[:world]
    return list(range(world))


class ReferenceGPUKernels:
    """The reference's own GPU kernels, built from its sources by
    ``baseline/build_reference.py`` into ``baseline/_ref`` (absent -> not timed):
    its CUDA extension under the op namespace ``crumpet_ref_ops`` and its Triton
    attention kernel as an sm_100 cubin, launched through the CUDA driver API with
    the parameter layout Triton's own launcher uses (every non-constexpr argument in
    order, then two null scratch pointers).  Used only for side-by-side timing."""

    DIR = ROOT / "baseline" / "_ref"

    def __init__(self):
        import ctypes

        import torch

        torch.ops.load_library(str(self.DIR / "crumpet_ref_ops.so"))
        self.ops = torch.ops.crumpet_ref_ops
        self.cuda = ctypes.CDLL("libcuda.so.1")
        vp, ui = ctypes.c_void_p, ctypes.c_uint
        self.cuda.cuModuleLoadData.argtypes = [ctypes.POINTER(vp), vp]
        self.cuda.cuModuleGetFunction.argtypes = [ctypes.POINTER(vp), vp, ctypes.c_char_p]
        self.cuda.cuLaunchKernel.argtypes = [vp, ui, ui, ui, ui, ui, ui, ui, vp, vp, vp]
        for fn in ("cuModuleLoadData", "cuModuleGetFunction", "cuLaunchKernel"):
            getattr(self.cuda, fn).restype = ctypes.c_int
        self.kernels = {}
        for meta_path in sorted(self.DIR.glob("ref_swin_attention_n*.json")):
            meta = json.loads(meta_path.read_text())
            image = meta_path.with_suffix(".cubin").read_bytes()
            module, func = ctypes.c_void_p(), ctypes.c_void_p()
            buf = ctypes.create_string_buffer(image, len(image))
            self._check(self.cuda.cuModuleLoadData(ctypes.byref(module), buf), "cuModuleLoadData")
            self._check(self.cuda.cuModuleGetFunction(ctypes.byref(func), module,
                                                      meta["kernel"].encode()), "cuModuleGetFunction")
            self.kernels[meta["constants"]["N"]] = (func, meta, module, buf)

    @classmethod
    def load(cls):
        if not (cls.DIR / "crumpet_ref_ops.so").exists():
            return None
        return cls()

    @staticmethod
    def _check(rc, what):
        if rc != 0:
            raise RuntimeError(f"{what} failed with CUresult {rc}")

    def attention(self, out, q, k, v, bias, mask, boundary, scale):
        """The reference launcher's call (fused_attention.py:149-226) for float16
        [B, H, N, 16] contiguous q/k/v/out, bias [H, N, N], mask [B or 1, N, N] and
        uint8 boundary [B], each checked against the cubin's specialisation first."""
        import ctypes

        import torch

        B, H, N, D = q.shape
        func, meta, _, _ = self.kernels[N]
        c = meta["constants"]
        tensors = (q, k, v, out, bias, mask, boundary)
        if (D != c["D"] or any(t.dtype != torch.float16 for t in (q, k, v, out, bias, mask))
                or boundary.dtype != torch.uint8 or not all(t.is_contiguous() for t in tensors)
                or tuple(bias.shape) != (H, N, N) or mask.shape[1:] != (N, N)
                or mask.shape[0] not in (1, B) or boundary.numel() != B
                or any(t.data_ptr() % 16 for t in tensors) or any(t.shape != q.shape for t in (k, v, out))
                or any(st % 16 for st in q.stride()[:3])):
            raise ValueError("arguments outside the compiled reference kernel's specialisation")
        mstride = (0 if mask.shape[0] == 1 else mask.stride(0), mask.stride(1))
        vals = {"Q": q, "K": k, "V": v, "BIAS": bias, "MASK": mask, "BOUNDARY": boundary,
                "OUT": out, "SCALE": float(scale),
                "stride_qb": q.stride(0), "stride_qh": q.stride(1), "stride_qn": q.stride(2),
                "stride_kb": k.stride(0), "stride_kh": k.stride(1), "stride_kn": k.stride(2),
                "stride_vb": v.stride(0), "stride_vh": v.stride(1), "stride_vn": v.stride(2),
                "stride_bh": bias.stride(0), "stride_bm": bias.stride(1),
                "stride_mb": mstride[0], "stride_mm": mstride[1],
                "stride_ob": out.stride(0), "stride_oh": out.stride(1), "stride_on": out.stride(2)}
        store = []
        for arg in meta["runtime_args"]:
            val = vals[arg["name"]]
            if arg["type"].startswith("*"):
                store.append(ctypes.c_uint64(val.data_ptr()))
            elif arg["type"] == "fp32":
                store.append(ctypes.c_float(val))
            else:
                store.append(ctypes.c_int32(int(val)))
        store += [ctypes.c_uint64(0)] * meta["trailing_null_pointers"]
        params = (ctypes.c_void_p * len(store))(*[ctypes.addressof(x) for x in store])
        grid = (-(-N // c["BLOCK_M"]), H, B)
        stream = ctypes.c_void_p(torch.cuda.current_stream(q.device).cuda_stream)
        self._check(self.cuda.cuLaunchKernel(func, *grid, meta["threads"], 1, 1,
                                             meta["shared_bytes"], stream, params, None),
                    "cuLaunchKernel")


def attention_stages(device, ref, timed) -> list:
    """The window attention of each Swin stage of one 8-ROI sliding-window batch (the
    bench's workload), this repository's packed entry (what the patched network runs)
    against the reference's Triton kernel on the same windows: exps, times, ratio."""
    import torch

    from crumpet_b200.fused_attention import attention_bias_tiles, swin_window_attention_qkv

    rows = []
    # (padded edge, heads, window, shift): 48^3 -> 49, 24^3 -> 28, 12^3 -> 14, 6^3
    for edge, H, w, sh in ((49, 3, 7, 3), (28, 6, 7, 3), (14, 12, 7, 3), (6, 24, 6, 0)):
        g = torch.Generator(device=device).manual_seed(edge)
        nw = (edge // w,) * 3
        B = 8 * nw[0] ** 3
        N = w ** 3
        qkv = (torch.randn((B, N, 3, H, 16), device=device, generator=g) * 0.5).half()
        table = torch.randn((13 ** 3, H), device=device, generator=g) * 0.02
        coords = torch.stack(torch.meshgrid(*(torch.arange(7),) * 3, indexing="ij")).flatten(1)
        rel = (coords[:, :, None] - coords[:, None, :]) + 6
        index = (rel[0] * 169 + rel[1] * 13 + rel[2]).to(device)
        ws, ss = (w,) * 3, (sh,) * 3
        # the patched network builds each module's bias tiles once and passes them
        tiles = attention_bias_tiles(table, index, N, 0.25, torch.float16)
        ms = timed(lambda: swin_window_attention_qkv(qkv, table, index, nw, ws, ss, 0.25,
                                                     bias_tiles=tiles), iters=10)
        ms_gather = timed(lambda: swin_window_attention_qkv(qkv, table, index, nw, ws, ss, 0.25),
                          iters=10)
        row = {"stage_windows": f"{edge}^3 padded, {B} windows x {H} heads, N={N}",
               "exps": B * H * N * N, "ms": ms, "ms_bias_gathered_per_cta": ms_gather,
               "sfu_frac": B * H * N * N / ms / 1e6 / (16 * 148 * 1965e-3)}
        if ref is not None and N in ref.kernels:
            q, k, v = (qkv[:, :, i].permute(0, 2, 1, 3).contiguous() for i in range(3))
            bias = table[index[:N, :N].reshape(-1)].reshape(N, N, H).permute(2, 0, 1)
            bias = bias.contiguous().half()
            if sh:
                import crumpet_b200 as crumpet

                mask = crumpet.compute_attn_mask_3d(edge, edge, edge, ws, ss, torch.float16, device)
                flags = (mask.reshape(mask.shape[0], -1).abs().amax(1) > 0).to(torch.uint8)
                mask = mask.repeat(8, 1, 1)  # the reference launcher wants B masks (or one)
                bnd = flags.repeat(8)
            else:  # the launcher's no-mask case: one zero mask, every window interior
                mask = torch.zeros((1, N, N), dtype=torch.float16, device=device)
                bnd = torch.zeros((B,), dtype=torch.uint8, device=device)
            out_r = torch.empty_like(q)
            ms_r = timed(lambda: ref.attention(out_r, q, k, v, bias, mask, bnd, 0.25), iters=10)
            ours = swin_window_attention_qkv(qkv, table, index, nw, ws, ss, 0.25)
            ours = ours.reshape(B, N, H, 16).permute(0, 2, 1, 3)
            row.update({"reference_triton_ms": ms_r, "speedup_vs_reference": ms_r / ms,
                        "max_abs_diff": float((out_r.float() - ours.float()).abs().max())})
        rows.append(row)
    return rows


def time_kernels(device, peaks) -> dict:
    """Stand-alone kernel timings at the BASELINE stage-0 sizes (configs 2 and 3)."""
    import torch

    import crumpet_b200 as crumpet

    flush = torch.empty(512 * 1024 * 1024, dtype=torch.uint8, device=device)
    clean = torch.zeros(256 * 1024 * 1024 // 4, dtype=torch.float32, device=device)

    def timed(fn, iters=20, warm=3):
        for _ in range(warm):
            fn()
        torch.cuda.synchronize()
        times = []
        for _ in range(iters):
            # evict L2 (126 MB) between iterations: write a buffer larger than L2, then read
            # another one so the write-backs of the dirty lines finish before the timed launch
            # (left dirty, they cost a write-only-flushed copy kernel ~20 % of its time), then
            # keep the stream busy ~150 us so the wrapper's host time never enters the events
            flush.zero_()
            clean.sum()
            torch.cuda._sleep(300_000)
            s = torch.cuda.Event(enable_timing=True)
            e = torch.cuda.Event(enable_timing=True)
            s.record()
            fn()
            e.record()
            torch.cuda.synchronize()
            times.append(s.elapsed_time(e))
        return statistics.median(times)

    hbm = peaks["hbm_gbs"]
    res = {}
    ref = ref_error = None
    try:
        ref = ReferenceGPUKernels.load()
    except Exception as exc:  # reported in the line, never fatal
        ref_error = repr(exc)

    def beside(name, ref_fn, agreement):
        """Time the reference's own kernel on the same call as res[name] and record how
        its output compares with this repository's."""
        if ref is None:
            return
        ms_r = timed(ref_fn, iters=10)
        d = res[name]
        d["reference"] = {"ms": ms_r, "gbs": d["bytes"] / ms_r / 1e6,
                          "frac_hbm": d["bytes"] / ms_r / 1e6 / hbm,
                          "speedup_vs_reference": ms_r / d["ms"], "outputs": agreement()}

    g = torch.Generator(device=device).manual_seed(2)
    x = torch.randn((1, 98, 98, 98, 48), device=device, generator=g).half()
    ws, ss = (7, 7, 7), (3, 3, 3)
    win = crumpet.fused_shift_partition_3d(x, ws, ss)
    nbytes = 2 * x.numel() * x.element_size()
    ms = timed(lambda: crumpet.fused_shift_partition_3d(x, ws, ss))
    res["fused_shift_partition_3d"] = {"config": "[1,98,98,98,48] fp16 ws7 ss3", "ms": ms,
                                       "bytes": nbytes, "gbs": nbytes / ms / 1e6,
                                       "frac_hbm": nbytes / ms / 1e6 / hbm}
    if ref is not None:
        win_r = torch.empty_like(win)
        beside("fused_shift_partition_3d",
               lambda: ref.ops.fused_shift_partition_3d(win_r, x, *ws, *ss),
               lambda: "bit-exact" if torch.equal(win_r, win) else "DIFFERENT")
        del win_r
    ms = timed(lambda: crumpet.fused_unshift_unpartition_3d(win, 1, 98, 98, 98, 48, ws, ss))
    res["fused_unshift_unpartition_3d"] = {"config": "[2744,343,48] fp16 ws7 ss3", "ms": ms,
                                           "bytes": nbytes, "gbs": nbytes / ms / 1e6,
                                           "frac_hbm": nbytes / ms / 1e6 / hbm}
    if ref is not None:
        x_r = torch.empty_like(x)
        beside("fused_unshift_unpartition_3d",
               lambda: ref.ops.fused_unshift_unpartition_3d(x_r, win, 1, 98, 98, 98, 48, *ws, *ss),
               lambda: "bit-exact" if torch.equal(x_r, x) else "DIFFERENT")
        del x_r
    mask = torch.empty((2744, 343, 343), dtype=torch.float16, device=device)
    ops = crumpet._ops.require()
    ms = timed(lambda: ops.compute_attn_mask_3d(mask, 98, 98, 98, *ws, *ss))
    mbytes = mask.numel() * 2
    res["compute_attn_mask_3d"] = {"config": "[2744,343,343] fp16 (write-only)", "ms": ms,
                                   "bytes": mbytes, "gbs": mbytes / ms / 1e6,
                                   "frac_hbm": mbytes / ms / 1e6 / hbm}
    if ref is not None:
        mask_r = torch.empty_like(mask)
        beside("compute_attn_mask_3d",
               lambda: ref.ops.compute_attn_mask_3d(mask_r, 98, 98, 98, *ws, *ss),
               lambda: "bit-exact" if torch.equal(mask_r, mask) else "DIFFERENT")
        del mask_r
    B, H, N = 2744, 3, 343
    w_qkv = torch.randn((3 * 48, 48), device=device, generator=g) * 0.02
    qkv = torch.nn.functional.linear(win.float(), w_qkv).half()
    qkv = qkv.reshape(B, N, 3, H, 16).permute(2, 0, 3, 1, 4)
    q, k, v = (t.contiguous() for t in qkv)
    table = torch.randn((13 ** 3, H), device=device, generator=g) * 0.02
    coords = torch.stack(torch.meshgrid(*(torch.arange(7),) * 3, indexing="ij")).flatten(1)
    rel = (coords[:, :, None] - coords[:, None, :]) + 6
    index = (rel[0] * 169 + rel[1] * 13 + rel[2]).to(device)
    bias = table[index.reshape(-1)].reshape(N, N, H).permute(2, 0, 1).contiguous().half()
    bnd = (mask.view(B, -1).abs().amax(1) > 0).to(torch.uint8)
    flops = 4 * B * H * N * N * 16
    # the drop-in call as the reference's patch makes it: the mask from compute_attn_mask_3d,
    # which the kernel recognises and adds on chip; then a mask tensor it must read (the one
    # the raw op wrote above is not one compute_attn_mask_3d returned)
    mask_api = crumpet.compute_attn_mask_3d(98, 98, 98, ws, ss, torch.float16, device)
    for row, m, mask_read in (("fused_swin_attention", mask_api, False),
                              ("fused_swin_attention_dense_mask", mask, True)):
        ms = timed(lambda: crumpet.fused_swin_attention(q, k, v, bias, m, bnd), iters=10)
        abytes = 4 * B * H * N * 16 * 2 + H * N * N * 2 + (int(bnd.sum()) * N * N * 2
                                                          if mask_read else 0)
        res[row] = {"config": "2744x3x343x16 fp16, mask+boundary, mask " +
                              ("tensor read from HBM" if mask_read
                               else "from compute_attn_mask_3d (added on chip)"),
                    "ms": ms, "bytes": abytes, "gbs": abytes / ms / 1e6,
                    "frac_hbm": abytes / ms / 1e6 / hbm, "tflops": flops / ms / 1e9,
                    "frac_tensor": flops / ms / 1e9 / peaks["bf16_tflops"],
                    "gexp_s": B * H * N * N / ms / 1e6}
    attn_ours = crumpet.fused_swin_attention(q, k, v, bias, mask_api, bnd)
    del mask_api
    if ref is not None:
        out_r = torch.empty_like(q)
        beside("fused_swin_attention",
               lambda: ref.attention(out_r, q, k, v, bias, mask, bnd, 0.25),
               lambda: {"max_abs_diff": float((out_r.float() - attn_ours.float()).abs().max())})
        res["fused_swin_attention"]["reference"]["kernel"] = (
            "reference Triton _fused_swin_attention_kernel, AOT-compiled for sm_100 "
            "(BLOCK_M 64, BLOCK_N 32, 4 warps, 3 stages)")
        # the reference reads the mask rows of flagged windows: its bandwidth counts them
        r = res["fused_swin_attention"]["reference"]
        r["gbs"] = res["fused_swin_attention_dense_mask"]["bytes"] / r["ms"] / 1e6
        r["frac_hbm"] = r["gbs"] / hbm
        del out_r
    # the patched-network path: packed qkv, in-kernel bias gather, on-chip mask
    from crumpet_b200.fused_attention import swin_window_attention_qkv

    qkv_packed = qkv.permute(1, 3, 0, 2, 4).contiguous()  # [B, N, 3, H, 16]
    ms = timed(lambda: swin_window_attention_qkv(qkv_packed, table, index, (14, 14, 14), ws, ss,
                                                 0.25), iters=10)
    pbytes = 4 * B * H * N * 16 * 2
    res["swin_window_attention_qkv"] = {"config": "2744x3x343x16 fp16 packed qkv, table bias, on-chip mask",
                                        "ms": ms, "bytes": pbytes, "gbs": pbytes / ms / 1e6,
                                        "frac_hbm": pbytes / ms / 1e6 / hbm,
                                        "tflops": flops / ms / 1e9,
                                        "frac_tensor": flops / ms / 1e9 / peaks["bf16_tflops"],
                                        "gexp_s": B * H * N * N / ms / 1e6,
                                        "sfu_frac": B * H * N * N / ms / 1e6 / (16 * 148 * 1965e-3)}
    if ref is not None:
        res["swin_window_attention_qkv"]["speedup_vs_reference_triton"] = (
            res["fused_swin_attention"]["reference"]["ms"] / ms)
        del attn_ours
        res["attention_by_stage"] = attention_stages(device, ref, timed)
    elif ref_error is not None:
        res["reference_unavailable"] = ref_error
    else:
        res["reference_unavailable"] = "baseline/_ref not built (python baseline/build_reference.py)"
    # the fused block glue at the first stage of an 8-ROI sliding-window batch:
    # [8,48,48,48,48] fp16 -> LayerNorm + pad to 49^3 + roll + partition -> fp16 windows,
    # and windows -> unpartition + roll back + crop + residual add
    del q, k, v, qkv, qkv_packed, mask, win, x
    xs = torch.randn((8, 48, 48, 48, 48), device=device, generator=g).half()
    gamma = torch.ones(48, device=device)
    beta = torch.zeros(48, device=device)
    wins = crumpet.norm_shift_partition_3d(xs, gamma, beta, 1e-5, ws, ss, torch.float16)
    nb_in = xs.numel() * 2
    nb = nb_in + wins.numel() * 2
    ms = timed(lambda: crumpet.norm_shift_partition_3d(xs, gamma, beta, 1e-5, ws, ss, torch.float16))
    res["norm_shift_partition_3d"] = {"config": "[8,48,48,48,48] fp16 -> [2744,343,48] fp16 (pad 49^3)",
                                      "ms": ms, "bytes": nb, "gbs": nb / ms / 1e6,
                                      "frac_hbm": nb / ms / 1e6 / hbm}
    nb = 3 * nb_in
    ms = timed(lambda: crumpet.unshift_unpartition_crop_3d(wins, 8, 48, 48, 48, 48, ws, ss,
                                                           residual=xs))
    res["unshift_unpartition_crop_3d"] = {"config": "[2744,343,48] fp16 -> [8,48,48,48,48] + residual",
                                          "ms": ms, "bytes": nb, "gbs": nb / ms / 1e6,
                                          "frac_hbm": nb / ms / 1e6 / hbm}
    # the same pass with the next LayerNorm fused: writes the block output and norm2 of it
    nb = 4 * nb_in
    ms = timed(lambda: crumpet.unshift_unpartition_crop_norm_3d(wins, 8, 48, 48, 48, 48, ws, ss,
                                                                gamma, beta, 1e-5, residual=xs))
    res["unshift_unpartition_crop_norm_3d"] = {
        "config": "[2744,343,48] fp16 + residual -> [8,48,48,48,48] out + LayerNorm(out)",
        "ms": ms, "bytes": nb, "gbs": nb / ms / 1e6, "frac_hbm": nb / ms / 1e6 / hbm}
    # patch merging of that stage: 2x2x2 neighbours + LayerNorm(384) -> [8,24,24,24,384] fp16
    g8 = torch.ones(384, device=device)
    b8 = torch.zeros(384, device=device)
    nb = 2 * nb_in
    ms = timed(lambda: crumpet.patch_merge_norm_3d(xs, g8, b8, 1e-5))
    res["patch_merge_norm_3d"] = {"config": "[8,48,48,48,48] fp16 -> [8,24,24,24,384] fp16",
                                  "ms": ms, "bytes": nb, "gbs": nb / ms / 1e6,
                                  "frac_hbm": nb / ms / 1e6 / hbm}
    # the trunk's hidden-state norm of the patch embedding (x0 of an 8-ROI batch):
    # channels-first fp16 in, channels-last fp32 out (LayerNorm's autocast dtype)
    xcf = xs.permute(0, 4, 1, 2, 3).contiguous()
    nb = nb_in + 2 * nb_in
    ms = timed(lambda: crumpet.proj_out_norm_3d(xcf, out_dtype=torch.float32))
    res["proj_out_norm_3d"] = {"config": "[8,48,48,48,48] fp16 channels-first -> fp32 channels-last",
                               "ms": ms, "bytes": nb, "gbs": nb / ms / 1e6,
                               "frac_hbm": nb / ms / 1e6 / hbm}
    # the window attention's qkv / proj Linears at the same stage (941,192 window tokens),
    # with torch's F.linear (cuBLAS) on the same operands beside them
    del xcf
    tok = wins.reshape(-1, 48)
    for name, n_out in (("window_linear_qkv", 144), ("window_linear_proj", 48)):
        w = (torch.randn((n_out, 48), device=device, generator=g) * 0.15).half()
        b = (torch.randn((n_out,), device=device, generator=g) * 0.1).half()
        nb = tok.numel() * 2 + tok.shape[0] * n_out * 2
        ms = timed(lambda: crumpet.window_linear(tok, w, b))
        ms_ref = timed(lambda: torch.nn.functional.linear(tok, w, b))
        res[name] = {"config": f"[941192,48] x [48,{n_out}] + bias fp16", "ms": ms, "bytes": nb,
                     "gbs": nb / ms / 1e6, "frac_hbm": nb / ms / 1e6 / hbm,
                     "cublas_ms": ms_ref, "cublas_frac_hbm": nb / ms_ref / 1e6 / hbm}
    del flush, clean
    return res


def cpu_baseline(roi: int, budget_s: float = 12.0) -> dict:
    """The unpatched eager network on the host cores: ROIs/s on a bounded sample."""
    import torch

    from crumpet_b200.swin_unetr import SwinUNETR

    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    torch.manual_seed(0)
    model = SwinUNETR(1, 14, 48).eval()
    x = torch.rand((1, 1, roi, roi, roi))
    with torch.no_grad():
        model(x)  # allocator warm-up
        n, t0 = 0, time.perf_counter()
        while True:
            model(x)
            n += 1
            dt = time.perf_counter() - t0
            if dt >= budget_s or n >= 8:
                break
    return {"value": n / dt, "unit": UNIT, "cores": torch.get_num_threads(), "kind": "port",
            "sample": f"{n} ROI(s) of {roi}^3 through the unpatched eager network, fp32, "
                      f"{dt:.1f} s"}


def kernels_vs_roofline(per_op: dict, peaks: dict, clock, steps: int, dev_ms: float):
    """This rank's crumpet_b200 kernels inside the timed end-to-end region against their
    roofline: per op, the CUDA-event time of its launches and its ideal time -- algorithmic
    bytes at the measured HBM copy rate, or for the attention the larger of that and its
    exponentials at the SFU rate (16 per clock per SM at the sampled SM clock).  The rest
    of the step (the UNETR convolution decoder, cuBLAS GEMMs, torch elementwise ops) is
    not crumpet_b200's and is left out."""
    if not per_op:
        return None
    sm_mhz = (clock or {}).get("sm_mhz") or 1965.0
    exp_per_ms = 16 * 148 * sm_mhz * 1e6 / 1e3
    hbm_bytes_per_ms = peaks["hbm_gbs"] * 1e6
    def ideal_ms(d):
        ideal, bound = d["bytes"] / hbm_bytes_per_ms, "hbm"
        if d["exps"] and d["exps"] / exp_per_ms > ideal:
            ideal, bound = d["exps"] / exp_per_ms, "sfu"
        return ideal, bound

    rows, tot_ms, tot_ideal = {}, 0.0, 0.0
    for op, d in sorted(per_op.items(), key=lambda kv: -kv[1]["ms"]):
        ideal, bound = ideal_ms(d)
        rows[op] = {"launches_per_step": d["launches"] / steps, "ms_per_step": d["ms"] / steps,
                    "ideal_ms_per_step": ideal / steps, "frac": ideal / d["ms"] if d["ms"] else None,
                    "bound": bound}
        # the same split by launch shape (largest first): where the time goes per stage
        sizes = []
        for nbytes, sd in sorted(d.get("sizes", {}).items(), key=lambda kv: -kv[0])[:6]:
            s_ideal, _ = ideal_ms(sd)
            sizes.append({"mb_per_launch": round(nbytes / 1e6, 3),
                          "launches_per_step": sd["launches"] / steps,
                          "us_per_launch": 1e3 * sd["ms"] / sd["launches"],
                          "frac": s_ideal / sd["ms"] if sd["ms"] else None})
        if len(sizes) > 1:
            rows[op]["by_launch_size"] = sizes
        tot_ms += d["ms"]
        tot_ideal += ideal
    return {"ms_per_step": tot_ms / steps, "ideal_ms_per_step": tot_ideal / steps,
            "frac_of_roofline": tot_ideal / tot_ms if tot_ms else None,
            "share_of_step": tot_ms / dev_ms if dev_ms else None,
            "peak_source": peaks["source"], "by_op": rows}


def workload_config(args, world: int) -> dict:
    """The workload both arms report."""
    from crumpet_b200.inferer import roi_grid

    spatial = tuple(args.volume)
    n_rois = len(roi_grid(spatial, (args.roi,) * 3, args.overlap))
    return {"workload": "swin_unetr_sliding_window", "volume": list(spatial),
            "roi": [args.roi] * 3, "overlap": args.overlap, "sw_batch": args.sw_batch,
            "rois_per_step": n_rois, "feature_size": 48, "depths": [2, 2, 2, 2],
            "heads": [3, 6, 12, 24], "window": 7, "classes": 14,
            "parallelism": f"roi-shard x{world}",
            "l2": "inputs larger than L2 (235 MB volume, 3.3 GB fp32 accumulator)"}


def run_reference(args) -> None:
    """The CPU reference arm: the unpatched eager network (the MONAI code path crumpet
    patches: torch.roll, window partition, eager attention) on the host cores, one ROI
    of the workload per step.  It imports crumpet_b200's pure-torch modules only; no
    native library of this repository is loaded (the line reports it)."""
    import torch

    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    from crumpet_b200 import _ops
    from crumpet_b200.swin_unetr import SwinUNETR

    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    torch.manual_seed(0)
    model = SwinUNETR(1, 14, 48).eval()
    x = torch.rand((1, 1, args.roi, args.roi, args.roi))
    times = []
    with torch.no_grad():
        for i in range(args.warmup + args.steps):
            t0 = time.perf_counter()
            model(x)
            dt = time.perf_counter() - t0
            if i >= args.warmup:
                times.append(dt)
    total = sum(times)
    value = len(times) / total
    n_rois = workload_config(args, 1)["rois_per_step"]
    sample = (f"each step: 1 of the workload's {n_rois} ROIs ({args.roi}^3) through the "
              f"unpatched eager network, fp32, {threads} threads")
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1000 * total / len(times),
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic",
        "config": workload_config(args, args.gpus),
        "sample": {"rois_per_step": 1, "roi": [args.roi] * 3, "device": "cpu",
                   "note": "value = ROIs/s over these one-ROI steps; config names the workload "
                           "the ROIs are drawn from"},
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": torch.get_num_threads(),
                         "kind": "port", "sample": sample},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "native_libraries_loaded": _ops.loaded(),
    }
    print(json.dumps(line), flush=True)


def main() -> None:
    args = parse_args()
    if args.impl == "reference":
        run_reference(args)
        return

    import torch
    import torch.distributed as dist

    import crumpet_b200 as crumpet
    from crumpet_b200 import monai_patch, profiling, swin_unetr
    from crumpet_b200.inferer import SlidingWindowInferer, roi_grid, synthetic_volume

    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    if args.only_kernels:
        if rank == 0:
            print(json.dumps({"kernels": time_kernels(device, load_peaks())}), flush=True)
        return
    if world > 1:
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=device)
    peaks = load_peaks()

    model = build_model(device)
    crumpet.patch_monai_swin_unetr(swin_unetr)
    inferer = SlidingWindowInferer(model, (args.roi,) * 3, args.sw_batch, args.overlap, 14,
                                   torch.float16, rank, world, cuda_graphs=not args.eager,
                                   device=device)
    # the same inference without graphs: its launches can be bracketed one by one
    eager_inferer = SlidingWindowInferer(model, (args.roi,) * 3, args.sw_batch, args.overlap,
                                         14, torch.float16, rank, world)
    spatial = tuple(args.volume)
    n_rois = len(roi_grid(spatial, (args.roi,) * 3, args.overlap))
    host = synthetic_volume((1, 1, *spatial)).pin_memory()
    vol = host.to(device)
    seg_host = torch.empty(spatial, dtype=torch.uint8).pin_memory()

    def barrier():
        if world > 1:
            dist.barrier()

    def max_over_ranks(x: float) -> float:
        if world == 1:
            return x
        t = torch.tensor([x], dtype=torch.float64, device=device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    for _ in range(args.warmup):
        inferer.segment(vol)
    torch.cuda.synchronize()

    # ---- timed region 1: volume resident in HBM
    launches0 = profiling.total_launches()
    # rank 0 starts the sampler (and waits for its first sample) before the barrier, so
    # every rank's clock starts together
    with ClockSampler(visible_gpu_ids(world) if rank == 0 else []) as clocks:
        barrier()
        torch.cuda.synchronize()
        start = torch.cuda.Event(enable_timing=True)
        end = torch.cuda.Event(enable_timing=True)
        start.record()
        for _ in range(args.steps):
            inferer.segment(vol)
        end.record()
        torch.cuda.synchronize()
        barrier()
    dev_ms = max_over_ranks(start.elapsed_time(end))
    launches = profiling.total_launches() - launches0
    clock = clocks.summary() if rank == 0 else None

    # ---- per-kernel pass: the same steps on the eager forward, with CUDA events around
    # every crumpet_b200 launch (a graph replay cannot be bracketed kernel by kernel)
    if args.eager:
        eager_inferer = inferer
    else:
        eager_inferer.segment(vol)  # warm
    barrier()
    torch.cuda.synchronize()
    with profiling.KernelTimer() as ktimer:
        s1 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        s1.record()
        for _ in range(args.steps):
            eager_inferer.segment(vol)
        e1.record()
        torch.cuda.synchronize()
        barrier()
    eager_ms = max_over_ranks(s1.elapsed_time(e1))
    attn = ktimer.summary()
    per_op = ktimer.by_op()

    # ---- timed region 2: host buffers in, segmentation out (the public call)
    barrier()
    torch.cuda.synchronize()
    s2 = torch.cuda.Event(enable_timing=True)
    e2 = torch.cuda.Event(enable_timing=True)
    s2.record()
    for _ in range(args.steps):
        # the public call with the host volume: each rank copies its z-slab to its GPU
        seg = inferer.segment(host)
        if seg is not None:
            seg_host.copy_(seg, non_blocking=True)
    e2.record()
    torch.cuda.synchronize()
    barrier()
    e2e_ms = max_over_ranks(s2.elapsed_time(e2))

    # per step, summed over ranks: launches, host->device bytes of the e2e call, and bytes
    # moved between GPUs (halo planes of the accumulators, owned label ranges to rank 0)
    plan = inferer.plan(spatial)
    label_bytes = 0 if rank == 0 else (plan[rank].own[1] - plan[rank].own[0]) * spatial[1] * spatial[2]
    counts = [launches, inferer.staged_bytes(spatial), inferer.exchanged_bytes + label_bytes]
    if world > 1:
        t = torch.tensor(counts, dtype=torch.int64, device=device)
        dist.all_reduce(t)
        counts = [int(v) for v in t.tolist()]
    total_launches, h2d_bytes, p2p_bytes = counts

    crumpet.unpatch_monai_swin_unetr()
    kernels = None
    if rank == 0 and not args.skip_kernels:
        kernels = time_kernels(device, peaks)
    cpu = None
    if rank == 0 and world == 1 and not args.skip_cpu:
        cpu = cpu_baseline(args.roi)

    if rank == 0:
        value = n_rois * args.steps / (dev_ms / 1000.0)
        e2e_value = n_rois * args.steps / (e2e_ms / 1000.0)
        roofline = None
        if attn.get("launches"):
            gbs = attn["bytes"] / attn["avg_ms"] / 1e6
            tflops = attn["flops"] / attn["avg_ms"] / 1e9
            f_hbm = gbs / peaks["hbm_gbs"]
            f_tc = tflops / peaks["bf16_tflops_sustained" if "bf16_tflops_sustained" in peaks else "bf16_tflops"]
            sm_mhz = (clock or {}).get("sm_mhz") or 1965.0
            exp_peak = 16 * 148 * sm_mhz * 1e6  # MUFU ex2 lanes per SM per clock
            exp_rate = attn["exps"] / (attn["avg_ms"] / 1e3)
            # The kernel's binding roof is the SFU: one ex2 per score, 16 per clock per SM
            # (measured with a micro-benchmark on this part), at the sampled SM clock.
            # Its HBM and tensor-pipe fractions are reported beside it.
            roofline = {
                "kernel": "window_attention_kernel (swin_window_attention_qkv: packed qkv, on-chip mask)",
                "bound": "sfu",
                "achieved": exp_rate / 1e9,
                "peak": exp_peak / 1e9,
                "unit": "Gexp/s",
                "frac": exp_rate / exp_peak,
                "peak_source": f"16 ex2/clk/SM x 148 SMs x {sm_mhz:.0f} MHz (sampled SM clock)",
                "traffic": None,
                "launches_timed": attn["launches"],
                "avg_launch_ms": attn["avg_ms"],
                "exps_per_launch": attn["exps"],
                "algorithmic_bytes_per_launch": attn["bytes"],
                "flops_per_launch": attn["flops"],
                "hbm": {"achieved": gbs, "peak": peaks["hbm_gbs"], "unit": "GB/s", "frac": f_hbm,
                        "peak_source": peaks["source"]},
                "tensor": {"achieved": tflops, "unit": "TFLOP/s", "frac": f_tc,
                           "peak": peaks.get("bf16_tflops_sustained", peaks["bf16_tflops"]),
                           "peak_source": peaks["source"]},
            }
            traffic_file = ROOT / "profiles" / "attention_traffic.json"
            if traffic_file.exists():
                tr = json.loads(traffic_file.read_text())
                # ncu DRAM bytes of one captured launch, scaled by algorithmic bytes
                roofline["traffic"] = attn["bytes"] * tr["dram_over_algorithmic"]
                roofline["traffic_source"] = tr["command"]
            roofline["timed_in"] = PER_KERNEL_PASS
        crumpet_kernels = kernels_vs_roofline(per_op, peaks, clock, args.steps, eager_ms)
        if crumpet_kernels is not None:
            crumpet_kernels["timed_in"] = PER_KERNEL_PASS
        line = {
            "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": dev_ms / args.steps, "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "fp16", "data": "synthetic",
            "config": workload_config(args, world),
            "execution": ("eager forward" if args.eager else
                          "CUDA graph replay of each ROI batch's forward (one graph per batch "
                          "size); crop and accumulate launches outside the graphs"),
            "eager": {"value": n_rois * args.steps / (eager_ms / 1000.0), "unit": UNIT,
                      "ms_per_step": eager_ms / args.steps,
                      "note": "same steps without CUDA graphs, every crumpet_b200 launch "
                              "bracketed by CUDA events (the per-kernel pass)"},
            "e2e": {"value": e2e_value, "unit": UNIT,
                    "h2d_bytes_per_step": h2d_bytes,
                    "d2h_bytes_per_step": seg_host.numel(),
                    "note": "each rank copies only the z-slab of the host volume its ROIs read"},
            "interconnect_bytes_per_step": p2p_bytes,
            "gpu_launches": total_launches,
            "clocks": clock,
            "roofline": roofline,
            "crumpet_kernels": crumpet_kernels,
            "kernels": kernels,
            "cpu_baseline": cpu,
        }
        print(json.dumps(line), flush=True)

    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
