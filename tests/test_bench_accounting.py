"""bench.py's in-step roofline accounting, on synthetic launch records (no GPU):
per-op ideal times at the HBM copy rate or the SFU exponential rate, and the split
of an op's launches by launch shape."""

from __future__ import annotations

import pytest

import bench

PEAKS = {"hbm_gbs": 6449.7, "source": "measured"}
CLOCK = {"sm_mhz": 1965.0}


def _rec(launches, ms, nbytes, exps=0):
    return {"launches": launches, "ms": ms, "bytes": nbytes, "exps": exps}


def test_hbm_and_sfu_bounds():
    per_op = {
        "copy": dict(_rec(2, 0.2, 1_289_940_000), sizes={}),
        # 2 * 4.65e9 exponentials per ms of SFU time at 1965 MHz: 1 ms ideal
        "attn": dict(_rec(1, 2.0, 1_000, exps=16 * 148 * 1965e3), sizes={}),
    }
    out = bench.kernels_vs_roofline(per_op, PEAKS, CLOCK, steps=1, dev_ms=10.0)
    assert out["by_op"]["copy"]["bound"] == "hbm"
    assert out["by_op"]["copy"]["frac"] == pytest.approx(1.0, rel=1e-3)
    assert out["by_op"]["attn"]["bound"] == "sfu"
    assert out["by_op"]["attn"]["frac"] == pytest.approx(0.5, rel=1e-6)
    assert out["share_of_step"] == pytest.approx(0.22)
    assert "by_launch_size" not in out["by_op"]["copy"]


def test_split_by_launch_size_largest_first():
    big, small = 175_000_000, 50_000_000
    per_op = {"norm": dict(_rec(6, 6.0, 2 * big + 4 * small), sizes={
        small: _rec(4, 5.92, 4 * small),
        big: _rec(2, 0.08, 2 * big),
    })}
    out = bench.kernels_vs_roofline(per_op, PEAKS, CLOCK, steps=2, dev_ms=100.0)
    sizes = out["by_op"]["norm"]["by_launch_size"]
    assert [s["mb_per_launch"] for s in sizes] == [175.0, 50.0]
    assert sizes[0]["launches_per_step"] == 1.0
    assert sizes[0]["us_per_launch"] == pytest.approx(40.0)
    assert sizes[0]["frac"] == pytest.approx(2 * big / (PEAKS["hbm_gbs"] * 1e6) / 0.08)
    assert out["by_op"]["norm"]["ms_per_step"] == pytest.approx(3.0)


def test_no_records():
    assert bench.kernels_vs_roofline({}, PEAKS, CLOCK, steps=1, dev_ms=1.0) is None


def test_capture_suspends_timers_and_hands_back_the_launch_counts():
    """While a CUDA graph is captured nothing runs: the launches counted then are taken
    out of the counters and handed back, to be added once per replay."""
    from crumpet_b200 import profiling

    timer = profiling.KernelTimer()
    with timer:
        profiling.count("roi_gather")
        before = dict(profiling.counters)
        with profiling.suspended() as cap:
            assert profiling._active == []
            assert profiling.kernel_begin("x", {}) is None  # no timer records during capture
            profiling.count("swin_window_attention_qkv", 8)
            profiling.count("window_linear", 6)
        assert profiling._active == [timer]
        assert dict(profiling.counters) == before
        assert dict(cap.delta) == {"swin_window_attention_qkv": 8, "window_linear": 6}
        profiling.count_replay(cap.delta)
        profiling.count_replay(cap.delta)
        assert profiling.counters["window_linear"] == before.get("window_linear", 0) + 12


def test_importing_the_package_maps_no_native_library():
    # the CPU reference arm imports crumpet_b200's pure-torch modules; loading the
    # kernels' libraries there would put this repository's native code in that arm
    import subprocess
    import sys

    code = ("import crumpet_b200, crumpet_b200.swin_unetr, crumpet_b200.inferer, "
            "crumpet_b200.monai_patch\n"
            "from crumpet_b200 import _ops\n"
            "maps = open('/proc/self/maps').read()\n"
            "assert _ops.ops is None and not _ops.loaded()\n"
            "assert 'libcrumpet_b200' not in maps and '_C.so' not in maps\n")
    subprocess.run([sys.executable, "-c", code], check=True, cwd=str(bench.ROOT))


def test_reference_arm_reports_its_sample_and_loads_nothing_native():
    import json
    import subprocess
    import sys

    proc = subprocess.run(
        [sys.executable, str(bench.ROOT / "bench.py"), "--impl", "reference", "--steps", "1",
         "--warmup", "0", "--roi", "64", "--volume", "128", "128", "64"],
        check=True, capture_output=True, text=True, timeout=600)
    line = json.loads(proc.stdout.strip().splitlines()[-1])
    assert line["impl"] == "reference"
    assert line["native_libraries_loaded"] is False
    assert line["sample"]["rois_per_step"] == 1
    assert line["config"]["rois_per_step"] == 9
    assert "execution" not in line["config"]
    assert line["e2e"]["value"] == line["value"]
