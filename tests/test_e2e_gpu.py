"""Patched vs eager Swin UNETR on the GPU under fp16 autocast (BASELINE config 5
criteria: segmentation arg-max agreement >= 99.9 %; logits within fp16
tolerance), and a Swin block at BASELINE config 1 geometry."""

from __future__ import annotations

import pytest
import torch

import crumpet_b200 as crumpet
from crumpet_b200 import profiling, swin_unetr
from crumpet_b200.inferer import SlidingWindowInferer

pytestmark = pytest.mark.gpu


def _run(model, x, patched):
    if patched:
        crumpet.patch_monai_swin_unetr(swin_unetr)
    try:
        with torch.no_grad(), torch.autocast("cuda", dtype=torch.float16):
            return model(x).float()
    finally:
        crumpet.unpatch_monai_swin_unetr()


def test_shifted_block_matches_eager(cuda_device):
    torch.manual_seed(0)
    blk = swin_unetr.SwinTransformerBlock(48, 3, (7, 7, 7), (3, 3, 3)).to(cuda_device).eval()
    with torch.no_grad():
        blk.attn.relative_position_bias_table.normal_(0, 0.02)
    x = torch.randn((1, 28, 28, 28, 48), device=cuda_device)
    mask = swin_unetr.compute_mask((28, 28, 28), (7, 7, 7), (3, 3, 3), cuda_device)
    before = profiling.total_launches()
    # a mask without recorded window geometry (a copy, not the cached tensor the
    # patched BasicLayer annotates): the block takes the dense-mask kernel
    dense = crumpet.compute_attn_mask_3d(28, 28, 28, (7, 7, 7), (3, 3, 3), torch.float16,
                                         cuda_device).clone()
    patched = _run(lambda t: blk(t, dense), x, True)
    assert profiling.counters["fused_swin_attention"] > 0
    assert profiling.total_launches() - before >= 3
    eager = _run(lambda t: blk(t, mask), x, False)
    assert (patched - eager).abs().max().item() < 2e-2


def test_network_argmax_agreement_one_batch(cuda_device):
    torch.manual_seed(0)
    model = swin_unetr.SwinUNETR(1, 14, 48).to(cuda_device).eval()
    x = torch.rand((2, 1, 96, 96, 96), device=cuda_device)
    patched = _run(model, x, True)
    eager = _run(model, x, False)
    agree = (patched.argmax(1) == eager.argmax(1)).float().mean().item()
    assert agree >= 0.999, agree
    assert (patched - eager).abs().max().item() < 5e-2


def test_sliding_window_patched_vs_eager(cuda_device):
    torch.manual_seed(0)
    model = swin_unetr.SwinUNETR(1, 14, 48).to(cuda_device).eval()
    vol = torch.rand((1, 1, 128, 128, 96), device=cuda_device)
    inf = SlidingWindowInferer(model, (96, 96, 96), 2, 0.5, 14, torch.float16)
    crumpet.patch_monai_swin_unetr(swin_unetr)
    try:
        seg_p = inf.segment(vol)
        logit_p = inf.logits(vol)
    finally:
        crumpet.unpatch_monai_swin_unetr()
    seg_e = inf.segment(vol)
    logit_e = inf.logits(vol)
    agree = (seg_p == seg_e).float().mean().item()
    assert agree >= 0.999, agree
    assert (logit_p - logit_e).abs().max().item() < 5e-2


def test_sliding_window_cuda_graphs_match_eager_bit_for_bit(cuda_device):
    """CUDA-graph mode replays the same kernels on the same data: logits and labels equal
    the eager patched run's exactly, over two volumes in a row (the second replays the
    graphs captured for the first) and unequal batches (10 ROIs in batches of at most 4
    run as 4 + 3 + 3: a graph per batch size), and each replay counts its crumpet_b200
    launches."""
    torch.manual_seed(0)
    model = swin_unetr.SwinUNETR(1, 14, 48).to(cuda_device).eval()
    vols = [torch.rand((1, 1, 96, 144, 288), device=cuda_device) for _ in range(2)]
    eager = SlidingWindowInferer(model, (96, 96, 96), 4, 0.5, 14, torch.float16)
    graphed = SlidingWindowInferer(model, (96, 96, 96), 4, 0.5, 14, torch.float16,
                                   cuda_graphs=True)
    assert len(graphed.rois((96, 144, 288))) == 10
    assert [len(b) for b in graphed.my_batches((96, 144, 288))] == [4, 3, 3]
    crumpet.patch_monai_swin_unetr(swin_unetr)
    try:
        for vol in vols:
            want_logits, want_seg = eager.logits(vol), eager.segment(vol)
            n0 = profiling.counters["swin_window_attention_qkv"]
            got_logits = graphed.logits(vol)
            n1 = profiling.counters["swin_window_attention_qkv"]
            got_seg = graphed.segment(vol)
            assert torch.equal(got_logits, want_logits)
            assert torch.equal(got_seg, want_seg)
            # 8 attention launches per forward, one forward per batch
            assert n1 - n0 == 3 * 8
        assert sorted(k[0] for k in graphed._graphs) == [3, 4]
    finally:
        crumpet.unpatch_monai_swin_unetr()
    # unpatched: the captured graphs still hold the patched forward until reset
    graphed.reset_graphs()
    n0 = profiling.counters["swin_window_attention_qkv"]
    assert torch.equal(graphed.logits(vols[1]), eager.logits(vols[1]))
    assert profiling.counters["swin_window_attention_qkv"] == n0


def test_head_dim_32_network_argmax_agreement(cuda_device):
    # feature size 96: heads (3, 6, 12, 24) of head_dim 32 at every stage
    torch.manual_seed(0)
    model = swin_unetr.SwinUNETR(1, 14, 96).to(cuda_device).eval()
    x = torch.rand((1, 1, 64, 64, 64), device=cuda_device)
    before = profiling.counters["swin_window_attention_qkv"]
    patched = _run(model, x, True)
    assert profiling.counters["swin_window_attention_qkv"] > before
    eager = _run(model, x, False)
    agree = (patched.argmax(1) == eager.argmax(1)).float().mean().item()
    assert agree >= 0.999, agree
    assert (patched - eager).abs().max().item() < 5e-2


def test_every_fusion_engages_in_the_patched_network(cuda_device):
    """One fp16-autocast forward of the patched feature-size-48 network launches each fused
    op: packed attention, norm1 + partition, crop + residual + norm2, patch merging (all four
    stages), the hidden-state norms (all five outputs) and the tensor-core qkv / proj
    Linears where their shapes fit."""
    torch.manual_seed(0)
    model = swin_unetr.SwinUNETR(1, 14, 48).to(cuda_device).eval()
    x = torch.rand((1, 1, 96, 96, 96), device=cuda_device)
    names = ["swin_window_attention_qkv", "norm_shift_partition_3d",
             "unshift_unpartition_crop_norm_3d", "patch_merge_norm_3d", "proj_out_norm_3d",
             "window_linear"]
    before = {n: profiling.counters[n] for n in names}
    _run(model, x, True)
    got = {n: profiling.counters[n] - before[n] for n in names}
    # tensor-core Linears: stage 1 qkv + proj (K = 48), stage 2 proj (K = 96, N = 96)
    assert got == {"swin_window_attention_qkv": 8, "norm_shift_partition_3d": 8,
                   "unshift_unpartition_crop_norm_3d": 8, "patch_merge_norm_3d": 4,
                   "proj_out_norm_3d": 5, "window_linear": 6}, got


def test_network_bf16_autocast(cuda_device):
    """bf16 autocast: the patched network is as faithful to the fp32 eager network as the
    eager bf16 network is (random-init logits have small class margins, so bf16 rounding
    alone flips ~1 % of the arg-maxes either way)."""
    torch.manual_seed(0)
    model = swin_unetr.SwinUNETR(1, 14, 48).to(cuda_device).eval()
    x = torch.rand((1, 1, 96, 96, 96), device=cuda_device)

    def run(patched, dtype):
        if patched:
            crumpet.patch_monai_swin_unetr(swin_unetr)
        try:
            with torch.no_grad(), torch.autocast("cuda", dtype=dtype, enabled=dtype is not None):
                return model(x).float()
        finally:
            crumpet.unpatch_monai_swin_unetr()

    ref = run(False, None)
    eager, patched = run(False, torch.bfloat16), run(True, torch.bfloat16)
    agree = lambda a: (a.argmax(1) == ref.argmax(1)).float().mean().item()
    a_e, a_p = agree(eager), agree(patched)
    d_e, d_p = (eager - ref).abs().max().item(), (patched - ref).abs().max().item()
    print(f"vs fp32: eager bf16 agree {a_e:.5f} diff {d_e:.4f}; patched bf16 agree {a_p:.5f} "
          f"diff {d_p:.4f}")
    assert a_p >= a_e - 0.005, (a_p, a_e)
    assert d_p <= 1.5 * d_e + 1e-2, (d_p, d_e)


def test_network_fp32_without_autocast(cuda_device):
    """fp32 activations: attention runs the module's eager forward, the fused norms,
    partition, merge and hidden-state kernels run in fp32.  cuDNN runs the UNETR
    convolutions in TF32 by default, which turns the norms' last-bit differences into
    ~1e-3 logit differences (1.4e-3 measured)."""
    torch.manual_seed(0)
    model = swin_unetr.SwinUNETR(1, 14, 48).to(cuda_device).eval()
    x = torch.rand((1, 1, 64, 64, 64), device=cuda_device)
    before = profiling.counters["norm_shift_partition_3d"]
    crumpet.patch_monai_swin_unetr(swin_unetr)
    try:
        with torch.no_grad():
            patched = model(x)
    finally:
        crumpet.unpatch_monai_swin_unetr()
    assert profiling.counters["norm_shift_partition_3d"] > before
    with torch.no_grad():
        eager = model(x)
    agree = (patched.argmax(1) == eager.argmax(1)).float().mean().item()
    diff = (patched - eager).abs().max().item()
    print(f"fp32 agreement {agree:.5f} max logit diff {diff:.2e}")
    assert agree >= 0.999, agree
    assert diff < 5e-3, diff


def test_cfg5_full_volume_patched_vs_eager(cuda_device):
    """BASELINE config 5 itself, as bench.py times it: the 1x1x512x512x224 synthetic
    volume, 96^3 ROIs at 0.5 overlap (400 ROIs), batches of 8, fp16 autocast, the
    patched network replayed from CUDA graphs -- against the unpatched eager network
    on the same GPU.  North-star criterion: segmentation arg-max agreement >= 99.9 %."""
    from crumpet_b200.inferer import roi_grid, synthetic_volume

    torch.manual_seed(0)
    model = swin_unetr.SwinUNETR(in_channels=1, out_channels=14, feature_size=48,
                                 depths=(2, 2, 2, 2), num_heads=(3, 6, 12, 24))
    model = model.to(cuda_device).eval()
    vol = synthetic_volume((1, 1, 512, 512, 224)).to(cuda_device)
    assert len(roi_grid((512, 512, 224), (96, 96, 96), 0.5)) == 400
    patched_inf = SlidingWindowInferer(model, (96, 96, 96), 8, 0.5, 14, torch.float16,
                                       cuda_graphs=True)
    crumpet.patch_monai_swin_unetr(swin_unetr)
    try:
        seg_p = patched_inf.segment(vol)
        logit_p = patched_inf.logits(vol)
    finally:
        crumpet.unpatch_monai_swin_unetr()
        patched_inf.reset_graphs()
    eager_inf = SlidingWindowInferer(model, (96, 96, 96), 8, 0.5, 14, torch.float16)
    logit_e = eager_inf.logits(vol)
    lab_p = logit_p[0].argmax(0).to(torch.uint8)
    lab_e = logit_e[0].argmax(0).to(torch.uint8)
    assert torch.equal(seg_p, lab_p)  # the arg-max kernel agrees with torch.argmax
    agree = (lab_p == lab_e).float().mean().item()
    max_diff = (logit_p - logit_e).abs().max().item()
    print(f"cfg5 full volume: arg-max agreement {agree:.6f}, max |logit diff| {max_diff:.4e}")
    assert agree >= 0.999, (agree, max_diff)
    assert max_diff < 5e-2, (agree, max_diff)
