"""Patch / unpatch contract, the bundled MONAI-architecture network and the ROI
driver, on the CPU (reference tests/test_monai_patch.py, plus the pieces the
end-to-end run relies on)."""

from __future__ import annotations

import numpy as np
import pytest
import torch

import crumpet_b200 as crumpet
from crumpet_b200 import monai_patch, swin_unetr
from crumpet_b200.inferer import SlidingWindowInferer, axis_starts, roi_grid
from oracle import mechanics as OM


def test_patch_unpatch_repeated_safe():
    def current():
        return (swin_unetr.SwinTransformerBlock.forward_part1, swin_unetr.SwinTransformerBlock.forward,
                swin_unetr.BasicLayer.forward, swin_unetr.WindowAttention.forward,
                swin_unetr.SwinTransformer.__dict__["proj_out"])

    originals = current()
    assert crumpet.patch_monai_swin_unetr(swin_unetr) is True
    assert crumpet.patch_monai_swin_unetr(swin_unetr) is False
    assert all(p is not o for p, o in zip(current(), originals))
    assert crumpet.unpatch_monai_swin_unetr() is True
    assert crumpet.unpatch_monai_swin_unetr() is False
    assert current() == originals


def test_patch_without_monai_raises():
    try:
        import monai  # noqa: F401
    except ImportError:
        with pytest.raises(RuntimeError, match="MONAI"):
            crumpet.patch_monai_swin_unetr()
    else:
        pytest.skip("MONAI is installed")


def test_fused_attention_opt_out(monkeypatch):
    monkeypatch.setenv("CRUMPET_DISABLE_FUSED_ATTN", "1")
    original = swin_unetr.WindowAttention.forward
    assert crumpet.patch_monai_swin_unetr(swin_unetr)
    try:
        assert swin_unetr.WindowAttention.forward is original
    finally:
        crumpet.unpatch_monai_swin_unetr()


def test_patched_proj_out_keeps_eager_semantics_off_gpu():
    """The patched hidden-state norm works as a bound method of the trunk and hands
    anything the kernel does not take (CPU tensors, normalize=False) to the original."""
    trunk = swin_unetr.SwinTransformer(1, 24, (7, 7, 7), (2, 2, 2), (1, 1, 1, 1), (3, 3, 3, 3))
    x = torch.randn(1, 24, 5, 6, 7)
    assert crumpet.patch_monai_swin_unetr(swin_unetr)
    try:
        assert trunk.proj_out(x, False) is x
        want = torch.nn.functional.layer_norm(x.permute(0, 2, 3, 4, 1), [24]).permute(0, 4, 1, 2, 3)
        assert torch.equal(trunk.proj_out(x, True), want)
    finally:
        crumpet.unpatch_monai_swin_unetr()
    assert isinstance(swin_unetr.SwinTransformer.__dict__["proj_out"], staticmethod)


def test_merge_fusion_plumbing_on_meta():
    """The channels-first patch-merging path: the module's own norm and reduction
    parameters go to the fused op, and the output is [B, 2C, D', H', W']."""
    ds = swin_unetr.PatchMerging(48, norm_layer=torch.nn.LayerNorm, spatial_dims=3)
    assert monai_patch._merge_order(ds) == crumpet.block_fusion.PRODUCT_ORDER
    x = torch.empty((2, 7, 6, 5, 48), device="meta")
    out = monai_patch._merge_channels_first(ds.to("meta"), x)
    assert out.shape == (2, 96, 4, 3, 3)
    assert not monai_patch._merge_fusable(ds, x)  # meta tensors take the eager path

    class Other(torch.nn.Module):
        pass

    assert monai_patch._merge_order(Other()) is None


def test_swin_unetr_shapes_and_parameter_count():
    model = swin_unetr.SwinUNETR(1, 14, 48)
    assert sum(p.numel() for p in model.parameters()) == 62_187_296
    small = swin_unetr.SwinUNETR(1, 3, 12, depths=(1, 1, 1, 1)).eval()
    with torch.no_grad():
        out = small(torch.rand((1, 1, 64, 64, 64)))
    assert out.shape == (1, 3, 64, 64, 64)


def test_eager_mask_matches_oracle():
    m = swin_unetr.compute_mask((14, 14, 14), (7, 7, 7), (3, 3, 3), "cpu")
    assert np.array_equal(m.numpy(), OM.attn_mask(14, 14, 14, (7, 7, 7), (3, 3, 3)))


@pytest.mark.parametrize("dims,ws,ss", [((49, 49, 49), (7, 7, 7), (3, 3, 3)),
                                         ((28, 28, 28), (7, 7, 7), (3, 3, 3)),
                                         ((14, 21, 7), (7, 7, 7), (3, 0, 2)),
                                         ((6, 6, 6), (6, 6, 6), (0, 0, 0))])
def test_boundary_flags_closed_form(dims, ws, ss):
    mask = OM.attn_mask(*dims, ws, ss)
    want = (np.abs(mask).reshape(mask.shape[0], -1).max(axis=1) > 0).astype(np.uint8)
    got = monai_patch.boundary_flags(dims, ws, ss, "cpu").numpy()
    assert np.array_equal(got, want)


def test_roi_grid_matches_config():
    assert axis_starts(512, 96, 0.5) == [0, 48, 96, 144, 192, 240, 288, 336, 384, 416]
    assert axis_starts(224, 96, 0.5) == [0, 48, 96, 128]
    assert len(roi_grid((512, 512, 224), (96, 96, 96), 0.5)) == 400
    assert axis_starts(64, 96, 0.5) == [0]


@pytest.mark.parametrize("world", [1, 2, 3, 4, 8])
def test_roi_sharding_partitions_the_batches(world):
    inf = [SlidingWindowInferer(None, (96,) * 3, 8, 0.5, rank=r, world=world) for r in range(world)]
    per_rank = [[roi for b in i.my_batches((512, 512, 224)) for roi in b] for i in inf]
    seen = [roi for rois in per_rank for roi in rois]
    # every ROI exactly once, in grid order, ranks balanced to one ROI
    assert seen == roi_grid((512, 512, 224), (96,) * 3, 0.5)
    assert max(map(len, per_rank)) - min(map(len, per_rank)) <= 1
    assert all(len(b) <= 8 for i in inf for b in i.my_batches((512, 512, 224)))
    # the fewest batches, as equal as possible (no two-ROI tail batch at 8 ranks)
    for i in inf:
        sizes = [len(b) for b in i.my_batches((512, 512, 224))]
        assert len(sizes) == -(-sum(sizes) // 8) and max(sizes) - min(sizes) <= 1


def test_sliding_window_eager_cpu_matches_single_forward():
    # a volume equal to one ROI: the sliding-window result is the plain forward
    torch.manual_seed(0)
    model = swin_unetr.SwinUNETR(1, 3, 12, depths=(1, 1, 1, 1)).eval()
    x = torch.rand((1, 1, 64, 64, 64))
    inf = SlidingWindowInferer(model, (64, 64, 64), 1, 0.5, num_classes=3, autocast_dtype=None)
    with torch.no_grad():
        got = inf.logits(x)
        want = model(x)
    assert torch.allclose(got, want)


def test_cuda_graphs_option_leaves_cpu_volumes_on_the_eager_path():
    # graphs apply to CUDA volumes only: a CPU volume runs the eager loop and captures nothing
    torch.manual_seed(0)
    model = swin_unetr.SwinUNETR(1, 3, 12, depths=(1, 1, 1, 1)).eval()
    x = torch.rand((1, 1, 64, 64, 80))
    plain = SlidingWindowInferer(model, (64, 64, 64), 1, 0.5, num_classes=3, autocast_dtype=None)
    graphed = SlidingWindowInferer(model, (64, 64, 64), 1, 0.5, num_classes=3,
                                   autocast_dtype=None, cuda_graphs=True)
    assert torch.equal(graphed.logits(x), plain.logits(x))
    assert torch.equal(graphed.segment(x), plain.segment(x))
    assert graphed._graphs == {}
    graphed.reset_graphs()
    assert graphed._graphs == {}
