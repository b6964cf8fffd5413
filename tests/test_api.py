"""Host-side behaviour that needs no GPU: the C ABI library, op registration,
argument validation, meta shapes and the mask cache (ports of the reference's
tests/test_padding.py, test_fake_tensor.py, test_cache.py)."""

from __future__ import annotations

import ctypes

import pytest
import torch

import crumpet_b200 as crumpet
from crumpet_b200 import _ops
from crumpet_b200.cache import clear_mask_cache, get_or_compute_mask, make_mask_key, mask_cache_info
from helpers import header_functions

REFERENCE_SCHEMAS = {
    "compute_attn_mask_3d": "crumpet_ops::compute_attn_mask_3d(Tensor($0! -> ) output, int D, int H, int W, int ws_d, int ws_h, int ws_w, int ss_d, int ss_h, int ss_w) -> ()",
    "fused_shift_partition_3d": "crumpet_ops::fused_shift_partition_3d(Tensor($0! -> ) output, Tensor x, int ws_d, int ws_h, int ws_w, int ss_d, int ss_h, int ss_w) -> ()",
    "fused_shift_partition_3d_backward": "crumpet_ops::fused_shift_partition_3d_backward(Tensor($0! -> ) grad_x, Tensor grad_windows, int B, int D, int H, int W, int C, int ws_d, int ws_h, int ws_w, int ss_d, int ss_h, int ss_w) -> ()",
    "fused_unshift_unpartition_3d": "crumpet_ops::fused_unshift_unpartition_3d(Tensor($0! -> ) output, Tensor windows, int B, int D, int H, int W, int C, int ws_d, int ws_h, int ws_w, int ss_d, int ss_h, int ss_w) -> ()",
    "fused_unshift_unpartition_3d_backward": "crumpet_ops::fused_unshift_unpartition_3d_backward(Tensor($0! -> ) grad_windows, Tensor grad_x, int ws_d, int ws_h, int ws_w, int ss_d, int ss_h, int ss_w) -> ()",
}


def test_capi_library_exports_every_declared_symbol():
    lib = _ops.capi()
    names = header_functions()
    assert len(names) >= 9
    for name in names:
        assert hasattr(lib, name), name
    assert lib.crumpet_abi_version() == 2


def test_capi_rejects_bad_arguments_without_touching_the_device():
    lib = _ops.capi()
    null = ctypes.c_void_p(0)
    # D not divisible by the window
    rc = lib.crumpet_fused_shift_partition_3d(null, null, 1, 1, 15, 14, 14, 4, 7, 7, 7, 3, 3, 3, null)
    assert rc == 1 and "divisible" in _ops.last_error()
    # shift >= window
    rc = lib.crumpet_fused_unshift_unpartition_3d(null, null, 1, 1, 14, 14, 14, 4, 7, 7, 7, 7, 0, 0, null)
    assert rc == 1 and "shift_size[0]" in _ops.last_error()
    # unknown dtype
    rc = lib.crumpet_compute_attn_mask_3d(null, 7, 14, 14, 14, 7, 7, 7, 3, 3, 3, null)
    assert rc == 1 and "float32" in _ops.last_error()
    # empty batch is a no-op
    rc = lib.crumpet_fused_shift_partition_3d(null, null, 1, 0, 14, 14, 14, 4, 7, 7, 7, 3, 3, 3, null)
    assert rc == 0
    # attention: unsupported head_dim / N / dtype, null pointers, and an empty batch
    rc = lib.crumpet_fused_swin_attention(null, null, null, null, null, null, 0, null, 1, 4, 3, 343, 48, 0.25, null)
    assert rc == 3 and "head_dim" in _ops.last_error()
    rc = lib.crumpet_fused_swin_attention(null, null, null, null, null, null, 0, null, 1, 4, 3, 0, 16, 0.25, null)
    assert rc == 3 and "N >= 1" in _ops.last_error()
    rc = lib.crumpet_fused_swin_attention(null, null, null, null, null, null, 0, null, 5, 4, 3, 343, 16, 0.25, null)
    assert rc == 3 and "float32" in _ops.last_error()
    for dtype, n, hd in ((0, 343, 16), (1, 343, 64), (1, 1000, 16), (2, 216, 256)):
        rc = lib.crumpet_fused_swin_attention(null, null, null, null, null, null, 0, null, dtype, 4, 3,
                                              n, hd, 0.25, null)
        assert rc == 1 and "null" in _ops.last_error()
    rc = lib.crumpet_fused_swin_attention(null, null, null, null, null, null, 0, null, 1, 0, 3, 343, 16, 0.25, null)
    assert rc == 0


def test_dispatcher_ops_keep_reference_schemas():
    ops = _ops.require()
    for name, schema in REFERENCE_SCHEMAS.items():
        assert str(getattr(ops, name).default._schema) == schema
    tags = ops.fused_shift_partition_3d.default.tags
    assert torch.Tag.pt2_compliant_tag in tags and torch.Tag.needs_fixed_stride_order in tags
    assert "Tensor? mask" in str(ops.fused_swin_attention.default._schema)
    assert str(ops.norm_shift_partition_3d.default._schema) == (
        "crumpet_ops::norm_shift_partition_3d(Tensor($0! -> ) output, Tensor x, Tensor weight, "
        "Tensor bias, float eps, int ws_d, int ws_h, int ws_w, int ss_d, int ss_h, int ss_w) -> ()")
    assert "Tensor(b!) normed" in str(ops.unshift_unpartition_crop_norm_3d.default._schema)
    assert str(ops.unshift_unpartition_crop_3d.default._schema) == (
        "crumpet_ops::unshift_unpartition_crop_3d(Tensor($0! -> ) output, Tensor windows, "
        "Tensor? residual, int B, int D, int H, int W, int C, int ws_d, int ws_h, int ws_w, "
        "int ss_d, int ss_h, int ss_w) -> ()")


def test_invalid_divisibility_fails_clearly():
    x = torch.randn((1, 15, 14, 14, 4))
    with pytest.raises(ValueError, match="divisible"):
        crumpet.fused_shift_partition_3d(x, (7, 7, 7), (3, 3, 3))


def test_invalid_shift_fails_clearly():
    x = torch.randn((1, 14, 14, 14, 4))
    with pytest.raises(ValueError, match="shift_size"):
        crumpet.fused_shift_partition_3d(x, (7, 7, 7), (7, 0, 0))


def test_bad_dtype_and_shape_errors():
    with pytest.raises(TypeError):
        crumpet.fused_shift_partition_3d(torch.zeros((1, 4, 4, 4, 2), dtype=torch.int32), (2, 2, 2), (1, 1, 1))
    with pytest.raises(ValueError, match="exactly three"):
        crumpet.fused_shift_partition_3d(torch.zeros((1, 4, 4, 4, 2)), (2, 2), (1, 1, 1))
    with pytest.raises(ValueError, match="windows must have shape"):
        crumpet.fused_unshift_unpartition_3d(torch.zeros((7, 8, 2)), 1, 4, 4, 4, 2, (2, 2, 2), (1, 1, 1))


def test_cpu_tensors_have_no_fallback():
    with pytest.raises(RuntimeError, match="CUDA"):
        crumpet.fused_shift_partition_3d(torch.zeros((1, 4, 4, 4, 2)), (2, 2, 2), (1, 1, 1))
    with pytest.raises(RuntimeError, match="CUDA"):
        crumpet.compute_attn_mask_3d(4, 4, 4, (2, 2, 2), (1, 1, 1), torch.float32, "cpu")


def test_meta_shape_propagation():
    x = torch.empty((2, 14, 14, 14, 48), device="meta", dtype=torch.float16)
    windows = crumpet.fused_shift_partition_3d(x, (7, 7, 7), (3, 3, 3))
    assert windows.shape == (16, 343, 48)
    restored = crumpet.fused_unshift_unpartition_3d(windows, 2, 14, 14, 14, 48, (7, 7, 7), (3, 3, 3))
    assert restored.shape == x.shape
    mask = crumpet.compute_attn_mask_3d(14, 14, 14, (7, 7, 7), (3, 3, 3), torch.float16, "meta")
    assert mask.shape == (8, 343, 343)


def test_cache_hit_and_miss():
    clear_mask_cache()
    calls = {"n": 0}
    key = make_mask_key(14, 14, 14, (7, 7, 7), (3, 3, 3), torch.float32, "cpu")

    def compute():
        calls["n"] += 1
        return torch.zeros((1,), dtype=torch.float32)

    a = get_or_compute_mask(key, compute)
    b = get_or_compute_mask(key, compute)
    assert a is b and calls["n"] == 1
    assert mask_cache_info()["entries"] == 1


def test_cache_disabled(monkeypatch):
    clear_mask_cache()
    monkeypatch.setenv("CRUMPET_DISABLE_MASK_CACHE", "1")
    key = make_mask_key(14, 14, 14, (7, 7, 7), (3, 3, 3), torch.float32, "cpu")
    a = get_or_compute_mask(key, lambda: torch.zeros((1,)))
    b = get_or_compute_mask(key, lambda: torch.ones((1,)))
    assert not torch.equal(a, b)


def test_cache_byte_cap(monkeypatch):
    clear_mask_cache()
    monkeypatch.setenv("CRUMPET_MASK_CACHE_MAX_BYTES", "1")
    key = make_mask_key(14, 14, 14, (7, 7, 7), (3, 3, 3), torch.float32, "cpu")
    get_or_compute_mask(key, lambda: torch.zeros((2,), dtype=torch.float32))
    assert mask_cache_info()["entries"] == 0


def test_cache_lru_eviction(monkeypatch):
    clear_mask_cache()
    monkeypatch.setenv("CRUMPET_MASK_CACHE_SIZE", "2")
    keys = [make_mask_key(d, 14, 14, (7, 7, 7), (3, 3, 3), torch.float32, "cpu") for d in (7, 14, 21)]
    for key in keys:
        get_or_compute_mask(key, lambda: torch.zeros((4,)))
    info = mask_cache_info()
    assert info["entries"] == 2 and info["bytes"] == 32


def test_reference_functions_round_trip_on_cpu():
    x = torch.randn((2, 8, 8, 8, 3))
    w = crumpet.unfused_shift_partition_3d_reference(x, (4, 4, 4), (2, 2, 2))
    back = crumpet.unfused_unshift_unpartition_3d_reference(w, 2, 8, 8, 8, 3, (4, 4, 4), (2, 2, 2))
    assert torch.equal(back, x)


def test_packed_attention_capi_validation():
    lib = _ops.capi()
    null = ctypes.c_void_p(0)
    # analytic geometry that does not multiply out to N
    rc = lib.crumpet_swin_window_attention_qkv(null, null, null, 1, 2197, null, 343, 2, 2, 2, 7, 7, 6, 3, 3,
                                               3, 1, 8, 3, 343, 16, 0.25, null)
    assert rc == 1 and _ops.last_error()
    # null pointers
    rc = lib.crumpet_swin_window_attention_qkv(null, null, null, 1, 2197, null, 343, 2, 2, 2, 7, 7, 7, 3, 3,
                                               3, 1, 8, 3, 343, 16, 0.25, null)
    assert rc == 1


def test_block_fusion_capi_validation():
    lib = _ops.capi()
    null = ctypes.c_void_p(0)
    norm = lib.crumpet_norm_shift_partition_3d
    # C not a multiple of 8 / above 768
    rc = norm(null, 1, null, 1, null, null, 1e-5, 1, 13, 10, 9, 44, 7, 7, 7, 3, 3, 3, null)
    assert rc == 3 and "multiple of 8" in _ops.last_error()
    rc = norm(null, 1, null, 1, null, null, 1e-5, 1, 13, 10, 9, 776, 7, 7, 7, 3, 3, 3, null)
    assert rc == 3
    # shift >= window, bad dtype, null pointers, empty batch
    rc = norm(null, 1, null, 1, null, null, 1e-5, 1, 13, 10, 9, 48, 7, 7, 7, 7, 3, 3, null)
    assert rc == 1 and "shift" in _ops.last_error()
    rc = norm(null, 5, null, 1, null, null, 1e-5, 1, 13, 10, 9, 48, 7, 7, 7, 3, 3, 3, null)
    assert rc == 1 and "float32" in _ops.last_error()
    rc = norm(null, 1, null, 1, null, null, 1e-5, 1, 13, 10, 9, 48, 7, 7, 7, 3, 3, 3, null)
    assert rc == 1 and "null" in _ops.last_error()
    rc = norm(null, 1, null, 1, null, null, 1e-5, 0, 13, 10, 9, 48, 7, 7, 7, 3, 3, 3, null)
    assert rc == 0
    # misaligned pointers (checked before any launch)
    rc = norm(ctypes.c_void_p(8), 1, ctypes.c_void_p(16), 1, ctypes.c_void_p(16), ctypes.c_void_p(16),
              1e-5, 1, 13, 10, 9, 48, 7, 7, 7, 3, 3, 3, null)
    assert rc == 1 and "aligned" in _ops.last_error()
    crop = lib.crumpet_unshift_unpartition_crop_3d
    rc = crop(null, null, null, 1, 1, 0, 10, 9, 48, 7, 7, 7, 3, 3, 3, null)
    assert rc == 1 and "positive" in _ops.last_error()
    rc = crop(null, null, null, 1, 1, 13, 10, 9, 48, 7, 7, 7, 3, 3, 3, null)
    assert rc == 1 and "null" in _ops.last_error()
    # fp16 rows of an odd C are not 4-byte multiples
    rc = crop(ctypes.c_void_p(16), ctypes.c_void_p(16), null, 1, 1, 13, 10, 9, 13, 7, 7, 7, 3, 3, 3,
              null)
    assert rc == 3
    rc = crop(null, null, null, 1, 0, 13, 10, 9, 48, 7, 7, 7, 3, 3, 3, null)
    assert rc == 0
    cnorm = lib.crumpet_unshift_unpartition_crop_norm_3d
    rc = cnorm(null, null, 1, null, null, 1, null, null, 1e-5, 1, 13, 10, 9, 44, 7, 7, 7, 3, 3, 3, null)
    assert rc == 3 and "multiple of 8" in _ops.last_error()
    rc = cnorm(null, null, 1, null, null, 1, null, null, 1e-5, 1, 13, 10, 9, 48, 7, 7, 7, 3, 3, 3, null)
    assert rc == 1 and "null" in _ops.last_error()
    rc = cnorm(null, null, 9, null, null, 1, null, null, 1e-5, 1, 13, 10, 9, 48, 7, 7, 7, 3, 3, 3, null)
    assert rc == 1 and "float32" in _ops.last_error()


def test_block_fusion_wrappers_validate_and_have_no_cpu_path():
    x = torch.randn(1, 13, 10, 9, 48)
    w, b = torch.ones(48), torch.zeros(48)
    with pytest.raises(ValueError, match="multiple of 8"):
        crumpet.norm_shift_partition_3d(torch.randn(1, 8, 8, 8, 12), torch.ones(12), torch.zeros(12),
                                        1e-5, (4, 4, 4), (2, 2, 2))
    with pytest.raises(ValueError, match="shift_size"):
        crumpet.norm_shift_partition_3d(x, w, b, 1e-5, (7, 7, 7), (7, 3, 3))
    with pytest.raises(RuntimeError, match="CUDA"):
        crumpet.norm_shift_partition_3d(x, w, b, 1e-5, (7, 7, 7), (3, 3, 3))
    meta = crumpet.norm_shift_partition_3d(x.to("meta"), w, b, 1e-5, (7, 7, 7), (3, 3, 3),
                                           torch.float16)
    assert meta.shape == (8, 343, 48) and meta.dtype == torch.float16
    win = torch.randn(8, 343, 48)
    with pytest.raises(ValueError, match="windows must have shape"):
        crumpet.unshift_unpartition_crop_3d(win, 1, 15, 10, 9, 48, (7, 7, 7), (3, 3, 3))
    with pytest.raises(TypeError, match="residual"):
        crumpet.unshift_unpartition_crop_3d(win, 1, 13, 10, 9, 48, (7, 7, 7), (3, 3, 3),
                                            residual=torch.randn(1, 13, 10, 9, 48).half())
    with pytest.raises(RuntimeError, match="CUDA"):
        crumpet.unshift_unpartition_crop_3d(win, 1, 13, 10, 9, 48, (7, 7, 7), (3, 3, 3))
    out = crumpet.unshift_unpartition_crop_3d(win.to("meta"), 1, 13, 10, 9, 48, (7, 7, 7), (3, 3, 3))
    assert out.shape == (1, 13, 10, 9, 48)


def test_patch_merge_capi_validation():
    lib = _ops.capi()
    null = ctypes.c_void_p(0)
    merge = lib.crumpet_patch_merge_norm_3d
    codes = (ctypes.c_int * 8)(*range(8))
    rc = merge(null, 1, null, 1, null, null, 1e-5, 1, 8, 8, 8, 12, codes, null)
    assert rc == 3 and "multiple of 8" in _ops.last_error()
    rc = merge(null, 1, null, 1, null, null, 1e-5, 1, 8, 8, 8, 392, codes, null)  # 8C = 3136
    assert rc == 3
    rc = merge(null, 1, null, 1, null, null, 1e-5, 1, 8, 8, 8, 48, None, null)
    assert rc == 1 and "part table" in _ops.last_error()
    bad = (ctypes.c_int * 8)(0, 1, 2, 3, 4, 5, 6, 8)
    rc = merge(null, 1, null, 1, null, null, 1e-5, 1, 8, 8, 8, 48, bad, null)
    assert rc == 1 and "0..7" in _ops.last_error()
    rc = merge(null, 7, null, 1, null, null, 1e-5, 1, 8, 8, 8, 48, codes, null)
    assert rc == 1 and "float32" in _ops.last_error()
    rc = merge(null, 1, null, 1, null, null, 1e-5, 1, 8, 8, 8, 48, codes, null)
    assert rc == 1 and "null" in _ops.last_error()
    rc = merge(ctypes.c_void_p(8), 1, ctypes.c_void_p(16), 1, ctypes.c_void_p(16),
               ctypes.c_void_p(16), 1e-5, 1, 8, 8, 8, 48, codes, null)
    assert rc == 1 and "aligned" in _ops.last_error()
    rc = merge(null, 1, null, 1, null, null, 1e-5, 0, 8, 8, 8, 48, codes, null)
    assert rc == 0


def test_patch_merge_wrapper_validates_and_has_no_cpu_path():
    w, b = torch.ones(384), torch.zeros(384)
    with pytest.raises(ValueError, match="multiple of 8"):
        crumpet.patch_merge_norm_3d(torch.randn(1, 4, 4, 4, 12), torch.ones(96), torch.zeros(96), 1e-5)
    with pytest.raises(ValueError, match=r"\[8C\]"):
        crumpet.patch_merge_norm_3d(torch.randn(1, 4, 4, 4, 48), torch.ones(48), torch.zeros(48), 1e-5)
    with pytest.raises(ValueError, match="eight"):
        crumpet.patch_merge_norm_3d(torch.randn(1, 4, 4, 4, 48), w, b, 1e-5, order=[(0, 0, 0)] * 7)
    with pytest.raises(ValueError, match="eight"):
        crumpet.patch_merge_norm_3d(torch.randn(1, 4, 4, 4, 48), w, b, 1e-5,
                                    order=[(0, 0, 2)] + [(0, 0, 0)] * 7)
    with pytest.raises(RuntimeError, match="CUDA"):
        crumpet.patch_merge_norm_3d(torch.randn(1, 4, 4, 4, 48), w, b, 1e-5)
    meta = crumpet.patch_merge_norm_3d(torch.empty(2, 7, 6, 5, 48, device="meta"), w, b, 1e-5,
                                       out_dtype=torch.float16)
    assert meta.shape == (2, 4, 3, 3, 384) and meta.dtype == torch.float16


def test_proj_out_norm_capi_validation():
    lib = _ops.capi()
    null = ctypes.c_void_p(0)
    pn = lib.crumpet_proj_out_norm_3d
    rc = pn(null, 0, null, 1, null, null, 1e-5, 1, 44, 4, 4, 4, null)
    assert rc == 3 and "multiple of 8" in _ops.last_error()
    rc = pn(null, 0, null, 1, null, null, 1e-5, 1, 776, 4, 4, 4, null)
    assert rc == 3
    rc = pn(null, 0, null, 1, null, null, 1e-5, 1, 200, 4, 4, 4, null)  # 200 / 16 lanes
    assert rc == 3 and "lanes" in _ops.last_error()
    rc = pn(null, 0, null, 1, ctypes.c_void_p(16), null, 1e-5, 1, 48, 4, 4, 4, null)
    assert rc == 1 and "both" in _ops.last_error()
    rc = pn(null, 0, null, 6, null, null, 1e-5, 1, 48, 4, 4, 4, null)
    assert rc == 1 and "float32" in _ops.last_error()
    rc = pn(null, 0, null, 1, null, null, 1e-5, 1, 48, 4, 0, 4, null)
    assert rc == 1 and "dims" in _ops.last_error()
    rc = pn(null, 0, null, 1, null, null, 1e-5, 1, 48, 4, 4, 4, null)
    assert rc == 1 and "null" in _ops.last_error()
    rc = pn(ctypes.c_void_p(16), 0, ctypes.c_void_p(18), 1, null, null, 1e-5, 1, 48, 4, 4, 4, null)
    assert rc == 1 and "aligned" in _ops.last_error()
    rc = pn(null, 0, null, 1, null, null, 1e-5, 0, 48, 4, 4, 4, null)
    assert rc == 0


def test_proj_out_norm_wrapper_validates_and_keeps_monai_strides():
    from crumpet_b200.block_fusion import proj_out_lanes

    assert [proj_out_lanes(c) for c in (24, 48, 96, 192, 384, 768, 64, 200, 12)] == \
        [1, 2, 4, 8, 16, 32, 4, 0, 0]
    with pytest.raises(ValueError, match="multiple of 8"):
        crumpet.proj_out_norm_3d(torch.randn(1, 12, 4, 4, 4))
    with pytest.raises(ValueError, match="both"):
        crumpet.proj_out_norm_3d(torch.randn(1, 48, 4, 4, 4), weight=torch.ones(48))
    with pytest.raises(ValueError, match=r"\[C\]"):
        crumpet.proj_out_norm_3d(torch.randn(1, 48, 4, 4, 4), weight=torch.ones(8),
                                 bias=torch.zeros(8))
    with pytest.raises(TypeError):
        crumpet.proj_out_norm_3d(torch.zeros(1, 48, 4, 4, 4, dtype=torch.int32))
    with pytest.raises(RuntimeError, match="CUDA"):
        crumpet.proj_out_norm_3d(torch.randn(1, 48, 4, 4, 4))
    x = torch.empty(2, 96, 7, 6, 5, device="meta", dtype=torch.float16)
    got = crumpet.proj_out_norm_3d(x, out_dtype=torch.float32)
    want = torch.nn.functional.layer_norm(torch.empty(2, 96, 7, 6, 5).permute(0, 2, 3, 4, 1),
                                          [96]).permute(0, 4, 1, 2, 3)
    assert got.shape == want.shape and got.stride() == want.stride()
    assert got.dtype == torch.float32


def test_window_linear_capi_validation():
    lib = _ops.capi()
    null = ctypes.c_void_p(0)
    lin = lib.crumpet_window_linear
    rc = lin(null, null, null, null, 0, 100, 48, 144, null)  # float32 operands
    assert rc == 1 and "float16" in _ops.last_error()
    rc = lin(null, null, null, null, 1, 100, 64, 144, null)  # K = 64
    assert rc == 3 and "K = 48" in _ops.last_error()
    rc = lin(null, null, null, null, 1, 100, 96, 288, null)  # stage-2 qkv: does not fit
    assert rc == 3
    rc = lin(null, null, null, null, 1, 100, 48, 100, null)  # N not a multiple of 16
    assert rc == 3
    rc = lin(null, null, null, null, 1, 100, 48, 144, null)
    assert rc == 1 and "null" in _ops.last_error()
    rc = lin(ctypes.c_void_p(16), ctypes.c_void_p(24), ctypes.c_void_p(16), null, 1, 100, 48, 144,
             null)
    assert rc == 1 and "aligned" in _ops.last_error()
    rc = lin(null, null, null, null, 1, 0, 48, 144, null)
    assert rc == 0


def test_window_linear_wrapper_validates_and_has_no_cpu_path():
    w, b = torch.randn(144, 48), torch.randn(144)
    with pytest.raises(TypeError, match="float16"):
        crumpet.window_linear(torch.randn(10, 48), w, b)
    x = torch.randn(10, 48).half()
    with pytest.raises(ValueError, match="K = 48"):
        crumpet.window_linear(torch.randn(10, 64).half(), torch.randn(144, 64), b)
    with pytest.raises(ValueError, match=r"\[N, K\]"):
        crumpet.window_linear(x, torch.randn(144, 32), b)
    with pytest.raises(ValueError, match=r"\[N\]"):
        crumpet.window_linear(x, w, torch.randn(12))
    with pytest.raises(RuntimeError, match="CUDA"):
        crumpet.window_linear(x, w, b)
    out = crumpet.window_linear(torch.empty(3, 343, 48, dtype=torch.float16, device="meta"), w, b)
    assert out.shape == (3, 343, 144) and out.dtype == torch.float16


def test_roi_capi_validation():
    lib = _ops.capi()
    null = ctypes.c_void_p(0)
    starts = (ctypes.c_int64 * 6)(0, 0, 0, 10, 0, 0)
    # ROI past the volume end, too many ROIs, null pointers, empty batch
    rc = lib.crumpet_roi_gather(null, 1, null, 0, 1, 100, 96, 96, starts, 2, 96, 96, 96, null)
    assert rc == 1 and "outside" in _ops.last_error()
    rc = lib.crumpet_roi_gather(null, 1, null, 0, 1, 200, 96, 96, starts, 65, 96, 96, 96, null)
    assert rc == 1 and "64" in _ops.last_error()
    rc = lib.crumpet_roi_gather(null, 1, null, 0, 1, 200, 96, 96, starts, 2, 96, 96, 96, null)
    assert rc == 1 and "null" in _ops.last_error()
    rc = lib.crumpet_roi_gather(null, 1, null, 0, 1, 200, 96, 96, starts, 0, 96, 96, 96, null)
    assert rc == 0
    rc = lib.crumpet_roi_accumulate(null, null, 1, 14, 200, 96, 96, starts, 2, 96, 96, 96, null)
    assert rc == 1 and "null" in _ops.last_error()
    rc = lib.crumpet_roi_accumulate(null, null, 7, 14, 200, 96, 96, starts, 2, 96, 96, 96, null)
    assert rc == 1 and "float32" in _ops.last_error()
    rc = lib.crumpet_roi_argmax(null, null, null, null, null, null, 300, 8, 8, 8, null)
    assert rc == 1 and "classes" in _ops.last_error()


def test_axis_counts_factorise_the_count_map():
    from crumpet_b200.inferer import SlidingWindowInferer, axis_counts

    inf = SlidingWindowInferer(None, (8, 6, 5), 2, 0.5, 3)
    spatial = (20, 13, 11)
    full = inf._count_map(spatial, torch.device("cpu"))[0, 0]
    cd, ch, cw = (torch.tensor(axis_counts(s, r, 0.5)) for s, r in zip(spatial, (8, 6, 5)))
    assert torch.equal(full, cd[:, None, None] * ch[None, :, None] * cw[None, None, :])


def test_loader_reload_is_idempotent():
    # a build running in the process that imported the package calls these afterwards
    assert _ops.reload() is True
    crumpet._register_fake_impls()
    crumpet._register_fake_impls()
    assert _ops.available()


def _ctype_of(c_type: str):
    """The ctypes class a C parameter or return type of the header must be bound as."""
    if c_type.replace(" ", "") == "constchar*":
        return ctypes.c_char_p
    if "*" in c_type:
        return ctypes.c_void_p
    base = c_type.replace("const ", "").strip()
    return {"int": ctypes.c_int, "int64_t": ctypes.c_int64, "float": ctypes.c_float}[base]


def test_ctypes_bindings_match_the_header():
    """Every function of include/crumpet_b200.h is bound in _ops.capi() with exactly the
    header's parameter list and return type (a wrong count or width would pass garbage to
    the kernels without any error)."""
    from helpers import header_prototypes

    protos = header_prototypes()
    assert set(protos) == set(header_functions())
    lib = _ops.capi()
    for name, (ret, params) in protos.items():
        fn = getattr(lib, name)
        assert fn.argtypes is not None, f"{name} has no argtypes"
        want = [_ctype_of(t) for t in params]
        got = list(fn.argtypes)
        assert len(got) == len(want), (name, len(got), len(want))
        for i, (g, w) in enumerate(zip(got, want)):
            assert g is w, (name, i, params[i], g, w)
        assert fn.restype is _ctype_of(ret), (name, ret, fn.restype)
