"""The registry that lets fused_swin_attention recognise masks compute_attn_mask_3d built
(host logic only): a mask is recognised until anyone writes to it, copies are not, and
collected masks drop out."""

from __future__ import annotations

import gc

import torch

from crumpet_b200 import cache
from crumpet_b200.cache import mask_geometry, remember_mask_geometry


def test_mask_geometry_follows_writes():
    m = torch.zeros(8, 343, 343)
    assert mask_geometry(m) is None
    remember_mask_geometry(m, (2, 2, 2), (7, 7, 7), (3, 3, 3))
    assert mask_geometry(m) == ((2, 2, 2), (7, 7, 7), (3, 3, 3))
    assert mask_geometry(m.clone()) is None
    m.add_(0)  # any in-place write, even one that keeps the values
    assert mask_geometry(m) is None


def test_registry_forgets_collected_masks():
    m = torch.zeros(2, 8, 8)
    remember_mask_geometry(m, (1, 1, 2), (2, 2, 2), (1, 1, 1))
    key = id(m)
    assert key in cache._GEOMETRY
    del m
    gc.collect()
    assert key not in cache._GEOMETRY


def test_inference_tensors_are_never_recognised():
    with torch.inference_mode():
        m = torch.zeros(8, 343, 343)
    remember_mask_geometry(m, (2, 2, 2), (7, 7, 7), (3, 3, 3))  # must not raise
    assert mask_geometry(m) is None
