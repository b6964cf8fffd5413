"""The CPU oracle against the reference's own golden fixtures (no GPU)."""

from __future__ import annotations

import hashlib
import json
from pathlib import Path

import numpy as np
import pytest
import torch

import inputs as I
from oracle import attention as OA
from oracle import block as OB
from oracle import mechanics as OM

GOLDEN = Path(__file__).resolve().parent / "golden"
MANIFEST = json.loads((GOLDEN / "manifest.json").read_text())
SMALL_MECH = [c for c in I.MECHANICS_CASES if np.prod(c[1]) <= 2 * 28**3 * 48]
SMALL_MASK = [c for c in I.MASK_CASES if np.prod(c[1]) <= 28**3]


def sha(t: torch.Tensor) -> str:
    return hashlib.sha256(t.contiguous().view(-1).view(torch.uint8).numpy().tobytes()).hexdigest()


def to_np(t: torch.Tensor) -> np.ndarray:
    # numpy has no bfloat16: carry the raw 16-bit patterns (copies are exact)
    if t.dtype == torch.bfloat16:
        return t.view(torch.int16).numpy()
    return t.numpy()


def from_np(a: np.ndarray, dtype: torch.dtype) -> torch.Tensor:
    t = torch.from_numpy(np.ascontiguousarray(a))
    return t.view(dtype) if dtype == torch.bfloat16 else t


@pytest.mark.parametrize("case", SMALL_MECH, ids=[c[0] for c in SMALL_MECH])
def test_oracle_partition_matches_reference_digest(case):
    name, shape, ws, ss, dtype, seed = case
    x = I.mechanics_input(case)
    assert sha(x) == MANIFEST["mechanics"][name]["input_sha256"]
    win = from_np(OM.shift_partition(to_np(x), ws, ss), x.dtype)
    assert list(win.shape) == MANIFEST["mechanics"][name]["partition_shape"]
    assert sha(win) == MANIFEST["mechanics"][name]["partition_sha256"]
    back = from_np(OM.unshift_unpartition(to_np(win), *shape, ws, ss), x.dtype)
    assert torch.equal(back, x)


@pytest.mark.parametrize("case", SMALL_MASK, ids=[c[0] for c in SMALL_MASK])
def test_oracle_mask_matches_reference_digest(case):
    name, dims, ws, ss, dtype = case
    m = torch.from_numpy(OM.attn_mask(*dims, ws, ss, np.float32)).to(getattr(torch, dtype))
    assert list(m.shape) == MANIFEST["mask"][name]["shape"]
    assert sha(m) == MANIFEST["mask"][name]["sha256"]


def test_partition_mapping_is_bijective():
    # tests/test_correctness.py:100-114 of the reference, on the oracle's index map
    idx = OM.window_source_index(14, 14, 14, (7, 7, 7), (3, 3, 3))
    assert np.unique(idx).size == idx.size == 14**3


@pytest.mark.parametrize("case", I.ATTENTION_CASES, ids=[c[0] for c in I.ATTENTION_CASES])
def test_oracle_attention_matches_reference_triton(case):
    q, k, v, bias, mask, boundary = I.attention_inputs(case)
    f = lambda t: None if t is None else t.float().numpy()
    got = OA.window_attention(f(q), f(k), f(v), f(bias), f(mask),
                              None if boundary is None else boundary.numpy())
    ref = np.load(GOLDEN / "attention_ref_out.npz")[case[0]]
    # The reference kernel rounds q*scale and P to the input precision and
    # its output to fp16/bf16; the oracle is exact float64.
    tol = 1e-2 if q.dtype == torch.bfloat16 else 2e-3
    assert np.abs(got - ref).max() <= tol


def test_relative_position_index_quirk():
    full = OA.relative_position_index((7, 7, 7))
    assert full.shape == (343, 343) and full.min() == 0 and full.max() == 13**3 - 1
    assert np.array_equal(full[:216, :216], I.relative_index((7, 7, 7))[:216, :216])


BLOCK_REF = np.load(GOLDEN / "block_ref.npz")


@pytest.mark.parametrize("case", I.BLOCK_CASES, ids=[c[0] for c in I.BLOCK_CASES])
def test_oracle_block_glue_matches_reference_forward_part1(case):
    """norm1 -> pad -> roll + partition and unpartition -> crop, against the
    outputs of the reference's own patched forward_part1 (monai_patch.py:72-114)."""
    name, shape, window, shift, _ = case
    x, w, b, eps = I.block_inputs(case)
    ws, ss = OB.window_geometry(shape[1:4], window, shift)
    win = OB.norm_shift_partition(x.numpy(), w.numpy(), b.numpy(), eps, ws, ss)
    ref_win = BLOCK_REF[name + ".windows"]
    assert list(win.shape) == MANIFEST["block"][name]["windows_shape"] == list(ref_win.shape)
    np.testing.assert_allclose(win, ref_win, rtol=0, atol=2e-5)
    attn = I.block_attn_output(case, win.shape).numpy()
    out = OB.unshift_unpartition_crop(attn, *shape, ws, ss)
    assert sha(torch.from_numpy(out)) == MANIFEST["block"][name]["out_sha256"]
    assert np.array_equal(out, BLOCK_REF[name + ".out"])
