"""Deterministic inputs shared by the golden-fixture generator and the tests.

Every input is regenerated from a seed with numpy's PCG64 generator (fp32
standard normal) and converted to the target dtype by torch, so the tests,
the fixture script and the GPU box build bit-identical tensors without storing
them.
"""

from __future__ import annotations

import numpy as np
import torch

# (name, (B, D, H, W, C), window, shift, dtype, seed)
MECHANICS_CASES = [
    ("c14_ws7_ss3_C13", (2, 14, 14, 14, 13), (7, 7, 7), (3, 3, 3), "float32", 11),
    ("c14_ws7_ss0_C48", (2, 14, 14, 14, 48), (7, 7, 7), (0, 0, 0), "float32", 12),
    ("c8_ws4_ss2_C7", (2, 8, 8, 8, 7), (4, 4, 4), (2, 2, 2), "float32", 13),
    ("dtype_f32", (1, 8, 8, 8, 4), (4, 4, 4), (2, 2, 2), "float32", 14),
    ("dtype_f16", (1, 8, 8, 8, 4), (4, 4, 4), (2, 2, 2), "float16", 14),
    ("dtype_bf16", (1, 8, 8, 8, 4), (4, 4, 4), (2, 2, 2), "bfloat16", 14),
    ("nonuniform_642_f16_C13", (3, 6, 4, 2, 13), (2, 2, 2), (1, 1, 1), "float16", 15),
    ("mixed_shift_f16", (1, 14, 21, 7, 24), (7, 7, 7), (3, 0, 2), "float16", 16),
    ("cfg1_28_f32", (1, 28, 28, 28, 48), (7, 7, 7), (3, 3, 3), "float32", 0),
    ("cfg4_28_f16_C96", (1, 28, 28, 28, 96), (7, 7, 7), (3, 3, 3), "float16", 41),
    ("cfg4_14_f16_C192", (1, 14, 14, 14, 192), (7, 7, 7), (3, 3, 3), "float16", 42),
    ("cfg4_7_f16_C384", (1, 7, 7, 7, 384), (7, 7, 7), (0, 0, 0), "float16", 43),
    ("cfg4_28_bf16_B4", (4, 28, 28, 28, 96), (7, 7, 7), (3, 3, 3), "bfloat16", 44),
    ("cfg2_98_f16", (1, 98, 98, 98, 48), (7, 7, 7), (3, 3, 3), "float16", 2),
]

# (name, (D, H, W), window, shift, dtype)
MASK_CASES = [
    ("m14_ws7_ss3_f32", (14, 14, 14), (7, 7, 7), (3, 3, 3), "float32"),
    ("m14_ws7_ss0_f32", (14, 14, 14), (7, 7, 7), (0, 0, 0), "float32"),
    ("m8_ws4_ss2_f32", (8, 8, 8), (4, 4, 4), (2, 2, 2), "float32"),
    ("m642_ws2_ss1_f32", (6, 4, 2), (2, 2, 2), (1, 1, 1), "float32"),
    ("m8_ws4_ss2_f16", (8, 8, 8), (4, 4, 4), (2, 2, 2), "float16"),
    ("m8_ws4_ss2_bf16", (8, 8, 8), (4, 4, 4), (2, 2, 2), "bfloat16"),
    ("m14x21x7_mixed_f16", (14, 21, 7), (7, 7, 7), (3, 0, 2), "float16"),
    ("m28_cfg1_f32", (28, 28, 28), (7, 7, 7), (3, 3, 3), "float32"),
    ("m98_cfg2_f16", (98, 98, 98), (7, 7, 7), (3, 3, 3), "float16"),
]

# (name, B, H, runtime window (gives N), configured window (gives the bias
#  table and index, sliced [:N, :N]), mask volume or None, mask shift, dtype,
#  seed, q/k scale)
ATTENTION_CASES = [
    ("a_n343_h3_mask_f16", 8, 3, (7, 7, 7), (7, 7, 7), (14, 14, 14), (3, 3, 3), "float16", 21, 1.0),
    ("a_n343_h3_small_f16", 4, 3, (7, 7, 7), (7, 7, 7), None, None, "float16", 22, 0.15),
    ("a_n216_h6_quirk_f16", 2, 6, (6, 6, 6), (7, 7, 7), None, None, "float16", 24, 1.0),
    ("a_n64_h2_mask_f16", 8, 2, (4, 4, 4), (4, 4, 4), (8, 8, 8), (2, 2, 2), "float16", 25, 1.0),
    # head_dim 32 (feature size 96 models): an optional 11th field
    ("a_n64_h2_d32_mask_f16", 8, 2, (4, 4, 4), (4, 4, 4), (8, 8, 8), (2, 2, 2), "float16", 31,
     1.0, 32),
    ("a_n125_h3_d32_f16", 3, 3, (5, 5, 5), (5, 5, 5), None, None, "float16", 32, 1.0, 32),
]

# Checked against the oracle only: the Triton CPU interpreter does not model
# bfloat16 (numpy has no such type), and it crashes on the N=343 head_dim 32
# launch, so these have no reference-kernel golden.
ORACLE_ONLY_ATTENTION_CASES = [
    ("a_n343_h2_d32_mask_f16", 8, 2, (7, 7, 7), (7, 7, 7), (14, 14, 14), (3, 3, 3), "float16", 34,
     1.0, 32),
    ("a_n343_h3_mask_bf16", 8, 3, (7, 7, 7), (7, 7, 7), (14, 14, 14), (3, 3, 3), "bfloat16", 23, 1.0),
    ("a_n125_h4_f16", 3, 4, (5, 5, 5), (5, 5, 5), None, None, "float16", 26, 1.0),
    ("a_n8_h1_f16", 5, 1, (2, 2, 2), (2, 2, 2), None, None, "float16", 27, 1.0),
    ("a_n343_h12_f16", 8, 12, (7, 7, 7), (7, 7, 7), (14, 14, 14), (3, 3, 3), "float16", 28, 1.0),
    ("a_n343_h2_d32_mask_bf16", 8, 2, (7, 7, 7), (7, 7, 7), (14, 14, 14), (3, 3, 3), "bfloat16",
     33, 1.0, 32),
]


def randn(seed: int, shape, dtype: str) -> torch.Tensor:
    rng = np.random.default_rng(seed)
    a = rng.standard_normal(size=tuple(shape), dtype=np.float32)
    return torch.from_numpy(a).to(getattr(torch, dtype))


def mechanics_input(case) -> torch.Tensor:
    _, shape, _, _, dtype, seed = case
    return randn(seed, shape, dtype)


def relative_index(window) -> np.ndarray:
    wd, wh, ww = window
    coords = np.stack(np.meshgrid(np.arange(wd), np.arange(wh), np.arange(ww), indexing="ij"))
    coords = coords.reshape(3, -1)
    rel = coords[:, :, None] - coords[:, None, :]
    rel = rel + np.array([wd - 1, wh - 1, ww - 1])[:, None, None]
    return rel[0] * (2 * wh - 1) * (2 * ww - 1) + rel[1] * (2 * ww - 1) + rel[2]


def attention_inputs(case, mask_fn=None):
    """q, k, v [B,H,N,hd] (hd 16 unless the case gives it); bias [H,N,N]; mask [nW,N,N] or None;
    boundary [B] or None.

    The bias follows the MONAI quirk: the table and index belong to the
    configured window and are sliced [:N, :N] when the runtime window is
    smaller.  ``mask_fn(D, H, W, window, shift)`` -> float32 numpy mask
    defaults to the test oracle.
    """
    name, B, H, window, cfg, mvol, mshift, dtype, seed, qscale = case[:10]
    hd = case[10] if len(case) > 10 else 16
    n = window[0] * window[1] * window[2]
    q = (randn(seed, (B, H, n, hd), "float32") * qscale).to(getattr(torch, dtype))
    k = (randn(seed + 1, (B, H, n, hd), "float32") * qscale).to(getattr(torch, dtype))
    v = randn(seed + 2, (B, H, n, hd), dtype)
    table = randn(seed + 3, ((2 * cfg[0] - 1) * (2 * cfg[1] - 1) * (2 * cfg[2] - 1), H), "float32")
    table = table * 0.5
    idx = relative_index(cfg)[:n, :n]
    bias = table[torch.from_numpy(idx.reshape(-1))].reshape(n, n, H).permute(2, 0, 1)
    bias = bias.contiguous().to(getattr(torch, dtype))
    mask = boundary = None
    if mvol is not None:
        if mask_fn is None:
            from oracle.mechanics import attn_mask as mask_fn  # test-side oracle
        m = np.asarray(mask_fn(*mvol, window, mshift), dtype=np.float32)
        mask = torch.from_numpy(m).to(getattr(torch, dtype))
        boundary = (mask.view(mask.shape[0], -1).abs().amax(dim=1) > 0).to(torch.uint8)
        reps = B // mask.shape[0]
        boundary = boundary.repeat(reps)
    return q, k, v, bias, mask, boundary


# Block glue around the attention (norm1 -> pad -> roll + partition ... unpartition
# -> crop).  (name, (B, D, H, W, C), configured window, configured shift, seed);
# the runtime window/shift follow MONAI's clamp (an axis no longer than its
# window uses the axis length and no shift).
BLOCK_CASES = [
    ("b_9x8x10_ws4_ss2_C16", (2, 9, 8, 10, 16), (4, 4, 4), (2, 2, 2), 51),
    ("b_13x10x9_ws7_ss3_C48", (1, 13, 10, 9, 48), (7, 7, 7), (3, 3, 3), 52),
    ("b_6x6x6_clamped_C24", (1, 6, 6, 6, 24), (7, 7, 7), (3, 3, 3), 53),
    ("b_5x9x11_mixed_C32", (2, 5, 9, 11, 32), (7, 7, 7), (3, 3, 3), 54),
    ("b_8x8x8_noshift_C40", (1, 8, 8, 8, 40), (4, 4, 4), (0, 0, 0), 55),
]


def block_inputs(case):
    """x [B,D,H,W,C] fp32, LayerNorm weight/bias fp32 [C], eps."""
    _, shape, _, _, seed = case
    C = shape[-1]
    x = randn(seed, shape, "float32") * 2.0 + 0.5
    weight = 1.0 + 0.25 * randn(seed + 1, (C,), "float32")
    bias = 0.1 * randn(seed + 2, (C,), "float32")
    return x, weight, bias, 1e-5


def block_attn_output(case, windows_shape):
    """The stand-in attention output fed back through the unpartition + crop."""
    return randn(case[-1] + 3, windows_shape, "float32")
