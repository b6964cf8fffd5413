"""Generate the golden fixtures under tests/golden/ from the REFERENCE code.

Run in a container where the reference checkout exists (it is not needed by
the tests themselves):

    TRITON_INTERPRET=1 python tests/golden/make_golden.py /path/to/crumpet

* Mechanics: SHA-256 digests of the outputs of the reference's pure-PyTorch
  functions (torch-ext/crumpet/reference.py: unfused_shift_partition_3d_reference,
  unfused_unshift_unpartition_3d_reference, compute_attn_mask_3d_reference) on
  the seeded inputs of tests/golden/inputs.py.
* Block glue: the reference's patched ``forward_part1``
  (torch-ext/crumpet/monai_patch.py:72-114) run on the CPU on a stand-in block
  (LayerNorm norm1, configured window/shift, an ``attn`` that records the
  windows it is given and returns a seeded tensor): the windows after
  norm1 -> pad -> roll + partition, and the cropped output.
* Attention: outputs of the reference Triton kernel
  (torch-ext/crumpet/fused_attention.py:48-146), launched exactly as its
  launcher does (:149-226), executed by the Triton CPU interpreter.
"""

from __future__ import annotations

import hashlib
import json
import os
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE))
sys.path.insert(0, str(HERE.parent.parent))

if os.environ.get("TRITON_INTERPRET") != "1":
    raise SystemExit("set TRITON_INTERPRET=1 so the reference Triton kernel runs on the CPU")


def sha(t) -> str:
    return hashlib.sha256(t.contiguous().view(-1).view(dtype=__import__("torch").uint8).numpy().tobytes()).hexdigest()


def main(ref_root: str) -> None:
    sys.path.insert(0, str(Path(ref_root) / "torch-ext"))
    import numpy as np
    import torch
    import triton

    from crumpet import reference as R
    from crumpet import fused_attention as FA
    import inputs as I

    manifest = {"mechanics": {}, "mask": {}, "attention": {}}
    for case in I.MECHANICS_CASES:
        name, shape, ws, ss, dtype, seed = case
        x = I.mechanics_input(case)
        B, D, H, W, C = shape
        win = R.unfused_shift_partition_3d_reference(x, ws, ss)
        back = R.unfused_unshift_unpartition_3d_reference(win, B, D, H, W, C, ws, ss)
        assert torch.equal(back, x)
        manifest["mechanics"][name] = {
            "input_sha256": sha(x),
            "partition_sha256": sha(win),
            "partition_shape": list(win.shape),
        }
        print("mechanics", name, flush=True)
    for name, dims, ws, ss, dtype in I.MASK_CASES:
        m = R.compute_attn_mask_3d_reference(*dims, ws, ss, getattr(torch, dtype), "cpu")
        manifest["mask"][name] = {"sha256": sha(m), "shape": list(m.shape),
                                  "neg_count": int((m != 0).sum())}
        print("mask", name, flush=True)

    arrays = {}
    for case in I.ATTENTION_CASES:
        name = case[0]
        mask_fn = lambda D, H, W, w, s: R.compute_attn_mask_3d_reference(
            D, H, W, w, s, torch.float32, "cpu").numpy()
        q, k, v, bias, mask, boundary = I.attention_inputs(case, mask_fn=mask_fn)
        B, Hh, N, Dh = q.shape
        scale = 1.0 / (Dh ** 0.5)
        # Launch the reference kernel the way fused_swin_attention does
        # (fused_attention.py:177-225), minus its is_cuda assertion.
        if mask is None:
            mask_t = torch.zeros((1, N, N), dtype=q.dtype)
            bnd = torch.zeros((B,), dtype=torch.uint8)
            mstr = (0, mask_t.stride(1), mask_t.stride(2))
        else:
            mask_t = mask.repeat(B // mask.shape[0], 1, 1) if mask.shape[0] != B else mask
            bnd = boundary
            mstr = (mask_t.stride(0), mask_t.stride(1), mask_t.stride(2))
        out = torch.empty_like(q)
        bn = min(32, triton.next_power_of_2(N))
        bm = min(64, triton.next_power_of_2(N))
        grid = (triton.cdiv(N, bm), Hh, B)
        FA._fused_swin_attention_kernel[grid](
            q, k, v, bias, mask_t, bnd, out, scale,
            *q.stride(), *k.stride(), *v.stride(), *bias.stride(), *mstr, *out.stride(),
            N=N, D=Dh, BLOCK_M=bm, BLOCK_N=bn)
        arrays[name] = out.float().numpy().astype(np.float32)
        manifest["attention"][name] = {"shape": list(out.shape), "dtype": str(q.dtype)}
        print("attention", name, flush=True)
    np.savez_compressed(HERE / "attention_ref_out.npz", **arrays)

    from crumpet import monai_patch as MP
    import crumpet_b200.swin_unetr as swin  # provides get_window_size (MONAI rule)

    class _Attn(torch.nn.Module):
        def __init__(self, case):
            super().__init__()
            self.case = case

        def forward(self, windows, mask=None):
            self.windows = windows.clone()
            return I.block_attn_output(self.case, windows.shape)

    class _Block(torch.nn.Module):
        def __init__(self, case):
            super().__init__()
            _, shape, window, shift, _ = case
            x, w, b, eps = I.block_inputs(case)
            self.norm1 = torch.nn.LayerNorm(shape[-1], eps=eps)
            with torch.no_grad():
                self.norm1.weight.copy_(w)
                self.norm1.bias.copy_(b)
            self.window_size, self.shift_size = window, shift
            self.attn = _Attn(case)

    part1 = MP._patched_forward_part1(lambda *a: None, swin)
    block_arrays = {}
    manifest["block"] = {}
    for case in I.BLOCK_CASES:
        name = case[0]
        blk = _Block(case)
        x = I.block_inputs(case)[0]
        with torch.no_grad():
            out = part1(blk, x, None)
        block_arrays[name + ".windows"] = blk.attn.windows.numpy()
        block_arrays[name + ".out"] = out.numpy()
        manifest["block"][name] = {"windows_shape": list(blk.attn.windows.shape),
                                   "out_sha256": sha(out)}
        print("block", name, flush=True)
    np.savez_compressed(HERE / "block_ref.npz", **block_arrays)
    (HERE / "manifest.json").write_text(json.dumps(manifest, indent=1, sort_keys=True) + "\n")


if __name__ == "__main__":
    if len(sys.argv) != 2:
        raise SystemExit("usage: TRITON_INTERPRET=1 python tests/golden/make_golden.py <reference checkout>")
    main(sys.argv[1])
