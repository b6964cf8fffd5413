"""Build the reference's own GPU kernels for a same-box comparison on a B200.

Run in a container that has the reference checkout (its sources are read where
they lie, never copied):

    python baseline/build_reference.py [--reference PATH]

Outputs go to ``baseline/_ref/`` (git-ignored; it travels to the GPU box with
the rest of the working tree, the reference checkout does not):

* ``crumpet_ref_ops.so`` -- the reference's CUDA extension: ``cuda/shift_partition_3d.cu``,
  ``cuda/unshift_unpartition_3d.cu``, ``cuda/attn_mask_3d.cu`` and
  ``torch-ext/torch_binding.cpp``, compiled as the reference's JIT build does
  (torch-ext/crumpet/_jit_ops.py:15-44: ``-O3 -lineinfo``, ``-DCUDA_KERNEL``, the
  ``torch-ext`` include path) for ``CRUMPET_CUDA_ARCH_LIST=10.0`` (sm_100), but under
  the op namespace ``crumpet_ref_ops`` so it can be loaded next to this repository's
  ``crumpet_ops``.  nvcc and g++ are driven directly; the reference's build system
  (torch.utils.cpp_extension.load / kernel-builder) is not run.
* ``ref_swin_attention_n{N}.cubin`` + ``.json`` -- the reference's Triton kernel
  ``_fused_swin_attention_kernel`` (torch-ext/crumpet/fused_attention.py:48-146),
  compiled ahead of time by ``triton.compile`` for target cuda:100 with the launch
  parameters its launcher uses on a B200 (fused_attention.py:203-226: 4 warps and
  Triton's default 3 stages, BLOCK_M = min(64, next_pow2(N)), BLOCK_N = min(32,
  next_pow2(N)), head_dim 16, float16) and the argument specialisation Triton's JIT
  gives contiguous tensors (16-byte aligned pointers, strides divisible by 16 marked
  as such, unit strides as constants).  The JSON records the kernel name, shared
  memory, warps and the runtime parameter order for a driver-API launch.

Nothing here is part of the crumpet_b200 product: bench.py loads these files, when
present, only to time the reference's kernels beside this repository's.
"""

from __future__ import annotations

import argparse
import importlib.util
import json
import os
import shutil
import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
OUT = HERE / "_ref"
EXT_NAME = "crumpet_ref_ops"
CUDA_SOURCES = ("shift_partition_3d.cu", "unshift_unpartition_3d.cu", "attn_mask_3d.cu")
ATTENTION_N = (343, 216)  # stage 0-2 windows (7^3) and the 6^3 stage


def _cuda_home() -> Path:
    for cand in (os.environ.get("CUDA_HOME"), "/usr/local/cuda"):
        if cand and (Path(cand) / "bin" / "nvcc").exists():
            return Path(cand)
    return Path(shutil.which("nvcc")).resolve().parent.parent


def _run(cmd, what):
    proc = subprocess.run(cmd, stdout=subprocess.PIPE, stderr=subprocess.STDOUT, text=True)
    if proc.returncode != 0:
        raise RuntimeError(f"{what} failed:\n{' '.join(map(str, cmd))}\n{proc.stdout[-4000:]}")


def build_cuda_extension(ref: Path) -> Path:
    import torch
    import torch.utils.cpp_extension as ce

    cuda = _cuda_home()
    work = OUT / "obj"
    work.mkdir(parents=True, exist_ok=True)
    abi = int(torch._C._GLIBCXX_USE_CXX11_ABI)
    defs = [f"-D_GLIBCXX_USE_CXX11_ABI={abi}", "-DTORCH_API_INCLUDE_EXTENSION_H",
            f"-DTORCH_EXTENSION_NAME={EXT_NAME}", "-DCUDA_KERNEL"]
    incs = []
    for i in [*ce.include_paths(), str(cuda / "include")]:
        incs += ["-isystem", i]
    incs += ["-I", str(ref / "torch-ext"), "-I", str(ref / "cuda")]
    # torch's own nvcc defaults for extensions, then the reference's flags
    nvcc_flags = ["-std=c++17", "-Xcompiler", "-fPIC", "--expt-relaxed-constexpr",
                  "-D__CUDA_NO_HALF_OPERATORS__", "-D__CUDA_NO_HALF_CONVERSIONS__",
                  "-D__CUDA_NO_BFLOAT16_CONVERSIONS__", "-D__CUDA_NO_HALF2_OPERATORS__",
                  "-gencode", "arch=compute_100,code=sm_100", "-O3", "-lineinfo"]
    procs, objs = [], []
    for src in CUDA_SOURCES:
        obj = work / (Path(src).stem + ".o")
        objs.append(obj)
        cmd = [str(cuda / "bin" / "nvcc"), *nvcc_flags, *defs, *incs, "-c", str(ref / "cuda" / src),
               "-o", str(obj)]
        procs.append((cmd, subprocess.Popen(cmd, stdout=subprocess.PIPE, stderr=subprocess.STDOUT,
                                            text=True)))
    binding = work / "torch_binding.o"
    _run(["g++", "-O3", "-std=c++17", "-fPIC", *defs, *incs, "-c",
          str(ref / "torch-ext" / "torch_binding.cpp"), "-o", str(binding)], "g++ torch_binding.cpp")
    for cmd, proc in procs:
        out, _ = proc.communicate()
        if proc.returncode != 0:
            raise RuntimeError(f"nvcc failed:\n{' '.join(cmd)}\n{out[-4000:]}")
    target = OUT / f"{EXT_NAME}.so"
    cmd = ["g++", "-shared", "-o", str(target), str(binding), *map(str, objs)]
    for d in [*ce.library_paths(), str(cuda / "lib64")]:
        cmd += ["-L", d]
    cmd += ["-lc10", "-lc10_cuda", "-ltorch", "-ltorch_cpu", "-ltorch_cuda", "-lcudart"]
    _run(cmd, f"link {target.name}")
    shutil.rmtree(work)
    return target


def build_triton_attention(ref: Path, n: int) -> Path:
    import triton
    from triton.backends.compiler import GPUTarget
    from triton.compiler import ASTSource, make_backend

    path = ref / "torch-ext" / "crumpet" / "fused_attention.py"
    sys.dont_write_bytecode = True
    spec = importlib.util.spec_from_file_location("reference_fused_attention", path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    kernel = mod._fused_swin_attention_kernel
    names = list(kernel.arg_names)
    p2 = 1 << (n - 1).bit_length()
    constants = {"N": n, "D": 16, "BLOCK_M": min(64, p2), "BLOCK_N": min(32, p2)}
    for s in ("stride_qd", "stride_kd", "stride_vd", "stride_bn", "stride_mn", "stride_od"):
        constants[s] = 1  # unit strides of contiguous tensors
    signature = {}
    for name in names:
        if name in constants:
            signature[name] = "constexpr"
        elif name == "BOUNDARY":
            signature[name] = "*u8"
        elif name in ("Q", "K", "V", "BIAS", "MASK", "OUT"):
            signature[name] = "*fp16"
        elif name == "SCALE":
            signature[name] = "fp32"
        else:
            signature[name] = "i32"
    # divisibility by 16 holds for every pointer and for the q/k/v/out strides of
    # contiguous [B, H, N, 16] tensors (N*16, 16); bias/mask strides (N*N, N) do not
    div16 = [nm for nm in names if signature[nm].startswith("*")]
    div16 += [f"stride_{t}{a}" for t in "qkvo" for a in "bhn"]
    attrs = {(names.index(nm),): [["tt.divisibility", 16]] for nm in div16}
    src = ASTSource(fn=kernel, signature=signature, attrs=attrs,
                    constexprs={(names.index(k),): v for k, v in constants.items()})
    target = GPUTarget("cuda", 100, 32)
    backend = make_backend(target)
    options = backend.parse_options({"num_warps": 4, "num_stages": 3})
    compiled = triton.compile(src, target=target, options=options.__dict__)
    md = compiled.metadata
    if getattr(md, "global_scratch_size", 0) or getattr(md, "profile_scratch_size", 0):
        raise RuntimeError("the compiled reference kernel needs scratch buffers")
    stem = OUT / f"ref_swin_attention_n{n}"
    stem.with_suffix(".cubin").write_bytes(compiled.asm["cubin"])
    runtime_args = [nm for nm in names if signature[nm] != "constexpr"]
    meta = {
        "kernel": md.name, "shared_bytes": md.shared, "num_warps": md.num_warps,
        "threads": md.num_warps * 32, "constants": constants,
        "runtime_args": [{"name": nm, "type": signature[nm]} for nm in runtime_args],
        "trailing_null_pointers": 2,  # Triton's global / profile scratch parameters
        "grid": "(ceil(N / BLOCK_M), H, B)",
        "source": "torch-ext/crumpet/fused_attention.py:48-146 (launcher :149-226)",
        "triton": triton.__version__,
    }
    stem.with_suffix(".json").write_text(json.dumps(meta, indent=1))
    return stem.with_suffix(".cubin")


def build(ref: Path) -> list[Path]:
    if not (ref / "cuda" / CUDA_SOURCES[0]).exists():
        raise FileNotFoundError(f"no reference checkout at {ref}")
    OUT.mkdir(parents=True, exist_ok=True)
    built = [build_cuda_extension(ref)]
    built += [build_triton_attention(ref, n) for n in ATTENTION_N]
    return built


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("CRUMPET_REFERENCE", "/root/reference"))
    args = ap.parse_args()
    for p in build(Path(args.reference)):
        print(p)


if __name__ == "__main__":
    main()
