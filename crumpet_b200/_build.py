"""In-tree build of the crumpet_b200 native libraries.

Two shared objects are produced next to this file:

* ``libcrumpet_b200.so`` -- every CUDA kernel plus the C ABI declared in
  ``include/crumpet_b200.h``, compiled by nvcc for sm_100a only.  It has no
  PyTorch dependency (the CUDA runtime is linked statically).
* ``_C.so`` -- the ``crumpet_ops`` torch dispatcher registration
  (``csrc/torch_binding.cpp``), a thin adapter that calls the C ABI.

``build()`` is incremental (sources newer than the target trigger a rebuild)
and needs no GPU: nvcc cross-compiles for sm_100a.
"""

from __future__ import annotations

import os
import shutil
import subprocess
from pathlib import Path

PKG = Path(__file__).resolve().parent
REPO = PKG.parent
CSRC = PKG / "csrc"
INCLUDE = REPO / "include"
LIB = PKG / "libcrumpet_b200.so"
EXT = PKG / "_C.so"

CUDA_SOURCES = ["capi.cu", "partition.cu", "mask.cu", "attention.cu", "attention_simt.cu",
                "norm_partition.cu", "sliding_window.cu", "proj_norm.cu", "linear.cu"]
CUDA_HEADERS = ["common.cuh", "sm100.cuh", "kernels.h"]
NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-lineinfo", "-O3", "-std=c++17",
    "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
    "--cudart", "static",
]


def _cuda_home() -> Path:
    for cand in (os.environ.get("CUDA_HOME"), "/usr/local/cuda"):
        if cand and (Path(cand) / "bin" / "nvcc").exists():
            return Path(cand)
    nvcc = shutil.which("nvcc")
    if nvcc:
        return Path(nvcc).resolve().parent.parent
    raise RuntimeError("nvcc not found: set CUDA_HOME")


def _stale(target: Path, deps: list[Path]) -> bool:
    if not target.exists():
        return True
    t = target.stat().st_mtime
    return any(d.stat().st_mtime > t for d in deps)


def _run(cmd: list[str], what: str) -> None:
    proc = subprocess.run(cmd, stdout=subprocess.PIPE, stderr=subprocess.STDOUT, text=True)
    if proc.returncode != 0:
        raise RuntimeError(f"{what} failed ({proc.returncode}):\n{' '.join(cmd)}\n{proc.stdout}")


def build_library(force: bool = False) -> Path:
    """Compile the CUDA kernels and the C ABI into libcrumpet_b200.so."""
    deps = [CSRC / s for s in CUDA_SOURCES + CUDA_HEADERS] + [INCLUDE / "crumpet_b200.h"]
    if not force and not _stale(LIB, deps):
        return LIB
    nvcc = str(_cuda_home() / "bin" / "nvcc")
    objs = []
    build_dir = PKG / "_build"
    build_dir.mkdir(exist_ok=True)
    procs = []
    for src in CUDA_SOURCES:
        obj = build_dir / (Path(src).stem + ".o")
        objs.append(obj)
        cmd = [nvcc, *NVCC_FLAGS, "-I", str(INCLUDE), "-c", str(CSRC / src), "-o", str(obj)]
        procs.append((cmd, subprocess.Popen(cmd, stdout=subprocess.PIPE,
                                            stderr=subprocess.STDOUT, text=True)))
    for cmd, proc in procs:
        out, _ = proc.communicate()
        if proc.returncode != 0:
            raise RuntimeError(f"nvcc failed:\n{' '.join(cmd)}\n{out}")
    tmp = LIB.with_suffix(".so.tmp")
    _run([nvcc, "-shared", "-gencode", "arch=compute_100a,code=sm_100a", "--cudart", "static",
          *map(str, objs), "-o", str(tmp)], "link libcrumpet_b200.so")
    os.replace(tmp, LIB)
    return LIB


def build_torch_binding(force: bool = False) -> Path:
    """Compile the crumpet_ops dispatcher registration into _C.so."""
    deps = [CSRC / "torch_binding.cpp", INCLUDE / "crumpet_b200.h", LIB]
    if not force and not _stale(EXT, deps):
        return EXT
    import torch
    import torch.utils.cpp_extension as ce

    cuda_home = _cuda_home()
    incs = [*ce.include_paths(), str(cuda_home / "include"), str(INCLUDE)]
    libdirs = [*ce.library_paths(), str(cuda_home / "lib64")]
    abi = int(torch._C._GLIBCXX_USE_CXX11_ABI)
    cmd = ["g++", "-O2", "-std=c++17", "-fPIC", "-shared", f"-D_GLIBCXX_USE_CXX11_ABI={abi}",
           "-DTORCH_API_INCLUDE_EXTENSION_H"]
    for i in incs:
        cmd += ["-isystem", i]
    cmd += [str(CSRC / "torch_binding.cpp"), "-o", str(EXT.with_suffix(".so.tmp"))]
    for d in libdirs:
        cmd += ["-L", d]
    cmd += ["-L", str(PKG), "-lcrumpet_b200", "-lc10", "-lc10_cuda", "-ltorch", "-ltorch_cpu",
            "-ltorch_cuda", "-Wl,-rpath,$ORIGIN"]
    _run(cmd, "build _C.so")
    os.replace(EXT.with_suffix(".so.tmp"), EXT)
    return EXT


def build(force: bool = False) -> None:
    build_library(force)
    build_torch_binding(force)
    # a package imported before the libraries existed picks them up now
    from . import _ops, _register_fake_impls

    _ops.reload()
    _register_fake_impls()


if __name__ == "__main__":
    import sys

    build(force="--force" in sys.argv)
    print(LIB)
    print(EXT)
