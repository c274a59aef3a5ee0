"""Build the native pieces in-tree (sm_100a only):

* ``libb2s.so``  -- CUDA kernels + the C-ABI of ``include/b2s_sampler.h`` (nvcc, static cudart, no torch);
* ``_build/b2s_torch_ops.so`` -- the ``torch.ops.minicpmo_sampler`` op layer over that C-ABI.

``python build.py`` from this directory, or ``__graft_entry__.build()`` from the repository root.
Compilation needs nvcc but no GPU.
"""

from __future__ import annotations

import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
INCLUDE = ROOT / "include"
BUILD = PKG / "_build"
LIB = PKG / "libb2s.so"
OPS = BUILD / "b2s_torch_ops.so"
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
CU_SOURCES = [CSRC / "b2s_sampler.cu", CSRC / "b2s_resident.cu", CSRC / "b2s_short.cu", CSRC / "b2s_shard.cu",
              CSRC / "b2s_lmhead.cu"]
CU_HEADERS = [CSRC / "b2s_device.cuh", CSRC / "b2s_list.cuh", CSRC / "b2s_row.cuh", CSRC / "b2s_rowpaths.cuh",
              CSRC / "b2s_head.cuh", INCLUDE / "b2s_sampler.h"]


def _nvcc() -> str:
    cuda_home = os.environ.get("CUDA_HOME", "/usr/local/cuda")
    cand = Path(cuda_home) / "bin" / "nvcc"
    return str(cand) if cand.exists() else (shutil.which("nvcc") or "nvcc")


def _stale(out: Path, deps) -> bool:
    if not out.exists():
        return True
    t = out.stat().st_mtime
    return any(Path(d).stat().st_mtime > t for d in deps)


def build_lib(force: bool = False, verbose: bool = False) -> Path:
    srcs = [s for s in CU_SOURCES if s.exists()]
    if not force and not _stale(LIB, srcs + CU_HEADERS):
        return LIB
    BUILD.mkdir(exist_ok=True)
    objs = []
    for s in srcs:
        o = BUILD / (s.stem + ".o")
        cmd = [_nvcc(), *ARCH, "-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "-Xptxas", "-v",
               f"-I{INCLUDE}", "-c", str(s), "-o", str(o)]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"nvcc failed for {s.name}:\n{r.stderr}")
        if verbose:
            print(r.stderr)
        (BUILD / (s.stem + ".ptxas.txt")).write_text(r.stderr)
        objs.append(str(o))
    tmp = LIB.with_suffix(".so.tmp")
    cmd = [_nvcc(), *ARCH, "-shared", "-cudart", "static", "-Xlinker", "-soname=libb2s.so", "-o", str(tmp), *objs]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc link failed:\n{r.stderr}")
    os.replace(tmp, LIB)
    return LIB


def build_ops(force: bool = False, verbose: bool = False) -> Path:
    src = CSRC / "torch_ops.cpp"
    if not force and not _stale(OPS, [src, INCLUDE / "b2s_sampler.h", LIB]):
        return OPS
    import ctypes

    import torch.utils.cpp_extension as ce

    BUILD.mkdir(exist_ok=True)
    ctypes.CDLL(str(LIB), mode=ctypes.RTLD_GLOBAL)  # resolves the op library's libb2s.so dependency (soname)
    ce.load(name="b2s_torch_ops", sources=[str(src)], extra_include_paths=[str(INCLUDE)],
            extra_cflags=["-O2", "-std=c++17"], extra_ldflags=[f"-L{PKG}", "-lb2s"],
            build_directory=str(BUILD), with_cuda=True, is_python_module=False, verbose=verbose)
    return OPS


def build(force: bool = False, verbose: bool = False) -> None:
    build_lib(force=force, verbose=verbose)
    build_ops(force=force, verbose=verbose)


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose="-v" in sys.argv)
    print("built", LIB, OPS)
