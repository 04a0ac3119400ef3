"""Build libsa_b200.so (the C-ABI library) in-tree with nvcc for sm_100a.

The library links the CUDA runtime statically and depends on no Python or
torch symbol: any host language can dlopen it and bind include/sa_b200.h.
"""
from __future__ import annotations

import os
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
LIB = PKG / "libsa_b200.so"
SOURCES = ["sa_runtime.cu", "kv_append.cu", "gqa_attend.cu", "gqa_decode_mma.cu", "gqa_decode_g8.cu",
           "matmul_nbits.cu", "matmul_nbits_umma.cu",
           "qkv_project.cu", "layer_glue.cu", "gqa_prefill_umma.cu", "lowrank.cu", "rotary.cu"]
HEADERS = ["sa_common.cuh", "sa_internal.h", "sa_append.cuh", "sa_async.cuh", "sa_decode_common.cuh", "sa_tma.cuh",
           "sa_qkv.cuh", "sa_tcgen05.cuh", "sa_gather.cuh"]
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC,-O2", "--expt-relaxed-constexpr",
         "-Xptxas", "-warn-spills"]


def _inputs():
    return [CSRC / s for s in SOURCES] + [CSRC / h for h in HEADERS] + [ROOT / "include" / "sa_b200.h",
                                                                         Path(__file__)]


def needs_build() -> bool:
    if not LIB.exists():
        return True
    t = LIB.stat().st_mtime
    return any(p.stat().st_mtime > t for p in _inputs())


def build(force: bool = False, verbose: bool = False) -> Path:
    if not force and not needs_build():
        return LIB
    from concurrent.futures import ThreadPoolExecutor

    objdir = ROOT / "_build"
    objdir.mkdir(exist_ok=True)
    cmds, objs = [], []
    for s in SOURCES:
        obj = objdir / (Path(s).stem + ".o")
        cmds.append([NVCC, *ARCH, *FLAGS, "-I", str(ROOT / "include"), "-c", str(CSRC / s), "-o", str(obj)])
        objs.append(str(obj))

    def compile_one(cmd):
        if verbose:
            print(" ".join(cmd), flush=True)
        subprocess.check_call(cmd)

    with ThreadPoolExecutor(max_workers=min(len(cmds), os.cpu_count() or 1)) as pool:
        list(pool.map(compile_one, cmds))  # re-raises the first failed compile
    tmp = LIB.with_suffix(f".so.tmp{os.getpid()}")
    cmd = [NVCC, *ARCH, "-shared", "-cudart", "static", "-o", str(tmp), *objs]
    if verbose:
        print(" ".join(cmd), flush=True)
    subprocess.check_call(cmd)
    os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose=True)
    print(LIB)
