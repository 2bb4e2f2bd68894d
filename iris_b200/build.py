"""Builds libiris_b200.so in-tree with nvcc for sm_100a (B200).

`python -m iris_b200.build` compiles the CUDA sources under iris_b200/csrc into
iris_b200/libiris_b200.so (static CUDA runtime, C ABI of include/iris_b200.h).
nvcc cross-compiles without a GPU.
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
LIB = PKG / "libiris_b200.so"
SOURCES = ["q8.cu", "layers.cu", "model.cu", "tp.cu", "step.cu", "tc.cu", "attn_tc.cu"]
HEADERS = ["common.cuh", "detnum.cuh", "sha256.cuh", "q8.cuh", "gemv.cuh", "layers.cuh", "synth.cuh", "tp.cuh", "step.cuh", "tc.cuh", "tcgen05.cuh"]
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
         "--expt-relaxed-constexpr"]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found: the CUDA toolkit is required to build libiris_b200.so")


def stale() -> bool:
    if not LIB.exists():
        return True
    built = LIB.stat().st_mtime
    deps = [CSRC / s for s in SOURCES + HEADERS] + [ROOT / "include" / "iris_b200.h"]
    return any(d.stat().st_mtime > built for d in deps)


def build(force: bool = False, verbose: bool = False) -> Path:
    if not force and not stale():
        return LIB
    objs = []
    build_dir = PKG / "_build"
    build_dir.mkdir(exist_ok=True)
    cmds = []
    for src in SOURCES:
        obj = build_dir / (Path(src).stem + ".o")
        cmds.append([nvcc(), *ARCH, *FLAGS, "-c", str(CSRC / src), "-o", str(obj)])
        objs.append(str(obj))
    procs = [subprocess.Popen(c, stdout=subprocess.PIPE, stderr=subprocess.STDOUT, text=True) for c in cmds]
    for c, p in zip(cmds, procs):
        out, _ = p.communicate()
        if verbose and out:
            print(out)
        if p.returncode:
            raise RuntimeError(f"nvcc failed ({' '.join(c)}):\n{out}")
    tmp = LIB.with_suffix(".so.tmp")
    link = [nvcc(), *ARCH, "-shared", "-o", str(tmp), *objs, "-Xcompiler", "-fPIC"]
    res = subprocess.run(link, stdout=subprocess.PIPE, stderr=subprocess.STDOUT, text=True)
    if res.returncode:
        raise RuntimeError(f"nvcc link failed:\n{res.stdout}")
    os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose=True))
