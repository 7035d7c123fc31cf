"""Build the native libraries of arm_ai_b200 in-tree.

  libarmai_cuda.so   — the sm_100a CUDA path + C ABI (include/armai.h)
  libarmai_synth.so  — host-only synthetic-model quantiser (csrc/synth.c)

Run ``python -m arm_ai_b200.build`` (or ``__graft_entry__.build()``).
"""
from __future__ import annotations

import glob
import os
import shutil
import subprocess
import sys

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
INCLUDE = os.path.join(ROOT, "include")

NVCC_ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
              "--expt-relaxed-constexpr", "-Xptxas", "-warn-spills"]


def _nvcc() -> str:
    for cand in (shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found")


def _run(cmd: list[str]) -> None:
    print("+", " ".join(cmd), flush=True)
    subprocess.run(cmd, check=True)


def _newer(out: str, deps: list[str]) -> bool:
    if not os.path.exists(out):
        return False
    t = os.path.getmtime(out)
    return all(os.path.getmtime(d) <= t for d in deps)


def build_synth(force: bool = False) -> str:
    out = os.path.join(PKG, "libarmai_synth.so")
    src = os.path.join(CSRC, "synth.c")
    if force or not _newer(out, [src]):
        _run(["gcc", "-O2", "-fPIC", "-shared", "-fopenmp", src, "-o", out, "-lm"])
    return out


def build_cuda(force: bool = False, jobs: int | None = None) -> str:
    out = os.path.join(PKG, "libarmai_cuda.so")
    cu = sorted(glob.glob(os.path.join(CSRC, "*.cu")))
    cpp = sorted(glob.glob(os.path.join(CSRC, "*.cpp")))
    hdrs = glob.glob(os.path.join(CSRC, "*.cuh")) + glob.glob(os.path.join(CSRC, "*.h")) + \
        glob.glob(os.path.join(INCLUDE, "*.h"))
    if not force and _newer(out, cu + cpp + hdrs):
        return out
    nvcc = _nvcc()
    objdir = os.path.join(PKG, "_build")
    os.makedirs(objdir, exist_ok=True)
    objs = []
    procs = []
    for src in cu + cpp:
        obj = os.path.join(objdir, os.path.basename(src) + ".o")
        objs.append(obj)
        if not force and _newer(obj, [src] + hdrs):
            continue
        cmd = [nvcc, *NVCC_ARCH, *NVCC_FLAGS, "-I", INCLUDE, "-I", CSRC, "-c", src, "-o", obj]
        if src.endswith(".cpp"):
            cmd = ["g++", "-O2", "-std=c++17", "-fPIC", "-fvisibility=hidden", "-I", INCLUDE, "-I", CSRC,
                   "-I", "/usr/local/cuda/include", "-c", src, "-o", obj]
        print("+", " ".join(cmd), flush=True)
        procs.append(subprocess.Popen(cmd))
        if len(procs) >= (jobs or os.cpu_count() or 4):
            procs.pop(0).wait()
    rc = [p.wait() for p in procs]
    if any(rc):
        raise RuntimeError("nvcc failed")
    _run([nvcc, *NVCC_ARCH, "-shared", "-o", out, *objs, "-lcudart", "-ldl"])
    return out


def build(force: bool = False) -> None:
    build_synth(force)
    build_cuda(force)


if __name__ == "__main__":
    build(force="--force" in sys.argv)
