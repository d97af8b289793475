"""Builds libdeepunity_cuda.so in place with nvcc for sm_100a.

    python -m deepunity_b200.build          # or deepunity_b200.build.build()

The library has no torch dependency: it links only the CUDA runtime; NCCL is
opened at run time when tensor parallelism is requested.
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
LIB = os.path.join(HERE, "libdeepunity_cuda.so")
SOURCES = ["capi.cu", "gemv.cu", "gemm.cu", "tgemv.cu", "attention.cu", "elementwise.cu", "model.cu", "noalloc.cu",
           "decode_step.cu", "tp_comm.cu", "sampler.cu", "snapshot.cu"]
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc() -> str:
    for c in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", shutil.which("nvcc")):
        if c and os.path.exists(c):
            return c
    raise RuntimeError("nvcc not found")


def _stale() -> bool:
    if not os.path.exists(LIB):
        return True
    t = os.path.getmtime(LIB)
    deps = [os.path.join(CSRC, f) for f in os.listdir(CSRC)]
    deps.append(os.path.join(HERE, "..", "include", "deepunity_cuda.h"))
    return any(os.path.getmtime(d) > t for d in deps if os.path.exists(d))


def build(force: bool = False, verbose: bool = False) -> str:
    if not force and not _stale():
        return LIB
    objdir = os.path.join(HERE, "_build")
    os.makedirs(objdir, exist_ok=True)
    objs = []
    flags = ARCH + ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC,-fvisibility=hidden",
                    "--expt-relaxed-constexpr", "-ccbin", "g++"]
    procs = []
    for src in SOURCES:
        obj = os.path.join(objdir, src.replace(".cu", ".o"))
        objs.append(obj)
        cmd = [nvcc(), "-c", os.path.join(CSRC, src), "-o", obj] + flags
        if verbose:
            cmd.append("-Xptxas=-v")
        procs.append((src, subprocess.Popen(cmd, stdout=subprocess.PIPE, stderr=subprocess.STDOUT, text=True)))
    errors = []
    for src, p in procs:
        out, _ = p.communicate()
        if p.returncode != 0 or verbose:
            (errors if p.returncode != 0 else [sys.stderr]).__class__  # noqa
            if p.returncode != 0:
                errors.append(f"--- {src}\n{out}")
            else:
                sys.stderr.write(out)
    if errors:
        raise RuntimeError("nvcc failed:\n" + "\n".join(errors))
    tmp = LIB + ".tmp"
    subprocess.run([nvcc(), "-shared", "-o", tmp] + objs + ARCH + ["-ccbin", "g++", "-ldl", "-lcudart"],
                   check=True)
    os.replace(tmp, LIB)
    return LIB


STAMPS_LIB = os.path.join(HERE, "libdeepunity_cuda_stamps.so")


def build_stamps() -> str:
    """The timing build: the library with gemv.cu compiled under DU_GEMV_STAMPS
    (per-CTA phase stamps of every decode GEMV launch, gemv_stamps.cuh), for
    ``bench.py --gemv-phases``.  The other objects are those of the library."""
    build()
    objdir = os.path.join(HERE, "_build")
    flags = ARCH + ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC,-fvisibility=hidden",
                    "--expt-relaxed-constexpr", "-ccbin", "g++", "-DDU_GEMV_STAMPS"]
    obj = os.path.join(objdir, "gemv_stamps.o")
    subprocess.run([nvcc(), "-c", os.path.join(CSRC, "gemv.cu"), "-o", obj] + flags, check=True)
    objs = [obj] + [os.path.join(objdir, s.replace(".cu", ".o")) for s in SOURCES if s != "gemv.cu"]
    tmp = STAMPS_LIB + ".tmp"
    subprocess.run([nvcc(), "-shared", "-o", tmp] + objs + ARCH + ["-ccbin", "g++", "-ldl", "-lcudart"], check=True)
    os.replace(tmp, STAMPS_LIB)
    return STAMPS_LIB


if __name__ == "__main__":
    if "--stamps" in sys.argv:
        print(build_stamps())
    else:
        build(force="--force" in sys.argv, verbose="-v" in sys.argv)
        print(LIB)
