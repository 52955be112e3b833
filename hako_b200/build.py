"""Build recipe for the native parts of hako_b200 (run in-tree).

    python -m hako_b200.build          # libhakm_cuda.so, libhakm_tok.so, libhakm_synth.so

libhakm_cuda.so is compiled by nvcc for sm_100a only (no PTX fallback, no
other architectures) with the CUDA runtime linked statically, so the library
is self-contained next to the package. libhakm_tok.so (the Qwen2 tokenizer,
include/hakm_tok.h) is plain C compiled by gcc. Outputs land in
hako_b200/_lib/.
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
LIB = os.path.join(HERE, "_lib")
ROOT = os.path.dirname(HERE)

CUDA_SOURCES = ["csrc/hakm_stream.cu", "csrc/hakm_step.cu", "csrc/hakm_kernels.cu", "csrc/hakm_batch.cu",
                "csrc/hakm_mma.cu", "csrc/hakm_prefill.cu", "csrc/hakm_rows.cu", "csrc/hakm_sample.cu",
                "csrc/hakm_runtime.cu"]
CUDA_HEADERS = ["csrc/hakm_internal.h", "csrc/hakm_device.cuh", "csrc/hakm_exact.cuh", "csrc/hakm_gemv.cuh",
                "csrc/hakm_attn.cuh", "csrc/hakm_ll.cuh", "csrc/hakm_tmap.h", "../include/hakm_cuda.h"]
# host tables that carry glibc's vector libm roundings: gcc with AVX2 + FMA
# (the vector entry points' calling convention), no contraction
HOST_C = "csrc/hakm_hostmath.c"
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def _nvcc() -> str:
    for cand in (shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found")


def _stale(out: str, deps: list[str]) -> bool:
    if not os.path.exists(out):
        return True
    t = os.path.getmtime(out)
    return any(os.path.getmtime(d) > t for d in deps)


def _run(cmd: list[str]) -> None:
    r = subprocess.run(cmd, cwd=HERE, capture_output=True, text=True)
    if r.returncode != 0:
        sys.stderr.write(r.stdout + r.stderr)
        raise RuntimeError("build failed: " + " ".join(cmd))


def build_cuda(force: bool = False, verbose_ptxas: bool = False) -> str:
    out = os.path.join(LIB, "libhakm_cuda.so")
    deps = [os.path.join(HERE, s) for s in CUDA_SOURCES + CUDA_HEADERS + [HOST_C]]
    if force or _stale(out, deps):
        os.makedirs(LIB, exist_ok=True)
        host_o = os.path.join(LIB, "hakm_hostmath.o")
        _run(["gcc", "-O2", "-std=c11", "-Wall", "-fPIC", "-mavx2", "-mfma", "-ffp-contract=off", "-c",
              "-o", host_o, HOST_C])
        cmd = [_nvcc(), *ARCH, "-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC,-O2",
               "-shared", "-cudart", "static", "-o", out, *CUDA_SOURCES, host_o, "-lmvec", "-lm"]
        if verbose_ptxas:
            cmd.insert(1, "-Xptxas=-v")
        _run(cmd)
    return out


def build_synth(force: bool = False) -> str:
    out = os.path.join(LIB, "libhakm_synth.so")
    exe = os.path.join(LIB, "hakm_synth")
    src = os.path.join(HERE, "synth", "mlf2_synth.c")
    if force or _stale(out, [src]):
        os.makedirs(LIB, exist_ok=True)
        _run(["gcc", "-O2", "-std=c11", "-Wall", "-fPIC", "-shared", "-o", out, src, "-lm", "-lpthread"])
    if force or _stale(exe, [src]):
        os.makedirs(LIB, exist_ok=True)
        _run(["gcc", "-O2", "-std=gnu11", "-Wall", "-DSYNTH_MAIN", "-o", exe, src, "-lm", "-lpthread"])
    return out


TOK_SOURCES = ["host/hakm_bpe.c", "host/hakm_pretok.c"]
TOK_HEADERS = ["host/hakm_unicode_tables.h", "../include/hakm_tok.h"]


def build_tok(force: bool = False) -> str:
    out = os.path.join(LIB, "libhakm_tok.so")
    deps = [os.path.join(HERE, s) for s in TOK_SOURCES + TOK_HEADERS]
    if force or _stale(out, deps):
        os.makedirs(LIB, exist_ok=True)
        _run(["gcc", "-O2", "-std=c11", "-Wall", "-Wextra", "-fPIC", "-shared", "-I", os.path.join(ROOT, "include"),
              "-o", out, *TOK_SOURCES])
    return out


def build_all(force: bool = False) -> None:
    build_synth(force)
    build_tok(force)
    build_cuda(force)


if __name__ == "__main__":
    build_all(force="--force" in sys.argv)
    print("built", os.listdir(LIB))
