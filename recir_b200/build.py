"""Compile the CUDA library in-tree: ``recir_b200/libb200_hstu.so`` (sm_100a only).

    python -m recir_b200.build [--force] [--verbose]

nvcc cross-compiles without a GPU.  The shared object sits beside the package so
that it is found (and seen) as an in-tree native library.
"""
from __future__ import annotations

import os
import subprocess
import sys

PKG = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(PKG, "csrc")
LIB = os.path.join(PKG, "libb200_hstu.so")
SOURCES = ["hstu_capi.cu", "hstu_simt.cu", "hstu_tc.cu", "hstu_tc_bwd.cu", "stu_rowwise.cu", "stu_rowwise_bwd.cu", "stu_gemm.cu", "stu_jagged.cu", "stu_embed.cu"]
NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a", "-lineinfo", "-O3", "-std=c++17",
    "-Xcompiler", "-fPIC", "-shared", "--use_fast_math=false",
]


OBJ_DIR = os.path.join(PKG, "_obj")  # per-source objects (git-ignored build cache)


def _headers_mtime() -> float:
    t = 0.0
    inc = os.path.join(os.path.dirname(PKG), "include")
    for d in (inc, CSRC):
        for f in os.listdir(d):
            if f.endswith((".h", ".cuh")):
                t = max(t, os.path.getmtime(os.path.join(d, f)))
    return t


def build(force: bool = False, verbose: bool = False, defines=()) -> str:
    """Compiles every source to an object (in parallel, only what changed) and links the shared
    library.  ``defines`` adds -D macros (e.g. ``B200_HSTU_PROFILING`` for the instrumented kernels);
    a build with defines always recompiles and should be followed by a plain forced build."""
    from concurrent.futures import ThreadPoolExecutor

    nvcc = os.environ.get("NVCC", "nvcc")
    os.makedirs(OBJ_DIR, exist_ok=True)
    hdr_t = _headers_mtime()
    compile_flags = [f for f in NVCC_FLAGS if f not in ("-shared",) and not f.startswith("--use_fast_math")]
    compile_flags += [f"-D{d}" for d in defines]
    if verbose:
        compile_flags += ["-Xptxas", "-v"]
    force = force or bool(defines)
    jobs = []
    for src in SOURCES:
        sp = os.path.join(CSRC, src)
        op = os.path.join(OBJ_DIR, src + ".o")
        if force or not os.path.exists(op) or os.path.getmtime(op) < max(os.path.getmtime(sp), hdr_t):
            jobs.append((sp, op))

    def compile_one(job):
        sp, op = job
        return job, subprocess.run([nvcc, *compile_flags, "-c", "-o", op, sp], capture_output=True, text=True)

    if jobs:
        with ThreadPoolExecutor(max_workers=min(len(jobs), os.cpu_count() or 4)) as ex:
            for (sp, op), r in ex.map(compile_one, jobs):
                if verbose or r.returncode != 0:
                    sys.stderr.write(r.stdout + r.stderr)
                if r.returncode != 0:
                    if os.path.exists(op):
                        os.remove(op)
                    raise RuntimeError(f"nvcc failed compiling {os.path.basename(sp)}")
    objs = [os.path.join(OBJ_DIR, s + ".o") for s in SOURCES]
    if jobs or not os.path.exists(LIB) or os.path.getmtime(LIB) < max(os.path.getmtime(o) for o in objs):
        r = subprocess.run([nvcc, "-gencode", "arch=compute_100a,code=sm_100a", "-shared", "-Xcompiler", "-fPIC",
                            "-o", LIB, *objs], capture_output=True, text=True)
        if r.returncode != 0:
            sys.stderr.write(r.stdout + r.stderr)
            raise RuntimeError("nvcc failed linking libb200_hstu.so")
    return LIB


if __name__ == "__main__":
    defs = tuple(a[2:] for a in sys.argv[1:] if a.startswith("-D"))
    print(build(force="--force" in sys.argv, verbose="--verbose" in sys.argv, defines=defs))
