"""Builds libsulimo_cuda.so (the C-ABI library of the sm_100a kernels) in-tree.

    python -m sulimo_b200.build          # or: python sulimo_b200/build.py

The library is compiled for sm_100a only, with the CUDA runtime linked statically, so the
resulting .so depends on nothing but the NVIDIA driver (libcuda) at run time.
"""
import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
LIB = os.path.join(HERE, "libsulimo_cuda.so")

SOURCES = [
    "capi.cu",
    "q8_0.cu",
    "gemv_q4_0_q8_0.cu",
    "gemv_fast_q4_0_q8_0.cu",
    "gemv_mma_q4_0_q8_0.cu",
    "attn_decode_q8_0.cu",
    "attn_decode_noalloc.cu",
    "attn_decode_mma.cu",
    "matvec_dense.cu",
    "repack_q4_0.cu",
    "gemm_q4_0_tc.cu",
    "gemm_q4_0_pair.cu",
    "shard.cu",
    "forward.cu",
    "attn_prefill_q8_0.cu",
    "attn_prefill_tc.cu",
]

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-lineinfo", "-O3", "-std=c++17",
    "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
    "--expt-relaxed-constexpr",
]


def nvcc_path():
    cand = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not os.path.exists(cand):
        raise RuntimeError("nvcc not found")
    return cand


def _newer(target, deps):
    if not os.path.exists(target):
        return False
    t = os.path.getmtime(target)
    return all(os.path.getmtime(d) <= t for d in deps)


def build(force=False, verbose=False, extra_flags=()):
    deps = [os.path.join(CSRC, s) for s in SOURCES]
    deps += [os.path.join(CSRC, h) for h in os.listdir(CSRC) if h.endswith((".cuh", ".h"))]
    deps.append(os.path.join(HERE, "..", "include", "sulimo_cuda.h"))
    if not force and _newer(LIB, deps):
        return LIB
    objdir = os.path.join(HERE, "_build")
    os.makedirs(objdir, exist_ok=True)
    nvcc = nvcc_path()
    headers = [d for d in deps if not d.endswith(".cu")]
    jobs = []
    for s in SOURCES:
        src = os.path.join(CSRC, s)
        obj = os.path.join(objdir, s.replace(".cu", ".o"))
        # an object is reused when it is newer than its source and every header (and the flags
        # did not change: extra flags force a rebuild)
        fresh = not force and not extra_flags and _newer(obj, [src] + headers)
        jobs.append(([nvcc, *NVCC_FLAGS, *extra_flags, "-c", src, "-o", obj], obj, fresh))
    from concurrent.futures import ThreadPoolExecutor

    def run(job):
        if job[2]:
            return job[1]
        if verbose:
            print(" ".join(job[0]), flush=True)
        subprocess.run(job[0], check=True)
        return job[1]

    with ThreadPoolExecutor(max_workers=min(len(jobs), os.cpu_count() or 1)) as ex:
        objs = list(ex.map(run, jobs))
    tmp = LIB + ".tmp"
    cmd = [nvcc, "-gencode", "arch=compute_100a,code=sm_100a", "-shared", "-o", tmp, *objs,
           "-Xcompiler", "-fPIC", "-cudart", "static"]
    if verbose:
        print(" ".join(cmd))
    subprocess.run(cmd, check=True)
    os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose=True,
          extra_flags=["-Xptxas", "-v"] if "--ptxas-v" in sys.argv else ())
    print(LIB)
