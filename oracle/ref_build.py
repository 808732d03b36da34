"""Builds oracle/_ref/libsulimo_ref_ocl.so: the reference's own OpenCL C kernels
(kernels/gemm_q4_0.cl, kernels/prefill.cl), compiled unchanged for the host CPU through the
shim oracle/ref_ocl_shim.cpp.

TEST INFRASTRUCTURE ONLY: the library pins the C restatement (sulimo_oracle.c) to values that
the reference's code produces.  The kernel sources are read from the reference checkout where
they lie (SULIMO_REFERENCE_DIR, else the default below) and never copied into this repository;
the only output is the shared library under oracle/_ref/ (git-ignored, carried to GPU machines
with the rest of the working tree, where the reference checkout is absent and the prebuilt
library is used as is).

Flags: strict IEEE order (-ffp-contract=off, no fast-math), like the C restatement.
"""
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
OUT_DIR = os.path.join(HERE, "_ref")
LIB = os.path.join(OUT_DIR, "libsulimo_ref_ocl.so")
SHIM = os.path.join(HERE, "ref_ocl_shim.cpp")
HDR = os.path.join(HERE, "sulimo_oracle.h")
DEFAULT_REFERENCE_DIR = "/root/reference"
KERNELS = ("gemm_q4_0.cl", "prefill.cl")
CXXFLAGS = ["-O2", "-std=gnu++20", "-ffp-contract=off", "-fno-fast-math", "-fno-strict-aliasing",
            "-fPIC", "-shared", "-pthread", "-Wall", "-Wno-unknown-pragmas", "-Wno-literal-suffix",
            "-Wno-unused-function", "-Wno-unused-label"]


def reference_kernels_dir():
    root = os.environ.get("SULIMO_REFERENCE_DIR", DEFAULT_REFERENCE_DIR)
    d = os.path.join(root, "kernels")
    if all(os.path.isfile(os.path.join(d, k)) for k in KERNELS):
        return d
    return None


def available():
    """True when the library is built (or can be built from a reference checkout)."""
    return os.path.exists(LIB) or reference_kernels_dir() is not None


def build(force=False):
    """Returns the library path; builds it when the reference checkout is present and the
    library is missing or older than its inputs.  Returns None when neither exists."""
    kdir = reference_kernels_dir()
    if kdir is None:
        return LIB if os.path.exists(LIB) else None
    inputs = [SHIM, HDR] + [os.path.join(kdir, k) for k in KERNELS]
    if (not force and os.path.exists(LIB)
            and os.path.getmtime(LIB) >= max(os.path.getmtime(p) for p in inputs)):
        return LIB
    os.makedirs(OUT_DIR, exist_ok=True)
    tmp = LIB + ".tmp"
    subprocess.run(["g++", *CXXFLAGS, "-I", HERE, "-I", kdir, SHIM, "-o", tmp, "-lm"],
                   check=True)
    os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    print(build(force="--force" in sys.argv))
