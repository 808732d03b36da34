"""Builds oracle/libsulimo_oracle.so — the CPU restatement of the reference's hot path.

TEST INFRASTRUCTURE ONLY: the checker for the CUDA kernels and the timed CPU baseline.

Flags follow the reference's Rust semantics: no FMA contraction unless an FMA intrinsic is
called (-ffp-contract=off), AVX2/FMA/F16C for the restated intrinsics, glibc libm.
"""
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
SRC = os.path.join(HERE, "sulimo_oracle.c")
HDR = os.path.join(HERE, "sulimo_oracle.h")
LIB = os.path.join(HERE, "libsulimo_oracle.so")
CFLAGS = ["-O2", "-mavx2", "-mfma", "-mf16c", "-ffp-contract=off", "-fno-fast-math",
          "-fPIC", "-shared", "-std=gnu11", "-Wall"]


def build(force=False):
    if (not force and os.path.exists(LIB)
            and os.path.getmtime(LIB) >= max(os.path.getmtime(SRC), os.path.getmtime(HDR))):
        return LIB
    tmp = LIB + ".tmp"
    subprocess.run(["gcc", *CFLAGS, SRC, "-o", tmp, "-lm", "-lpthread"], check=True)
    os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    print(build(force="--force" in sys.argv))
