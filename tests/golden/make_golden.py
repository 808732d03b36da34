"""Generates tests/golden/*.npz from the exact-arithmetic restatement (exact_ref.py).

    python tests/golden/make_golden.py

Inputs are the deterministic patterns of the reference's own unit tests (computed here in
float32 and stored explicitly, so the fixtures do not depend on a libm) plus a small seeded
sample of benchmark config 1.  Outputs are what the reference's arithmetic produces on them,
evaluated exactly and rounded once per IEEE operation.  tests/test_oracle.py checks the C
oracle against these bit for bit; the GPU tests check the kernels against the C oracle.
"""
import os
import struct
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, HERE)
import exact_ref as X  # noqa: E402


def f32(a):
    return np.asarray(a, dtype=np.float32)


def case_avx2_test():
    """crates/sulimo-cpu/src/avx2.rs:357-391 (8 blocks)."""
    nb = 8
    aos = bytearray()
    for b in range(nb):
        aos += struct.pack("<H", X.f16_bits(X.r16(X.f32_value(np.float32(0.8) + np.float32(b) * np.float32(0.1)))))
        for i in range(16):
            val = (i * 3 + b) % 16
            aos.append(val | ((15 - val) << 4))
    ws = bytearray()
    wq = bytearray()
    for b in range(nb):
        ws += aos[18 * b:18 * b + 2]
        wq += aos[18 * b + 2:18 * b + 18]
    x = (np.arange(nb * 32, dtype=np.float32) * np.float32(0.05))
    x = np.sin(x.astype(np.float64)).astype(np.float32)  # stored explicitly below
    xq8 = X.quantize_q8_0([float(v) for v in x])
    avx = X.vec_dot_avx2(bytes(ws), bytes(wq), xq8, nb)
    sca = X.vec_dot_scalar(bytes(ws), bytes(wq), xq8, nb)
    sums = X.block_sums(bytes(wq), xq8, 1, nb)
    return dict(aos=np.frombuffer(bytes(aos), np.uint8), x=x,
                xq8=np.frombuffer(xq8, np.uint8),
                ws=np.frombuffer(bytes(ws), np.uint8), wq=np.frombuffer(bytes(wq), np.uint8),
                dot_avx2=f32([float(avx)]), dot_scalar=f32([float(sca)]),
                block_sums=np.array(sums, np.int32))


def case_repack_test():
    """crates/sulimo-core/src/repack.rs:140-178 (4 blocks)."""
    aos = bytearray()
    deq = []
    for b in range(4):
        s_val = X.r16(X.f32_value(np.float32(0.5) + np.float32(b) * np.float32(0.25)))
        aos += struct.pack("<H", X.f16_bits(s_val))
        lo_vals, hi_vals = [], []
        for i in range(16):
            lo = (i + b) % 16
            hi = (i * 2 + b) % 16
            aos.append(lo | (hi << 4))
            lo_vals.append(X.r32((lo - 8) * s_val))
            hi_vals.append(X.r32((hi - 8) * s_val))
        deq += lo_vals + hi_vals
    return dict(aos=np.frombuffer(bytes(aos), np.uint8), deq=f32([float(v) for v in deq]))


def case_q8_roundtrip():
    """crates/sulimo-core/src/kv_cache.rs:216-233 (64 values: i*0.1 - 3.2 in f32)."""
    src = np.arange(64, dtype=np.float32) * np.float32(0.1) - np.float32(3.2)
    q8 = X.quantize_q8_0([float(v) for v in src])
    deq = []
    for b in range(2):
        d = X.f16_value(struct.unpack_from("<H", q8, 34 * b)[0])
        for q in struct.unpack_from("<32b", q8, 34 * b + 2):
            deq.append(float(X.r32(q * d)))
    return dict(src=src, q8=np.frombuffer(q8, np.uint8), deq=f32(deq))


def case_gemm_small():
    """test_gemm.rs:110-127 data generators on a reduced shape (n=2, k=64, m=16)."""
    n, k, m = 2, 64, 16
    nb = m * (k // 32)
    i = np.arange(nb)
    scales = (np.float32(0.05) + np.float32(0.01) * (i % 13).astype(np.float32)).astype(np.float16)
    j = np.arange(nb * 16)
    quants = (((j * 3) % 16) | (((j * 7 + 1) % 16) << 4)).astype(np.uint8)
    xi = np.arange(n * k)
    x = (((xi % 19).astype(np.float32) - np.float32(9.0)) * np.float32(0.1)).astype(np.float16)
    acc = X.gemm_scalar_reference([int(v) for v in scales.view(np.uint16)], quants.tobytes(),
                                  [int(v) for v in x.view(np.uint16)], m, k, n)
    out_f32 = f32([float(a) for a in acc])
    out_f16 = np.array([X.f16_bits(X.r16(a)) for a in acc], np.uint16)
    return dict(scales=scales.view(np.uint16), quants=quants, x=x.view(np.uint16),
                shape=np.array([m, k, n], np.int64), out_f32=out_f32, out_f16=out_f16)


def case_config1_sample():
    """8 rows of benchmark config 1 (seed 0): d=f16(|N(0,1)|*0.02), nibbles U{0..15}, K=1536."""
    rng = np.random.default_rng(0)
    rows, cols = 8, 1536
    nb = cols // 32
    d = (np.abs(rng.standard_normal(rows * nb, dtype=np.float32)) * np.float32(0.02)).astype(np.float16)
    wq = rng.integers(0, 256, size=rows * nb * 16, dtype=np.uint8)
    x = rng.standard_normal(cols, dtype=np.float32)
    xq8 = X.quantize_q8_0([float(v) for v in x])
    ws = d.view(np.uint16).tobytes()
    out = [X.vec_dot_avx2(ws[r * nb * 2:(r + 1) * nb * 2], wq[r * nb * 16:(r + 1) * nb * 16].tobytes(),
                          xq8, nb) for r in range(rows)]
    sums = X.block_sums(wq.tobytes(), xq8, rows, nb)
    return dict(ws=d.view(np.uint16), wq=wq, x=x, xq8=np.frombuffer(xq8, np.uint8),
                out_avx2=f32([float(v) for v in out]), block_sums=np.array(sums, np.int32))


def main():
    cases = {
        "avx2_test": case_avx2_test,
        "repack_test": case_repack_test,
        "q8_roundtrip": case_q8_roundtrip,
        "gemm_small": case_gemm_small,
        "config1_sample": case_config1_sample,
    }
    for name, fn in cases.items():
        path = os.path.join(HERE, f"{name}.npz")
        np.savez_compressed(path, **fn())
        print("wrote", path)


if __name__ == "__main__":
    main()
