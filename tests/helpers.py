"""Shared generators and metrics for the parity tests.

Generators follow BASELINE.json's synthetic distributions (seeded numpy):
  Q4_0 weights: d = f16(|N(0,1)| * 0.02), nibbles uniform 0..15 (w = d*(q-8)), SoA layout
  activations:  fp32 / fp16 N(0,1)
and the deterministic patterns of the reference's own tests.
"""
import numpy as np


def make_q4_0(rows, cols, seed=0):
    """Random Q4_0 SoA tensor: (scales u16 [rows*nb], quants u8 [rows*nb*16])."""
    assert cols % 32 == 0
    rng = np.random.default_rng(seed)
    nb = rows * (cols // 32)
    d = (np.abs(rng.standard_normal(nb, dtype=np.float32)) * np.float32(0.02)).astype(np.float16)
    quants = rng.integers(0, 256, size=nb * 16, dtype=np.uint8)
    return d.view(np.uint16).copy(), quants


def make_q4_0_pattern_gemm(m, k):
    """crates/sulimo-ocl/tests/test_gemm.rs:110-122: scales 0.05+0.01(i%13), nibbles
    (3i)%16 | ((7i+1)%16)<<4."""
    nb = m * (k // 32)
    i = np.arange(nb)
    scales = (0.05 + 0.01 * (i % 13)).astype(np.float32).astype(np.float16).view(np.uint16)
    j = np.arange(nb * 16)
    quants = (((j * 3) % 16) | (((j * 7 + 1) % 16) << 4)).astype(np.uint8)
    return scales.copy(), quants


def make_x_pattern_gemm(n, k):
    """test_gemm.rs:124-127: x = ((i % 19) - 9) * 0.1 as f16."""
    i = np.arange(n * k)
    return (((i % 19) - 9.0) * 0.1).astype(np.float32).astype(np.float16)


def make_q4_0_pattern_prefill(rows, cols, seed):
    """crates/sulimo-ocl/tests/test_prefill.rs:194-246 (helper_alloc_q4)."""
    blocks = rows * cols // 32
    i = np.arange(blocks)
    scales = (0.02 + 0.005 * ((i + seed) % 7)).astype(np.float32).astype(np.float16)
    j = np.arange(blocks * 16)
    quants = ((((j + seed) * 3) % 15) | ((((j + seed) * 7 + 1) % 15) << 4)).astype(np.uint8)
    return scales.view(np.uint16).copy(), quants


def rel_l2(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    den = np.linalg.norm(b)
    return float(np.linalg.norm(a - b) / (den if den > 0 else 1.0))


def max_rel_err(gpu, cpu):
    """test_gemm.rs:44-56: max |g-c| / max(|c|, 1)."""
    g = np.asarray(gpu, np.float64)
    c = np.asarray(cpu, np.float64)
    return float(np.max(np.abs(g - c) / np.maximum(np.abs(c), 1.0))) if c.size else 0.0


def cosine(a, b):
    a = np.asarray(a, np.float64).ravel()
    b = np.asarray(b, np.float64).ravel()
    na, nb = np.linalg.norm(a), np.linalg.norm(b)
    if na == 0 or nb == 0:
        return 0.0
    return float(a @ b / (na * nb))
