"""CPU tests of the oracle: the reference's own unit tests re-expressed against the C
restatement, plus bit-exact agreement with the golden fixtures made by the independent
exact-arithmetic restatement (tests/golden/exact_ref.py)."""
import os

import numpy as np
import pytest

import oracle.ffi as O
from helpers import make_q4_0

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def load(name):
    return np.load(os.path.join(GOLDEN, f"{name}.npz"))


# ---- f16 conversion (half 2.7.1 semantics: RNE) vs numpy's float16 cast --------------------

def test_f16_conversion_matches_ieee_rne():
    rng = np.random.default_rng(1)
    x = np.concatenate([
        rng.standard_normal(20000).astype(np.float32) * 10,
        rng.standard_normal(5000).astype(np.float32) * 1e-5,   # f16 subnormal range
        np.array([0.0, -0.0, 65504, 65519.99, 65520, 1e-8, 6e-8, 2.98e-8, -1e9], np.float32),
    ])
    ours = O.f32_to_f16(x)
    with np.errstate(over="ignore"):
        ref = x.astype(np.float16).view(np.uint16)
    assert np.array_equal(ours, ref)
    back = O.f16_to_f32(ref)
    assert np.array_equal(back.view(np.uint32), ref.view(np.float16).astype(np.float32).view(np.uint32))


# ---- crates/sulimo-core/src/repack.rs:138-179 ------------------------------------------------

def test_repack_and_dequantize_roundtrip_bit_exact():
    g = load("repack_test")
    nb, sc, qu = O.repack_q4_0_aos_to_soa(g["aos"])
    assert nb == 4
    w_aos = O.dequantize_q4_0_aos(g["aos"])
    w_soa = O.dequantize_q4_0_soa(sc, qu, 4)
    assert np.array_equal(w_aos.view(np.uint32), w_soa.view(np.uint32))
    assert np.array_equal(w_soa.view(np.uint32), g["deq"].view(np.uint32))


def test_repack_errors():
    # InvalidAosLength / ScalesBufferTooSmall / QuantsBufferTooSmall (repack.rs:50-70)
    assert O.repack_q4_0_aos_to_soa(np.zeros(17, np.uint8))[0] == -1
    assert O.repack_q4_0_aos_to_soa(np.zeros(36, np.uint8), scales_len=3)[0] == -2
    assert O.repack_q4_0_aos_to_soa(np.zeros(36, np.uint8), quants_len=31)[0] == -3


# ---- crates/sulimo-core/src/kv_cache.rs:216-233 ----------------------------------------------

def test_quantize_and_dequantize_q8_0():
    g = load("q8_roundtrip")
    q8 = O.quantize_f32_to_q8_0(g["src"])
    assert np.array_equal(q8, g["q8"])
    deq = O.dequantize_q8_0_to_f32(q8, 2)
    assert np.array_equal(deq.view(np.uint32), g["deq"].view(np.uint32))
    assert np.max(np.abs(g["src"] - deq)) < 0.05


def test_quantize_edge_cases():
    x = np.zeros(32 * 6, np.float32)
    x[32:64] = 1e-40                      # subnormal block: d underflows in f16
    x[64:96] = np.linspace(-1e4, 1e4, 32)
    x[96:128] = -7.0                      # constant negative block
    x[128] = np.nan                       # NaN is skipped by the max (a > max_abs is false)
    x[129:160] = 2.0
    x[160:192] = np.float32(3.4e38)
    q8 = O.quantize_f32_to_q8_0(x)
    # all-zero block: d = 0, id = 0, q = 0
    assert np.all(q8[0:34] == 0)
    assert q8[34 * 3 + 2] == (np.int8(-127).view(np.uint8))
    assert q8[34 * 4 + 2] == 0            # NaN -> 0
    assert np.all(q8[34 * 4 + 3:34 * 4 + 34].view(np.int8) == 127)


# ---- crates/sulimo-cpu/src/avx2.rs:352-396 ---------------------------------------------------

def test_avx2_vs_scalar_q4_0_q8_0_precision():
    g = load("avx2_test")
    xq8 = O.quantize_f32_to_q8_0(g["x"])
    assert np.array_equal(xq8, g["xq8"])
    s = O.vec_dot_q4_0_q8_0_scalar(g["ws"], g["wq"], xq8, 8)
    a = O.vec_dot_q4_0_q8_0_avx2(g["ws"], g["wq"], xq8, 8)
    rel = abs(s - a) / max(abs(s), 1e-5)
    assert rel <= 1e-3
    # bit-exact against the exact-arithmetic restatement
    assert np.float32(a).view(np.uint32) == g["dot_avx2"].view(np.uint32)[0]
    assert np.float32(s).view(np.uint32) == g["dot_scalar"].view(np.uint32)[0]
    sums = O.block_sums_q4_0_q8_0(g["ws"], g["wq"], xq8, 1, 256)
    assert np.array_equal(sums, g["block_sums"])


def test_config1_sample_bit_exact():
    g = load("config1_sample")
    xq8 = O.quantize_f32_to_q8_0(g["x"])
    assert np.array_equal(xq8, g["xq8"])
    out = O.matvec_q4_0_q8_0_avx2(g["ws"], g["wq"], xq8, 8, 1536)
    assert np.array_equal(out.view(np.uint32), g["out_avx2"].view(np.uint32))
    out_mt = O.matvec_q4_0_q8_0_avx2(g["ws"], g["wq"], xq8, 8, 1536, threads=3)
    assert np.array_equal(out_mt.view(np.uint32), out.view(np.uint32))
    sums = O.block_sums_q4_0_q8_0(g["ws"], g["wq"], xq8, 8, 1536)
    assert np.array_equal(sums, g["block_sums"])


def test_avx2_scalar_block_sum_identity():
    """The eight AVX2 lane sums add up to the scalar block_sum (avx2.rs:146-155 vs
    scalar.rs:189-199): float(sum) * d summed over blocks agrees with the scalar dot."""
    ws, wq = make_q4_0(64, 512, seed=3)
    x = np.random.default_rng(4).standard_normal(512).astype(np.float32)
    xq8 = O.quantize_f32_to_q8_0(x)
    a = O.matvec_q4_0_q8_0_avx2(ws, wq, xq8, 64, 512)
    s = O.matvec_q4_0_q8_0_scalar(ws, wq, xq8, 64, 512)
    assert np.max(np.abs(a - s) / np.maximum(np.abs(s), 1e-3)) < 1e-4


# ---- crates/sulimo-ocl/src/gemm.rs:106-147 ---------------------------------------------------

def test_gemm_scalar_reference_bit_exact():
    g = load("gemm_small")
    m, k, n = (int(v) for v in g["shape"])
    out16 = O.gemm_q4_0_f16_scalar_reference(g["scales"], g["quants"], g["x"], m, k, n)
    assert np.array_equal(out16, g["out_f16"])
    out32 = O.gemm_q4_0_f16_f32out(g["scales"], g["quants"], g["x"], m, k, n, threads=2)
    assert np.array_equal(out32.view(np.uint32), g["out_f32"].view(np.uint32))


def test_cpu_prefill_projection_is_per_token_matvec():
    ws, wq = make_q4_0(40, 256, seed=5)
    x = np.random.default_rng(6).standard_normal((3, 256)).astype(np.float32)
    out = O.cpu_prefill_projection(ws, wq, x, 40, 256, 3, threads=2).reshape(3, 40)
    for t in range(3):
        ref = O.matvec_q4_0_q8_0_avx2(ws, wq, O.quantize_f32_to_q8_0(x[t]), 40, 256)
        assert np.array_equal(out[t].view(np.uint32), ref.view(np.uint32))


# ---- crates/sulimo-cpu/src/scalar.rs tests (:365-427) ----------------------------------------

def test_rmsnorm_scalar():
    out = O.rmsnorm_scalar(np.array([1, 2, 3, 4], np.float32), np.ones(4, np.float32), 1e-5)
    assert abs(np.sqrt(np.mean(out.astype(np.float64) ** 2)) - 1.0) < 1e-3


def test_rmsnorm_avx2_matches_scalar():
    x = np.sin(np.arange(64) * 0.1).astype(np.float32)
    w = np.cos(np.arange(64) * 0.05).astype(np.float32)
    assert np.max(np.abs(O.rmsnorm_avx2(x, w, 1e-5) - O.rmsnorm_scalar(x, w, 1e-5))) < 1e-5


def test_rmsnorm_gemma_with_zero_weight_equals_rmsnorm():
    """scalar.rs:390-403: (1 + 0) weights give rmsnorm with unit weights (here through the
    AVX2 restatement, whose tail and vector paths both run at length 4 and 12)."""
    for n in (4, 12):
        x = np.arange(1, n + 1, dtype=np.float32)
        out = O.rmsnorm_gemma_avx2(x, np.zeros(n, np.float32), 1e-5)
        ref = O.rmsnorm_scalar(x, np.ones(n, np.float32), 1e-5)
        assert np.max(np.abs(out - ref)) < 1e-6


def test_rmsnorm_gemma_avx2_vs_scalar_form():
    """avx2.rs:399-425: sin / cos inputs of length 64 against the scalar form
    x * scale * (1 + w) (scalar.rs:43-58), restated here in float32 numpy."""
    x = np.sin(np.arange(64, dtype=np.float32) * np.float32(0.1)).astype(np.float32)
    w = np.cos(np.arange(64, dtype=np.float32) * np.float32(0.05)).astype(np.float32)
    ss = np.float32(0)
    for v in x:
        ss = np.float32(ss + v * v)
    scale = np.float32(1) / np.sqrt(np.float32(ss / np.float32(64)) + np.float32(1e-5))
    ref = (x * scale * (np.float32(1) + w)).astype(np.float32)
    assert np.max(np.abs(O.rmsnorm_gemma_avx2(x, w, 1e-5) - ref)) < 1e-5


def test_logit_softcap():
    """scalar.rs:406-416."""
    out = O.logit_softcap(np.array([1000.0, -1000.0, 0.0, 100.0], np.float32), 50.0)
    assert 49.99 < out[0] <= 50.0 and -50.0 <= out[1] < -49.99
    assert out[2] == 0.0 and abs(out[3] - 48.2014) < 1e-3
    same = np.array([1.0, -2.0], np.float32)
    assert np.array_equal(O.logit_softcap(same, 0.0), same)  # cap <= 0: untouched


def test_geglu():
    """scalar.rs:419-427, plus the tanh-form value at 1.0."""
    out = O.geglu(np.array([0.0, 1.0, -1.0], np.float32), np.array([2.0, 3.0, 4.0], np.float32))
    assert out[0] == 0.0 and out[1] > 0.0 and out[2] < 0.0
    g1 = 0.5 * (1.0 + np.tanh(0.7978846 * (1.0 + 0.044715)))
    assert abs(out[1] - 3.0 * g1) < 1e-6


def test_softmax_scalar():
    x = O.softmax(np.array([1, 2, 3], np.float32))
    assert abs(float(x.sum()) - 1.0) < 1e-5 and x[2] > x[1] > x[0]


def test_rope_modes():
    v = np.arange(8, dtype=np.float32)
    norm = O.rope_head(v, 0, 8, 10000.0, 0)
    assert np.array_equal(norm, v)  # position 0 is the identity
    neox = O.rope_head(v, 3, 8, 10000.0, 1)
    assert abs(np.linalg.norm(neox) - np.linalg.norm(v)) < 1e-4


# ---- crates/sulimo-cpu/src/scalar.rs:287-359 + kv_cache.rs:114-128 ---------------------------

def test_decode_attention_single_position_returns_v():
    """With one position the softmax weight is 1: out == dequant(V[0]) for every head."""
    H, Hkv, hd, cap = 4, 2, 32, 8
    rng = np.random.default_rng(7)
    kv_dim = Hkv * hd
    kr = np.zeros(cap * kv_dim // 32 * 34, np.uint8)
    vr = np.zeros_like(kr)
    O.kv_store_f32(rng.standard_normal(kv_dim).astype(np.float32), kr, 0, cap, kv_dim // 32)
    vv = rng.standard_normal(kv_dim).astype(np.float32)
    O.kv_store_f32(vv, vr, 0, cap, kv_dim // 32)
    q = rng.standard_normal(H * hd).astype(np.float32)
    out = O.causal_gqa_decode(q, kr, vr, cap, 1, H, Hkv, hd)
    vdeq = O.dequantize_q8_0_to_f32(vr, kv_dim // 32)
    for h in range(H):
        assert np.allclose(out[h * hd:(h + 1) * hd], vdeq[(h // 2) * hd:(h // 2 + 1) * hd], atol=1e-6)


def test_kv_store_ring_wraps():
    cap, bpp = 4, 2
    kv = np.zeros(cap * bpp * 34, np.uint8)
    act = np.random.default_rng(8).standard_normal((6, bpp * 32)).astype(np.float16)
    O.kv_store_q8_0(act.view(np.uint16), kv, 3, cap, bpp, 6)  # positions 3..8 -> slots 3,0,1,2,3,0
    # the last writer of each slot wins: slot 3 <- t=4 (pos 7), slot 0 <- t=5 (pos 8)
    exp = np.zeros_like(kv)
    for t in range(6):
        blk = O.quantize_f32_to_q8_0(act[t].astype(np.float32))
        s = (3 + t) % cap
        exp[s * bpp * 34:(s + 1) * bpp * 34] = blk
    assert np.array_equal(kv, exp)


# ---- crates/sulimo-cpu/src/{avx2,scalar}.rs: the raw F32 / F16 matvecs ------------------------

@pytest.mark.parametrize("kind", ["f32", "f16"])
def test_dense_matvec_avx2_vs_scalar(kind):
    """matvec_f32/f16_avx2 (avx2.rs:259-331) against the scalar kernels (scalar.rs:228-251) and
    a float64 product: only the summation order differs."""
    rng = np.random.default_rng(11)
    rows, cols = 48, 1001
    w = rng.standard_normal((rows, cols)).astype(np.float32)
    if kind == "f16":
        w = w.astype(np.float16).view(np.uint16)
        wd = w.view(np.float16).astype(np.float64)
    else:
        wd = w.astype(np.float64)
    x = rng.standard_normal(cols).astype(np.float32)
    a = O.matvec_dense(w, x, rows, cols, kind, avx2=True)
    s = O.matvec_dense(w, x, rows, cols, kind, avx2=False)
    exact = wd @ x.astype(np.float64)
    assert np.max(np.abs(a - exact)) < 1e-3 and np.max(np.abs(s - exact)) < 1e-3
    assert not np.array_equal(a, s)  # different orders: the AVX2 lanes are what the GPU mirrors
