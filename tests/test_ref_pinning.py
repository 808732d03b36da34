"""CPU tests pinning the C restatement (oracle/sulimo_oracle.c) to values produced by the
reference's own code: its OpenCL C kernels kernels/gemm_q4_0.cl and kernels/prefill.cl,
compiled unchanged for the host (oracle/_ref, oracle/ref_ocl_shim.cpp).

Two sources: the committed fixture tests/golden/ref_ocl.npz (made from those kernels by
tests/golden/make_ref_ocl_golden.py; always checked), and the live library where it is built
(checked on more shapes; skipped when neither the library nor a reference checkout exists).
The bar is bit-exact everywhere: the restatement performs the kernels' float operations in
their source order with the same roundings.
"""
import os

import numpy as np
import pytest

import oracle.ffi as O
import oracle.ref_ffi as R
from helpers import (make_act_pattern_kv_store, make_model_pattern_prefill, make_q4_0,
                     make_q4_0_pattern_gemm, make_x_pattern_gemm, make_x_pattern_prefill)
from sulimo_b200.synthetic import make_model_numpy

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "ref_ocl.npz")

live = pytest.mark.skipif(not R.available(),
                          reason="oracle/_ref not built and no reference checkout to build it")


def bits(a):
    a = np.asarray(a)
    return a.view(np.uint32) if a.dtype == np.float32 else a


def same(a, b):
    return np.array_equal(bits(a), bits(b))


# ---- fixture (values produced by the reference's kernels) --------------------------------------

def test_fixture_gemm_portable():
    g = np.load(GOLDEN)
    for tag in ("g0", "g1"):
        n, k, m = (int(v) for v in g[f"{tag}_shape"])
        out = O.gemm_q4_0_f16_scalar_reference(g[f"{tag}_scales"], g[f"{tag}_quants"],
                                               g[f"{tag}_x"], m, k, n)
        assert same(out, g[f"{tag}_out"]), tag


def test_fixture_kv_store_q8_0():
    g = np.load(GOLDEN)
    kv = np.zeros_like(g["kv_ring"])
    O.kv_store_q8_0(g["kv_act"], kv, 5, 64, 8, 16)
    assert same(kv, g["kv_ring"])


def test_fixture_logits_f16_output():
    g = np.load(GOLDEN)
    x = g["lg_x"].reshape(3, 256)
    out = O.gemm_q4_0_f16_f32out(g["lg_scales"], g["lg_quants"], np.ascontiguousarray(x[2]),
                                 96, 256, 1)
    assert same(out, g["lg_out"])


def test_fixture_execute_prefill_ubatch():
    """test_prefill.rs:296-566's model and prompt through the restated ubatch."""
    g = np.load(GOLDEN)
    om = O.OracleModel(make_model_pattern_prefill())
    logits, x = om.prefill_ubatch(np.zeros(16, np.int32), 0, x_f16=g["pf_x0"])
    assert same(logits, g["pf_logits"])
    assert same(x, g["pf_x"])
    for l, (kr, vr) in enumerate(om.rings):
        assert same(kr, g[f"pf_k{l}"]) and same(vr, g[f"pf_v{l}"]), l


# ---- live library --------------------------------------------------------------------------

@live
@pytest.mark.parametrize("n,k,m", [(8, 256, 256), (32, 512, 512), (128, 512, 1024),
                                   (512, 1024, 1024)])
def test_gemm_reference_test_shapes(n, k, m):
    """crates/sulimo-ocl/tests/test_gemm.rs:75-127: shapes and data generators."""
    s, q = make_q4_0_pattern_gemm(m, k)
    x = make_x_pattern_gemm(n, k).view(np.uint16)
    assert same(O.gemm_q4_0_f16_scalar_reference(s, q, x, m, k, n),
                R.gemm_q4_0_f16_portable(s, q, x, m, k, n, threads=8))


@live
def test_gemm_config2_sample():
    """benchmark config 2's generators (seeded Q4_0 8960 x 1536, f16 N(0,1) activations) on a
    48-token sample, f16 outputs and (logits_f16_output) fp32 outputs."""
    m, k, n = 8960, 1536, 48
    s, q = make_q4_0(m, k, seed=0)
    x = np.random.default_rng(1).standard_normal(n * k).astype(np.float16).view(np.uint16)
    assert same(O.gemm_q4_0_f16_scalar_reference(s, q, x, m, k, n),
                R.gemm_q4_0_f16_portable(s, q, x, m, k, n, threads=8))
    f32 = O.gemm_q4_0_f16_f32out(s, q, x, m, k, n, threads=8).reshape(n, m)
    for t in (0, n - 1):
        assert same(f32[t], R.logits_f16_output(x, s, q, m, k, t, threads=8))


@live
def test_gemm_down_shape_sample():
    """The reversed down-projection shape (K = 8960) on a 16-token sample."""
    m, k, n = 1536, 8960, 16
    s, q = make_q4_0(m, k, seed=2)
    x = np.random.default_rng(3).standard_normal(n * k).astype(np.float16).view(np.uint16)
    assert same(O.gemm_q4_0_f16_scalar_reference(s, q, x, m, k, n),
                R.gemm_q4_0_f16_portable(s, q, x, m, k, n, threads=8))


@live
@pytest.mark.parametrize("start,cap,n", [(5, 64, 16), (0, 8, 20), (61, 64, 9)])
def test_kv_store(start, cap, n):
    """test_prefill.rs:57-192's case, then rings that wrap (the last writer of a slot wins)."""
    bpp = 8
    act = make_act_pattern_kv_store(n, bpp)
    a = np.zeros(cap * bpp * 34, np.uint8)
    b = a.copy()
    O.kv_store_q8_0(act, a, start, cap, bpp, n)
    R.kv_store_q8_0(act, b, start, cap, bpp, n)
    assert same(a, b)
    rnd = (np.random.default_rng(start).standard_normal(n * bpp * 32) * 30).astype(np.float16)
    O.kv_store_q8_0(rnd.view(np.uint16), a, start, cap, bpp, n)
    R.kv_store_q8_0(rnd.view(np.uint16), b, start, cap, bpp, n)
    assert same(a, b)


@live
def test_small_kernels():
    rng = np.random.default_rng(5)
    D, N = 96, 7
    x = (rng.standard_normal(N * D) * 3).astype(np.float16).view(np.uint16)
    w = (1 + 0.1 * rng.standard_normal(D)).astype(np.float32)
    assert same(O.rmsnorm_f16(x, w, 1e-6, D), R.rmsnorm_f16_f32w(x, w, 1e-6, D))
    for mode, rope_dim in ((0, 64), (1, 64), (1, 32)):
        v = (rng.standard_normal(N * 3 * 64)).astype(np.float16).view(np.uint16)
        assert same(O.rope_f16(v, 3, 64, rope_dim, 1e6, mode, 1000),
                    R.rope_f16(v, 3, 64, rope_dim, 1e6, mode, 1000)), (mode, rope_dim)
    g = (rng.standard_normal(999) * 4).astype(np.float16).view(np.uint16)
    u = rng.standard_normal(999).astype(np.float16).view(np.uint16)
    assert same(O.silu_mul_f16(g, u), R.silu_mul_f16(g, u))
    assert same(O.add_f16(g, u), R.add_f16(g, u))


@live
@pytest.mark.parametrize("H,Hkv,hd,start,n,cap", [(4, 2, 32, 0, 12, 64), (12, 2, 128, 20, 9, 64),
                                                  (8, 8, 64, 3, 6, 8)])
def test_attention_prefill(H, Hkv, hd, start, n, cap):
    """causal_gqa_attention_prefill over a ring holding positions 0..start+n-1 (the last case
    has more keys than slots: both read slot p % capacity)."""
    rng = np.random.default_rng(H + start)
    bpp = Hkv * hd // 32
    kr = np.zeros(cap * bpp * 34, np.uint8)
    vr = np.zeros_like(kr)
    for p in range(start + n):
        O.kv_store_f32(rng.standard_normal(Hkv * hd).astype(np.float32), kr, p, cap, bpp)
        O.kv_store_f32(rng.standard_normal(Hkv * hd).astype(np.float32), vr, p, cap, bpp)
    q = rng.standard_normal(n * H * hd).astype(np.float16).view(np.uint16)
    assert same(O.attention_prefill_f16(q, kr, vr, start, cap, H, Hkv, hd),
                R.causal_gqa_attention_prefill(q, kr, vr, start, cap, H, Hkv, hd, threads=4))


@live
def test_execute_prefill_ubatch_reference_test_model():
    w = make_model_pattern_prefill()
    a, b = O.OracleModel(w), O.OracleModel(w)
    x0 = make_x_pattern_prefill(16, w["cfg"]["embd"])
    la, xa = a.prefill_ubatch(np.zeros(16, np.int32), 0, x_f16=x0)
    lb, xb = R.execute_prefill_ubatch(b, np.zeros(16, np.int32), 0, x_f16=x0)
    assert same(la, lb) and same(xa, xb)
    for (ka, va), (kb, vb) in zip(a.rings, b.rings):
        assert same(ka, kb) and same(va, vb)


@live
@pytest.mark.parametrize("rope_mode,H,Hkv", [(1, 4, 2), (0, 8, 2), (1, 4, 4)])
def test_execute_prefill_ubatch_seeded_models(rope_mode, H, Hkv):
    """Seeded models (benchmark distributions), three ubatches of 16/9/7 tokens continuing the
    same rings, embeddings from lookup_token_embedding_f16."""
    hd = 256 // H
    cfg = dict(n_layers=2, embd=256, ffn=512, head_count=H, head_count_kv=Hkv, head_dim=hd,
               vocab=500, rope_dim=hd, rope_mode=rope_mode, eps=1e-6, rope_base=1e6,
               attn_softcap=0.0, bias=False)
    w = make_model_numpy(cfg, seed=7 + H, kv_capacity=64)
    a, b = O.OracleModel(w), O.OracleModel(w)
    toks = np.random.default_rng(H).integers(0, 500, 32)
    pos = 0
    for n in (16, 9, 7):
        la, xa = a.prefill_ubatch(toks[pos:pos + n], pos, threads=4)
        lb, xb = R.execute_prefill_ubatch(b, toks[pos:pos + n], pos, threads=4)
        assert same(la, lb) and same(xa, xb), pos
        pos += n
    for (ka, va), (kb, vb) in zip(a.rings, b.rings):
        assert same(ka, kb) and same(va, vb)


@live
def test_reference_prefill_test_replayed_on_the_host():
    """crates/sulimo-ocl/tests/test_prefill.rs:296-890 end to end on the host: the reference's
    own GPU kernels (execute_prefill_ubatch over kernels/prefill.cl and gemm_q4_0.cl) against the
    restated CPU oracle of that test, with the test's model, prompt and bars: every K/V element
    within 1.05 * d + 1e-4 of the oracle's, logits cosine >= 0.99, the same greedy token."""
    w = make_model_pattern_prefill()
    gpu, cpu = O.OracleModel(w), O.OracleModel(w)
    x0 = make_x_pattern_prefill(16, w["cfg"]["embd"])
    lg, _ = R.execute_prefill_ubatch(gpu, np.zeros(16, np.int32), 0, x_f16=x0)
    lc = cpu.prefill_ubatch_f32(None, 0, x_f16=x0)
    slot = w["cfg"]["head_count_kv"] * w["cfg"]["head_dim"] // 32 * 34
    nbytes = 16 * slot
    for (kg, vg), (kc, vc) in zip(gpu.rings, cpu.rings):
        for a, b in ((kg, kc), (vg, vc)):
            g = O.dequantize_q8_0_to_f32(a[:nbytes], nbytes // 34)
            c = O.dequantize_q8_0_to_f32(b[:nbytes], nbytes // 34)
            d = O.f16_to_f32(b[:nbytes].reshape(-1, 34)[:, :2].copy().view(np.uint16).ravel())
            assert np.all(np.abs(g - c) <= np.repeat(d, 32) * 1.05 + 1e-4)
    cos = float(lg.astype(np.float64) @ lc / (np.linalg.norm(lg) * np.linalg.norm(lc)))
    assert cos >= 0.99
    assert int(np.argmax(lg)) == int(np.argmax(lc))
