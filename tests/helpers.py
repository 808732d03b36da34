"""Shared generators and metrics for the parity tests.

Generators follow the benchmark's synthetic distributions (seeded numpy):
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


def make_norm_pattern_prefill(dim, seed):
    """crates/sulimo-ocl/tests/test_prefill.rs:248-272 (helper_alloc_norm): 1 + 0.02*((i+seed)%5)."""
    i = np.arange(dim)
    return (np.float32(1.0) + np.float32(0.02) * ((i + seed) % 5).astype(np.float32)).astype(np.float32)


# The model of crates/sulimo-ocl/tests/test_prefill.rs:296-331: Llama, 2 layers, embd 64,
# ffn 128, 4 query / 2 KV heads of 16, vocab 64, ring capacity 64, RoPE base 1e4, eps 1e-5.
PREFILL_TEST_CFG = dict(n_layers=2, embd=64, ffn=128, head_count=4, head_count_kv=2, head_dim=16,
                        vocab=64, rope_dim=16, rope_mode=0, eps=1e-5, rope_base=10000.0,
                        attn_softcap=0.0, bias=False, kv_capacity=64)


def make_model_pattern_prefill(overrides=None):
    """The reference test's weights (test_prefill.rs:398-463): layer l's q/k/v/o/gate/up/down use
    helper_alloc_q4 seeds l*10+2 .. l*10+9, norms seeds l*10+1 and l*10+6, the output norm
    seed 99 and the output projection seed 100.  Returns the numpy model dict that
    oracle.ffi.OracleModel and sulimo_b200.synthetic.to_device take (the token embedding is
    the output matrix; the test feeds x directly, make_x_pattern_prefill).  `overrides`
    changes dimensions (same generators)."""
    cfg = dict(PREFILL_TEST_CFG, **(overrides or {}))
    E, F = cfg["embd"], cfg["ffn"]
    qd = cfg["head_count"] * cfg["head_dim"]
    kvd = cfg["head_count_kv"] * cfg["head_dim"]
    shapes = dict(wq=(qd, E), wk=(kvd, E), wv=(kvd, E), wo=(E, qd), wg=(F, E), wu=(F, E),
                  wd=(E, F))
    seeds = dict(wq=2, wk=3, wv=4, wo=5, wg=7, wu=8, wd=9)
    layers = []
    for l in range(cfg["n_layers"]):
        L = {name: make_q4_0_pattern_prefill(*shapes[name], l * 10 + seeds[name])
             for name in shapes}
        L["attn_norm"] = make_norm_pattern_prefill(E, l * 10 + 1)
        L["ffn_norm"] = make_norm_pattern_prefill(E, l * 10 + 6)
        L["bq"] = L["bk"] = L["bv"] = None
        layers.append(L)
    out = make_q4_0_pattern_prefill(cfg["vocab"], E, 100)
    return dict(cfg=cfg, tok=out, out=out, out_norm=make_norm_pattern_prefill(E, 99),
                layers=layers)


def make_x_pattern_prefill(n, embd):
    """test_prefill.rs:516-522: x = f16(((i % 17) - 8) * 0.15) as f16 bits [n*embd]."""
    i = np.arange(n * embd)
    return (((i % 17) - 8.0).astype(np.float32) * np.float32(0.15)).astype(np.float16).view(np.uint16)


def make_act_pattern_kv_store(n_tokens, blocks_per_pos):
    """test_prefill.rs:84-89: f16(sin(0.17 i) * 5 + (i % 7 - 3)), with numpy's float32 sin."""
    i = np.arange(n_tokens * blocks_per_pos * 32)
    v = np.sin(i.astype(np.float32) * np.float32(0.17)) * np.float32(5.0) + ((i % 7) - 3).astype(np.float32)
    return v.astype(np.float32).astype(np.float16).view(np.uint16)
