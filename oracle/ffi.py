"""numpy bindings of liboracle (the CPU restatement of the reference's hot path).

TEST INFRASTRUCTURE ONLY: imported by tests/, __graft_entry__.smoke() and bench.py's CPU
baseline leg as the checker.  The product library (libsulimo_cuda.so) never uses it.
"""
import ctypes as C
import os

import numpy as np

from . import build as _build

_lib = None


def lib():
    global _lib
    if _lib is None:
        path = _build.build()
        L = C.CDLL(path)
        vp, sz, i32, f32 = C.c_void_p, C.c_size_t, C.c_int, C.c_float
        sig = {
            "oracle_f32_to_f16": (C.c_uint16, [f32]),
            "oracle_f16_to_f32": (f32, [C.c_uint16]),
            "oracle_f32_to_f16_array": (None, [vp, vp, sz]),
            "oracle_f16_to_f32_array": (None, [vp, vp, sz]),
            "oracle_repack_q4_0_aos_to_soa": (C.c_long, [vp, sz, vp, sz, vp, sz]),
            "oracle_dequantize_q4_0_aos": (None, [vp, sz, vp]),
            "oracle_dequantize_q4_0_soa": (None, [vp, vp, sz, vp]),
            "oracle_lookup_token_embedding_f16": (None, [vp, vp, sz, C.c_uint32, vp]),
            "oracle_quantize_f32_to_q8_0": (None, [vp, sz, vp]),
            "oracle_dequantize_q8_0_to_f32": (None, [vp, sz, vp]),
            "oracle_kv_store_q8_0": (None, [vp, vp, sz, sz, sz, sz]),
            "oracle_kv_store_f32": (None, [vp, vp, sz, sz, sz]),
            "oracle_vec_dot_q4_0_q8_0_scalar": (f32, [vp, vp, vp, sz]),
            "oracle_matvec_q4_0_q8_0_scalar": (None, [vp, vp, vp, sz, sz, vp]),
            "oracle_vec_dot_q4_0_q8_0_avx2": (f32, [vp, vp, vp, sz]),
            "oracle_matvec_q4_0_q8_0_avx2": (None, [vp, vp, vp, sz, sz, vp]),
            "oracle_matvec_q4_0_q8_0_avx2_mt": (None, [vp, vp, vp, sz, sz, vp, i32]),
            "oracle_block_sums_q4_0_q8_0": (None, [vp, vp, vp, sz, sz, vp]),
            "oracle_gemm_q4_0_f16_scalar_reference": (None, [vp, vp, vp, sz, sz, sz, vp]),
            "oracle_gemm_q4_0_f16_scalar_f32out": (None, [vp, vp, vp, sz, sz, sz, vp, i32]),
            "oracle_cpu_prefill_projection": (None, [vp, vp, vp, sz, sz, sz, vp, i32]),
            "oracle_rmsnorm_scalar": (None, [vp, vp, sz, f32, vp]),
            "oracle_rmsnorm_avx2": (None, [vp, vp, sz, f32, vp]),
            "oracle_rope_head_scalar": (None, [vp, sz, sz, f32, i32]),
            "oracle_softmax_scalar": (None, [vp, sz]),
            "oracle_swiglu_scalar": (None, [vp, vp, vp, sz]),
            "oracle_rmsnorm_gemma_avx2": (None, [vp, vp, sz, f32, vp]),
            "oracle_geglu_scalar": (None, [vp, vp, vp, sz]),
            "oracle_logit_softcap_scalar": (None, [vp, sz, f32]),
            "oracle_causal_gqa_decode": (None, [vp, vp, vp, sz, sz, sz, sz, sz, vp, vp, f32]),
            "oracle_rmsnorm_f16": (None, [vp, vp, vp, sz, f32, sz]),
            "oracle_rope_f16": (None, [vp, sz, sz, sz, f32, i32, sz, sz]),
            "oracle_attention_prefill_f16": (None, [vp, vp, vp, vp, sz, sz, sz, sz, sz, sz]),
            "oracle_silu_mul_f16": (None, [vp, vp, vp, sz]),
            "oracle_add_f16": (None, [vp, vp, sz]),
            "oracle_prefill_ubatch": (i32, [vp, vp, sz, sz, vp, i32]),
            "oracle_prefill_ubatch_f32": (i32, [vp, vp, sz, sz, vp, i32]),
            "oracle_matvec_f32_avx2": (None, [vp, vp, sz, sz, vp]),
            "oracle_matvec_f16_avx2": (None, [vp, vp, sz, sz, vp]),
            "oracle_matvec_f32_scalar": (None, [vp, vp, sz, sz, vp]),
            "oracle_matvec_f16_scalar": (None, [vp, vp, sz, sz, vp]),
        }
        for name, (res, args) in sig.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


def _p(a):
    assert a.flags["C_CONTIGUOUS"], "arrays passed to the oracle must be C-contiguous"
    return a.ctypes.data_as(C.c_void_p)


def f32_to_f16(x):
    x = np.ascontiguousarray(x, dtype=np.float32)
    out = np.empty(x.shape, np.uint16)
    lib().oracle_f32_to_f16_array(_p(x), _p(out), x.size)
    return out


def f16_to_f32(h):
    h = np.ascontiguousarray(h, dtype=np.uint16)
    out = np.empty(h.shape, np.float32)
    lib().oracle_f16_to_f32_array(_p(h), _p(out), h.size)
    return out


def repack_q4_0_aos_to_soa(aos, scales_len=None, quants_len=None):
    aos = np.ascontiguousarray(aos, dtype=np.uint8)
    nb = aos.size // 18
    sc = np.zeros(scales_len if scales_len is not None else nb * 2, np.uint8)
    qu = np.zeros(quants_len if quants_len is not None else nb * 16, np.uint8)
    r = lib().oracle_repack_q4_0_aos_to_soa(_p(aos), aos.size, _p(sc), sc.size, _p(qu), qu.size)
    return r, sc, qu


def dequantize_q4_0_aos(aos):
    aos = np.ascontiguousarray(aos, dtype=np.uint8)
    nb = aos.size // 18
    out = np.empty(nb * 32, np.float32)
    lib().oracle_dequantize_q4_0_aos(_p(aos), nb, _p(out))
    return out


def dequantize_q4_0_soa(scales_u8, quants, num_blocks):
    scales_u8 = np.ascontiguousarray(scales_u8).view(np.uint8)
    quants = np.ascontiguousarray(quants, dtype=np.uint8)
    out = np.empty(num_blocks * 32, np.float32)
    lib().oracle_dequantize_q4_0_soa(_p(scales_u8), _p(quants), num_blocks, _p(out))
    return out


def lookup_token_embedding_f16(scales, quants, embd, token_id):
    scales = np.ascontiguousarray(scales).view(np.uint8)
    quants = np.ascontiguousarray(quants, dtype=np.uint8)
    out = np.empty(embd, np.uint16)
    lib().oracle_lookup_token_embedding_f16(_p(scales), _p(quants), embd, token_id, _p(out))
    return out


def quantize_f32_to_q8_0(x):
    x = np.ascontiguousarray(x, dtype=np.float32)
    assert x.size % 32 == 0
    out = np.empty(x.size // 32 * 34, np.uint8)
    lib().oracle_quantize_f32_to_q8_0(_p(x), x.size, _p(out))
    return out


def dequantize_q8_0_to_f32(q8, num_blocks):
    q8 = np.ascontiguousarray(q8, dtype=np.uint8)
    out = np.empty(num_blocks * 32, np.float32)
    lib().oracle_dequantize_q8_0_to_f32(_p(q8), num_blocks, _p(out))
    return out


def kv_store_q8_0(act_f16, kv, start_pos, capacity, blocks_per_pos, n):
    act_f16 = np.ascontiguousarray(act_f16, dtype=np.uint16)
    assert kv.flags["C_CONTIGUOUS"] and kv.dtype == np.uint8
    lib().oracle_kv_store_q8_0(_p(act_f16), _p(kv), start_pos, capacity, blocks_per_pos, n)


def kv_store_f32(vec, kv, pos, capacity, blocks_per_pos):
    vec = np.ascontiguousarray(vec, dtype=np.float32)
    lib().oracle_kv_store_f32(_p(vec), _p(kv), pos, capacity, blocks_per_pos)


def vec_dot_q4_0_q8_0_scalar(ws, wq, xq8, nb):
    return lib().oracle_vec_dot_q4_0_q8_0_scalar(_p(ws), _p(wq), _p(xq8), nb)


def vec_dot_q4_0_q8_0_avx2(ws, wq, xq8, nb):
    return lib().oracle_vec_dot_q4_0_q8_0_avx2(_p(ws), _p(wq), _p(xq8), nb)


def matvec_q4_0_q8_0_avx2(ws, wq, xq8, rows, cols, threads=1):
    out = np.empty(rows, np.float32)
    lib().oracle_matvec_q4_0_q8_0_avx2_mt(_p(ws), _p(wq), _p(xq8), rows, cols, _p(out), threads)
    return out


def matvec_q4_0_q8_0_scalar(ws, wq, xq8, rows, cols):
    out = np.empty(rows, np.float32)
    lib().oracle_matvec_q4_0_q8_0_scalar(_p(ws), _p(wq), _p(xq8), rows, cols, _p(out))
    return out


def block_sums_q4_0_q8_0(ws, wq, xq8, rows, cols):
    out = np.empty(rows * (cols // 32), np.int32)
    lib().oracle_block_sums_q4_0_q8_0(_p(ws), _p(wq), _p(xq8), rows, cols, _p(out))
    return out


def gemm_q4_0_f16_scalar_reference(scales_f16, quants, x_f16, m, k, n):
    out = np.empty(n * m, np.uint16)
    lib().oracle_gemm_q4_0_f16_scalar_reference(_p(scales_f16), _p(quants), _p(x_f16), m, k, n,
                                                _p(out))
    return out


def gemm_q4_0_f16_f32out(scales_f16, quants, x_f16, m, k, n, threads=1):
    out = np.empty(n * m, np.float32)
    lib().oracle_gemm_q4_0_f16_scalar_f32out(_p(scales_f16), _p(quants), _p(x_f16), m, k, n,
                                             _p(out), threads)
    return out


def cpu_prefill_projection(ws, wq, x_f32, m, k, n, threads=1):
    out = np.empty(n * m, np.float32)
    lib().oracle_cpu_prefill_projection(_p(ws), _p(wq), _p(x_f32), m, k, n, _p(out), threads)
    return out


def rmsnorm_scalar(x, w, eps):
    x = np.ascontiguousarray(x, np.float32)
    w = np.ascontiguousarray(w, np.float32)
    out = np.empty_like(x)
    lib().oracle_rmsnorm_scalar(_p(x), _p(w), x.size, eps, _p(out))
    return out


def rmsnorm_avx2(x, w, eps):
    x = np.ascontiguousarray(x, np.float32)
    w = np.ascontiguousarray(w, np.float32)
    out = np.empty_like(x)
    lib().oracle_rmsnorm_avx2(_p(x), _p(w), x.size, eps, _p(out))
    return out


def rmsnorm_gemma_avx2(x, w, eps):
    """rmsnorm_gemma_avx2 (crates/sulimo-cpu/src/avx2.rs:236-268): (x * scale) * (1 + w)."""
    x = np.ascontiguousarray(x, np.float32)
    w = np.ascontiguousarray(w, np.float32)
    out = np.empty_like(x)
    lib().oracle_rmsnorm_gemma_avx2(_p(x), _p(w), x.size, eps, _p(out))
    return out


def geglu(gate, up):
    """geglu_scalar (crates/sulimo-cpu/src/scalar.rs:77-89)."""
    gate = np.ascontiguousarray(gate, np.float32)
    up = np.ascontiguousarray(up, np.float32)
    out = np.empty_like(gate)
    lib().oracle_geglu_scalar(_p(gate), _p(up), _p(out), gate.size)
    return out


def logit_softcap(v, cap):
    """logit_softcap_scalar (crates/sulimo-cpu/src/scalar.rs:63-71), on a copy."""
    v = np.array(v, dtype=np.float32, copy=True)
    lib().oracle_logit_softcap_scalar(_p(v), v.size, cap)
    return v


def rope_head(vec, pos, rope_dim, freq_base, mode):
    v = np.array(vec, dtype=np.float32, copy=True)
    lib().oracle_rope_head_scalar(_p(v), pos, rope_dim, freq_base, mode)
    return v


def softmax(x):
    v = np.array(x, dtype=np.float32, copy=True)
    lib().oracle_softmax_scalar(_p(v), v.size)
    return v


def swiglu(gate, up):
    gate = np.ascontiguousarray(gate, np.float32)
    up = np.ascontiguousarray(up, np.float32)
    out = np.empty_like(gate)
    lib().oracle_swiglu_scalar(_p(gate), _p(up), _p(out), gate.size)
    return out


def causal_gqa_decode(q, k_ring, v_ring, capacity, context_len, head_count, head_count_kv,
                      head_dim, softcap=0.0):
    q = np.ascontiguousarray(q, np.float32)
    k_ring = np.ascontiguousarray(k_ring, np.uint8)
    v_ring = np.ascontiguousarray(v_ring, np.uint8)
    scores = np.empty(max(context_len, 1), np.float32)
    out = np.empty(head_count * head_dim, np.float32)
    lib().oracle_causal_gqa_decode(_p(q), _p(k_ring), _p(v_ring), capacity, context_len,
                                   head_count, head_count_kv, head_dim, _p(scores), _p(out),
                                   softcap)
    return out


# ---- forward_token (crates/sulimo-engine/src/forward_pass.rs:190-417) -----------------------
class _OracleLayer(C.Structure):
    _fields_ = [(n, C.c_void_p) for n in (
        "attn_norm", "ffn_norm", "bq", "bk", "bv", "wq_s", "wq_q", "wk_s", "wk_q", "wv_s", "wv_q",
        "wo_s", "wo_q", "wg_s", "wg_q", "wu_s", "wu_q", "wd_s", "wd_q", "k_ring", "v_ring",
        "post_attn_norm", "post_ffn_norm")]


class _OracleModel(C.Structure):
    _fields_ = [("n_layers", C.c_int), ("embd", C.c_int), ("ffn", C.c_int),
                ("head_count", C.c_int), ("head_count_kv", C.c_int), ("head_dim", C.c_int),
                ("vocab", C.c_int), ("rope_dim", C.c_int), ("rope_mode", C.c_int),
                ("eps", C.c_float), ("rope_base", C.c_float), ("attn_softcap", C.c_float),
                ("kv_capacity", C.c_size_t), ("tok_s", C.c_void_p), ("tok_q", C.c_void_p),
                ("out_s", C.c_void_p), ("out_q", C.c_void_p), ("out_norm", C.c_void_p),
                ("layers", C.POINTER(_OracleLayer)), ("arch", C.c_int),
                ("final_softcap", C.c_float)]


class OracleModel:
    """A synthetic model held as numpy arrays for oracle_forward_token.  `w` is the dict made by
    sulimo_b200.synthetic.make_model_numpy; the K/V rings live here and advance with every
    forward_token call."""

    def __init__(self, w):
        self.w = w
        cfg = w["cfg"]
        self.cfg = cfg
        kv_bytes = cfg["kv_capacity"] * cfg["head_count_kv"] * cfg["head_dim"] // 32 * 34
        self.rings = [(np.zeros(kv_bytes, np.uint8), np.zeros(kv_bytes, np.uint8))
                      for _ in range(cfg["n_layers"])]
        layers = (_OracleLayer * cfg["n_layers"])()
        for i, (L, (kr, vr)) in enumerate(zip(w["layers"], self.rings)):
            ent = layers[i]
            for name in ("attn_norm", "ffn_norm", "bq", "bk", "bv", "post_attn_norm",
                         "post_ffn_norm"):
                setattr(ent, name, L[name].ctypes.data if L.get(name) is not None else None)
            for name in ("wq", "wk", "wv", "wo", "wg", "wu", "wd"):
                setattr(ent, name + "_s", L[name][0].ctypes.data)
                setattr(ent, name + "_q", L[name][1].ctypes.data)
            ent.k_ring, ent.v_ring = kr.ctypes.data, vr.ctypes.data
        self.layers = layers
        m = _OracleModel()
        for k in ("n_layers", "embd", "ffn", "head_count", "head_count_kv", "head_dim", "vocab",
                  "rope_dim", "rope_mode", "eps", "rope_base", "attn_softcap", "kv_capacity"):
            setattr(m, k, cfg[k])
        m.tok_s, m.tok_q = w["tok"][0].ctypes.data, w["tok"][1].ctypes.data
        m.out_s, m.out_q = w["out"][0].ctypes.data, w["out"][1].ctypes.data
        m.out_norm = w["out_norm"].ctypes.data
        m.layers = layers
        m.arch = cfg.get("arch", 0)
        m.final_softcap = cfg.get("final_softcap", 0.0)
        self.m = m

    def forward_token(self, token, pos):
        out = np.empty(self.cfg["vocab"], np.float32)
        lib().oracle_forward_token(C.byref(self.m), C.c_uint32(token), C.c_size_t(pos),
                                   out.ctypes.data_as(C.POINTER(C.c_float)))
        return out

    def embed_f16(self, tokens):
        """lookup_token_embedding_f16 per token (crates/sulimo-engine/src/scheduler.rs:329-374):
        the f16 rows the engine writes into the prefill ubatch's x."""
        E = self.cfg["embd"]
        return np.concatenate([lookup_token_embedding_f16(self.w["tok"][0], self.w["tok"][1], E,
                                                          int(t)) for t in tokens])

    def prefill_ubatch(self, tokens, start_pos, threads=1, x_f16=None):
        """oracle_prefill_ubatch (execute_prefill_ubatch, crates/sulimo-ocl/src/prefill.rs:337-566)
        for `tokens` at positions start_pos..: returns (last-token fp32 logits, the f16 residual
        stream [n][embd]).  The K/V rings of this model advance."""
        x = self.embed_f16(tokens) if x_f16 is None else np.array(x_f16, np.uint16, copy=True)
        logits = np.empty(self.cfg["vocab"], np.float32)
        st = lib().oracle_prefill_ubatch(C.byref(self.m), _p(x), start_pos, len(tokens),
                                         _p(logits), threads)
        assert st == 0, "oracle_prefill_ubatch rejected its arguments"
        return logits, x.reshape(len(tokens), -1)

    def prefill_ubatch_f32(self, tokens, start_pos, threads=1, x_f16=None):
        """oracle_prefill_ubatch_f32: the reference prefill test's CPU oracle
        (crates/sulimo-ocl/tests/test_prefill.rs:583-800), fp32 residual; returns the last
        token's logits.  The K/V rings of this model advance."""
        x = self.embed_f16(tokens) if x_f16 is None else np.ascontiguousarray(x_f16, np.uint16)
        n = x.size // self.cfg["embd"]
        logits = np.empty(self.cfg["vocab"], np.float32)
        st = lib().oracle_prefill_ubatch_f32(C.byref(self.m), _p(x), start_pos, n, _p(logits),
                                             threads)
        assert st == 0, "oracle_prefill_ubatch_f32 rejected its arguments"
        return logits


def matvec_dense(w, x, rows, cols, kind="f32", avx2=True):
    """matvec_f32/f16 (avx2.rs:259-331 when avx2, else scalar.rs:228-251): w [rows][cols] f32 or
    f16 bits, x [cols] f32 -> [rows] f32."""
    x = np.ascontiguousarray(x, np.float32)
    w = np.ascontiguousarray(w, np.float32 if kind == "f32" else np.uint16)
    out = np.empty(rows, np.float32)
    fn = f"oracle_matvec_{kind}_{'avx2' if avx2 else 'scalar'}"
    getattr(lib(), fn)(_p(w), _p(x), rows, cols, _p(out))
    return out


def _f16_buf(a):
    return np.array(a, dtype=np.uint16, copy=True)


def rmsnorm_f16(x_f16, w, eps, D):
    x = np.ascontiguousarray(x_f16, np.uint16)
    out = np.empty_like(x)
    lib().oracle_rmsnorm_f16(_p(x), _p(np.ascontiguousarray(w, np.float32)), _p(out), D, eps,
                             x.size // D)
    return out


def rope_f16(vec_f16, head_count, head_dim, rope_dim, base, mode, start_pos):
    v = _f16_buf(vec_f16)
    lib().oracle_rope_f16(_p(v), head_count, head_dim, rope_dim, base, mode, start_pos,
                          v.size // (head_count * head_dim))
    return v


def attention_prefill_f16(q_f16, k_ring, v_ring, start_pos, capacity, head_count, head_count_kv,
                          head_dim):
    q = np.ascontiguousarray(q_f16, np.uint16)
    out = np.empty_like(q)
    lib().oracle_attention_prefill_f16(_p(q), _p(np.ascontiguousarray(k_ring, np.uint8)),
                                       _p(np.ascontiguousarray(v_ring, np.uint8)), _p(out),
                                       start_pos, capacity, head_count, head_count_kv, head_dim,
                                       q.size // (head_count * head_dim))
    return out


def silu_mul_f16(gate_f16, up_f16):
    g = np.ascontiguousarray(gate_f16, np.uint16)
    u = np.ascontiguousarray(up_f16, np.uint16)
    out = np.empty_like(g)
    lib().oracle_silu_mul_f16(_p(g), _p(u), _p(out), g.size)
    return out


def add_f16(a_f16, b_f16):
    a = _f16_buf(a_f16)
    lib().oracle_add_f16(_p(a), _p(np.ascontiguousarray(b_f16, np.uint16)), a.size)
    return a
