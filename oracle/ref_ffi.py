"""numpy bindings of oracle/_ref/libsulimo_ref_ocl.so: the reference's own OpenCL C kernels
(kernels/gemm_q4_0.cl, kernels/prefill.cl) compiled unchanged for the host (oracle/ref_build.py,
oracle/ref_ocl_shim.cpp).

TEST INFRASTRUCTURE ONLY: used by tests/ and tests/golden/make_ref_ocl_golden.py to pin the C
restatement (oracle.ffi) to values the reference's code produces.  `available()` is False when
the library is neither built nor buildable (no reference checkout); callers skip then.
"""
import ctypes as C

import numpy as np

from . import ref_build as _build
from .ffi import OracleModel  # noqa: F401  (the same model struct drives both)

_lib = None


def available():
    return _build.available()


def lib():
    global _lib
    if _lib is None:
        path = _build.build()
        if path is None:
            raise RuntimeError("oracle/_ref is not built and no reference checkout is present")
        L = C.CDLL(path)
        vp, i32, f32, sz = C.c_void_p, C.c_int, C.c_float, C.c_size_t
        sig = {
            "ref_gemm_q4_0_f16_portable": (None, [vp, vp, vp, vp, i32, i32, i32, i32]),
            "ref_rmsnorm_f16_f32w": (None, [vp, vp, vp, i32, f32, i32]),
            "ref_rope_f16": (None, [vp, i32, i32, i32, f32, i32, i32, i32]),
            "ref_kv_store_q8_0": (None, [vp, vp, i32, i32, i32, i32]),
            "ref_causal_gqa_attention_prefill": (None, [vp, vp, vp, vp, i32, i32, i32, i32, i32,
                                                        i32, i32]),
            "ref_silu_mul_f16": (None, [vp, vp, vp, i32]),
            "ref_add_f16": (None, [vp, vp, i32]),
            "ref_logits_f16_output": (None, [vp, vp, vp, vp, i32, i32, i32, i32]),
            "ref_execute_prefill_ubatch": (i32, [vp, vp, sz, sz, vp, i32]),
        }
        for name, (res, args) in sig.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


def _p(a):
    assert a.flags["C_CONTIGUOUS"]
    return a.ctypes.data_as(C.c_void_p)


def _u16(a):
    return np.ascontiguousarray(a, dtype=np.uint16)


def gemm_q4_0_f16_portable(scales, quants, x_f16, m, k, n, threads=1):
    out = np.empty(n * m, np.uint16)
    lib().ref_gemm_q4_0_f16_portable(_p(_u16(scales)), _p(np.ascontiguousarray(quants, np.uint8)),
                                     _p(_u16(x_f16)), _p(out), m, k, n, threads)
    return out


def rmsnorm_f16_f32w(x_f16, w, eps, D):
    x = _u16(x_f16)
    out = np.empty_like(x)
    lib().ref_rmsnorm_f16_f32w(_p(x), _p(np.ascontiguousarray(w, np.float32)), _p(out), D, eps,
                               x.size // D)
    return out


def rope_f16(vec_f16, head_count, head_dim, rope_dim, base, mode, start_pos):
    v = np.array(vec_f16, np.uint16, copy=True)
    lib().ref_rope_f16(_p(v), head_count, head_dim, rope_dim, base, mode, start_pos,
                       v.size // (head_count * head_dim))
    return v


def kv_store_q8_0(act_f16, kv, start_pos, capacity, blocks_per_pos, n):
    assert kv.flags["C_CONTIGUOUS"] and kv.dtype == np.uint8
    lib().ref_kv_store_q8_0(_p(_u16(act_f16)), _p(kv), start_pos, capacity, blocks_per_pos, n)


def causal_gqa_attention_prefill(q_f16, k_ring, v_ring, start_pos, capacity, head_count,
                                 head_count_kv, head_dim, threads=1):
    q = _u16(q_f16)
    out = np.empty_like(q)
    lib().ref_causal_gqa_attention_prefill(
        _p(q), _p(np.ascontiguousarray(k_ring, np.uint8)), _p(np.ascontiguousarray(v_ring, np.uint8)),
        _p(out), start_pos, capacity, head_count, head_count_kv, head_dim,
        q.size // (head_count * head_dim), threads)
    return out


def silu_mul_f16(gate_f16, up_f16):
    g = _u16(gate_f16)
    out = np.empty_like(g)
    lib().ref_silu_mul_f16(_p(g), _p(_u16(up_f16)), _p(out), g.size)
    return out


def add_f16(a_f16, b_f16):
    a = np.array(a_f16, np.uint16, copy=True)
    lib().ref_add_f16(_p(a), _p(_u16(b_f16)), a.size)
    return a


def logits_f16_output(x_all_f16, scales, quants, M, K, token_idx, threads=1):
    out = np.empty(M, np.float32)
    lib().ref_logits_f16_output(_p(_u16(x_all_f16)), _p(_u16(scales)),
                                _p(np.ascontiguousarray(quants, np.uint8)), _p(out), M, K,
                                token_idx, threads)
    return out


def execute_prefill_ubatch(om, tokens, start_pos, threads=1, x_f16=None):
    """The reference's execute_prefill_ubatch over its own kernels, for an oracle.ffi.OracleModel
    (whose K/V rings advance): (last-token logits, f16 residual stream [n][embd])."""
    x = om.embed_f16(tokens) if x_f16 is None else np.array(x_f16, np.uint16, copy=True)
    logits = np.empty(om.cfg["vocab"], np.float32)
    st = lib().ref_execute_prefill_ubatch(C.byref(om.m), _p(x), start_pos, len(tokens),
                                          _p(logits), threads)
    assert st == 0
    return logits, x.reshape(len(tokens), -1)
