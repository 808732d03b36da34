"""GPU parity: decode attention over the Q8_0 ring vs causal_gqa_decode_scalar_ext
(crates/sulimo-cpu/src/scalar.rs:287-359), relative L2 <= 2e-3 (fp32 sums reordered)."""
import numpy as np
import pytest

import oracle.ffi as O
import sulimo_b200 as sb
from gpu_util import dev, empty, host
from helpers import rel_l2

pytestmark = pytest.mark.gpu
TOL = 2e-3


def make_ring(rng, cap, fill, Hkv, hd, scale=1.0):
    """A ring whose first `fill` slots hold Q8_0 of N(0,1)*scale vectors (kv_cache.rs layout)."""
    kv_dim = Hkv * hd
    bpp = kv_dim // 32
    ring = np.zeros(cap * bpp * 34, np.uint8)
    for p in range(fill):
        O.kv_store_f32((rng.standard_normal(kv_dim) * scale).astype(np.float32), ring, p, cap, bpp)
    return ring


def run(ctx, q, kr, vr, cap, ctx_len, H, Hkv, hd, batch=1, seq_stride=0, softcap=0.0):
    import torch
    out = empty(batch * H * hd, torch.float32)
    sb.causal_gqa_decode(ctx, dev(q), dev(kr), dev(vr), cap, ctx_len, H, Hkv, hd, out,
                         batch=batch, seq_stride_bytes=seq_stride, softcap=softcap)
    ctx.finish()
    return host(out)


@pytest.mark.parametrize("H,Hkv,hd,cap,ctx_len", [
    (12, 2, 128, 4096, 1),       # Qwen2.5-1.5B geometry, first decode position
    (12, 2, 128, 4096, 7),
    (12, 2, 128, 4096, 300),
    (12, 2, 128, 4096, 2304),    # after a 2048-token prefill + 256 decode steps
    (24, 8, 128, 4096, 4096),    # Llama-3.2-3B geometry, full ring
    (4, 2, 64, 256, 200),
    (8, 8, 32, 64, 64),
    (6, 3, 96, 128, 77),
    (8, 1, 256, 512, 333),
])
def test_attn_decode_matches_oracle(ctx, H, Hkv, hd, cap, ctx_len):
    rng = np.random.default_rng(H * 1000 + ctx_len)
    kr = make_ring(rng, cap, min(ctx_len, cap), Hkv, hd)
    vr = make_ring(rng, cap, min(ctx_len, cap), Hkv, hd)
    q = rng.standard_normal(H * hd).astype(np.float32)
    got = run(ctx, q, kr, vr, cap, ctx_len, H, Hkv, hd)
    ref = O.causal_gqa_decode(q, kr, vr, cap, ctx_len, H, Hkv, hd)
    assert rel_l2(got, ref) <= TOL


def test_attn_decode_ring_wrap_reads_modulo(ctx):
    """context_len > capacity reads slot p % capacity, as key_ptr does (kv_cache.rs:114-119)."""
    rng = np.random.default_rng(3)
    H, Hkv, hd, cap, n = 4, 2, 64, 48, 100
    kr = make_ring(rng, cap, cap, Hkv, hd)
    vr = make_ring(rng, cap, cap, Hkv, hd)
    q = rng.standard_normal(H * hd).astype(np.float32)
    got = run(ctx, q, kr, vr, cap, n, H, Hkv, hd)
    ref = O.causal_gqa_decode(q, kr, vr, cap, n, H, Hkv, hd)
    assert rel_l2(got, ref) <= TOL


def test_attn_decode_sharp_softmax_and_softcap(ctx):
    rng = np.random.default_rng(4)
    H, Hkv, hd, cap, n = 8, 2, 128, 1024, 900
    kr = make_ring(rng, cap, n, Hkv, hd, scale=4.0)   # large scores: softmax close to one-hot
    vr = make_ring(rng, cap, n, Hkv, hd)
    q = (rng.standard_normal(H * hd) * 3).astype(np.float32)
    for cap_val in (0.0, 50.0):
        got = run(ctx, q, kr, vr, cap, n, H, Hkv, hd, softcap=cap_val)
        ref = O.causal_gqa_decode(q, kr, vr, cap, n, H, Hkv, hd, softcap=cap_val)
        assert rel_l2(got, ref) <= TOL


def test_attn_decode_batch_of_sequences(ctx):
    """Config-4 batching: independent sequences, each with its own ring seq_stride apart."""
    rng = np.random.default_rng(5)
    H, Hkv, hd, cap, n, B = 24, 8, 128, 1024, 1000, 3
    kv_dim = Hkv * hd
    ring_bytes = cap * kv_dim // 32 * 34
    krs = [make_ring(rng, cap, n, Hkv, hd) for _ in range(B)]
    vrs = [make_ring(rng, cap, n, Hkv, hd) for _ in range(B)]
    q = rng.standard_normal((B, H * hd)).astype(np.float32)
    got = run(ctx, q, np.concatenate(krs), np.concatenate(vrs), cap, n, H, Hkv, hd, batch=B,
              seq_stride=ring_bytes).reshape(B, -1)
    for b in range(B):
        ref = O.causal_gqa_decode(q[b], krs[b], vrs[b], cap, n, H, Hkv, hd)
        assert rel_l2(got[b], ref) <= TOL


def test_attn_decode_rejects_bad_geometry(ctx):
    import torch
    t = empty(1024, torch.float32)
    with pytest.raises(sb.SulimoError):
        sb.causal_gqa_decode(ctx, t, t, t, 16, 4, 12, 5, 128, t)   # 12 % 5 != 0
    with pytest.raises(sb.SulimoError):
        sb.causal_gqa_decode(ctx, t, t, t, 16, 4, 4, 2, 48, t)     # head_dim % 32 != 0
