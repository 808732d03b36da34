"""GPU parity of the prefill path.

- The tensor-core causal prefill attention over the Q8_0 ring (causal_gqa_attention_prefill,
  kernels/prefill.cl:120-237) against the oracle's scalar causal attention of every token:
  q is f16 (as the reference's kernel takes it) and the Q8_0 scales are applied in fp32,
  rel-L2 <= 5e-3 per token.
- A whole prefill ubatch (execute_prefill_ubatch, crates/sulimo-ocl/src/prefill.rs:337-566)
  against both of the reference's definitions of it: the restatement of its GPU kernels
  (oracle_prefill_ubatch, bit-identical to the reference's own OpenCL C run on the host; every
  activation f16 between kernels, attention accumulated in f16) and the CPU oracle of its prefill
  test (oracle_prefill_ubatch_f32, test_prefill.rs:583-800; fp32 residual).  This path keeps the
  residual in fp32 and rounds each weight to f16 for the tensor cores.  Bars: last-token logits
  rel-L2 <= 5e-3, cosine >= 0.99 and the same greedy token (the reference test's own bars,
  test_prefill.rs:860-890); the first layer's K/V within one Q8_0 step (test_prefill.rs:826-850;
  the step of the larger scale, plus what the two scales' difference moves a code); every
  layer's dequantised K/V within rel-L2 1.5e-2.  Deeper layers cannot be held to one step: the
  reference's two definitions differ from each other by 4e-3..7e-3 rel-L2 and by more than a
  step in up to a few hundred elements of the second layer's K/V on these inputs (the
  reference's test passes its one-step bar only because its head_dim 16 holds no whole Q8_0
  block, so its attention reads nothing).  The reference's GPU ubatch applies no QKV bias;
  these models have none.
- The CPU prefill semantics (the reference prefills with forward_token token by token when no
  GPU ubatch runs, engine.rs:287-318) on a model with QKV biases: Q8_0 activations there against
  f16 here (relative step 1/254), so rel-L2 <= 4e-2, and a decode step continuing from both
  sides' rings."""
import numpy as np
import pytest

import oracle.ffi as O
import sulimo_b200 as sb
from gpu_util import dev, empty, host
from helpers import cosine, make_model_pattern_prefill, make_x_pattern_prefill, rel_l2

pytestmark = pytest.mark.gpu


def make_ring(rng, cap, hkv, hd):
    kv = rng.standard_normal((cap, hkv * hd)).astype(np.float32)
    return np.concatenate([O.quantize_f32_to_q8_0(r) for r in kv])


@pytest.mark.parametrize("n,start,H,Hkv,hd,cap", [
    (100, 0, 12, 2, 128, 128),    # Qwen geometry, first ubatch, ragged last tile
    (70, 130, 12, 2, 128, 256),   # second ubatch: earlier positions come from the ring
    (64, 0, 24, 8, 128, 64),      # Llama geometry, exactly one tile, full ring
    (33, 7, 8, 8, 64, 48),        # MHA, head_dim 64
    (300, 200, 12, 2, 128, 512),  # three 128-token tiles, eight 64-key chunks per tile
    (512, 1024, 12, 2, 128, 1536),  # config-3 sized ubatch late in the prompt: 24 chunks
    (257, 0, 4, 4, 64, 300),      # head_dim 64, a one-token last tile
])
def test_prefill_attention_matches_oracle(ctx, n, start, H, Hkv, hd, cap):
    import torch
    rng = np.random.default_rng(n + start)
    kr, vr = make_ring(rng, cap, Hkv, hd), make_ring(rng, cap, Hkv, hd)
    q = rng.standard_normal((n, H, hd)).astype(np.float32)
    out = empty(n * H * hd, torch.float16)
    sb.causal_gqa_attention_prefill(ctx, dev(q.ravel()), dev(kr), dev(vr), start, cap, n, H, Hkv,
                                    hd, out)
    ctx.finish()
    got = host(out).astype(np.float32).reshape(n, H, hd)
    for t in range(n):
        ref = O.causal_gqa_decode(q[t].ravel(), kr, vr, cap, start + t + 1, H, Hkv, hd)
        assert rel_l2(got[t].ravel(), ref.ravel()) <= 5e-3, t


def ring_scales(ring, nbytes):
    return O.f16_to_f32(ring[:nbytes].reshape(-1, 34)[:, :2].copy().view(np.uint16).ravel())


def check_ring(got_ring, ref_ring, nbytes, layer, where):
    """Dequantised K/V: rel-L2 <= 1.5e-2 in every layer; in the first layer every element within
    one Q8_0 step (test_prefill.rs:826-850: 1.05 * d + 1e-4, with d the larger of the two
    blocks' scales) plus 127 * |d_got - d_ref| (a code of 127 moved by the scale difference)."""
    g = O.dequantize_q8_0_to_f32(got_ring[:nbytes], nbytes // 34)
    r = O.dequantize_q8_0_to_f32(ref_ring[:nbytes], nbytes // 34)
    err = rel_l2(g, r)
    dg, dr = ring_scales(got_ring, nbytes), ring_scales(ref_ring, nbytes)
    bound = np.repeat(np.maximum(dg, dr) * 1.05 + 127 * np.abs(dg - dr), 32) + 1e-4
    bad = int((np.abs(g - r) > bound).sum())
    print(f"{where}: K/V rel-L2 {err:.2e}, {bad} of {g.size} beyond one step")
    assert err <= 1.5e-2, (where, err)
    if layer == 0:
        assert bad == 0, where


def check_ubatch_logits(got, ref, where, tol=5e-3):
    assert np.isfinite(got).all(), where
    err = rel_l2(got, ref)
    print(f"{where}: logits rel-L2 {err:.3e} cosine {cosine(got, ref):.7f}")
    assert err <= tol, (where, err)
    assert cosine(got, ref) >= 0.99, where
    top = np.argsort(ref)[-2:]
    if (ref[top[1]] - ref[top[0]]) / max(abs(ref[top[1]]), 1e-6) > 1e-3:
        assert int(np.argmax(got)) == int(top[1]), where


def test_prefill_ubatch_reference_test_data(ctx):
    """The model and prompt generators of test_prefill.rs:296-566 (pattern weights, norms and
    x = f16(((i % 17) - 8) * 0.15), 16 tokens, Llama RoPE base 1e4, eps 1e-5, ring 64) at
    head_dim 64 (the reference test's head_dim 16 is below one Q8_0 block per head, which makes
    its kernels read zero blocks), x supplied by the caller as execute_prefill_ubatch expects."""
    import torch
    from sulimo_b200.model import DecodeModel
    from sulimo_b200.synthetic import to_device
    w = make_model_pattern_prefill(dict(embd=256, ffn=512, head_count=4, head_count_kv=2,
                                        head_dim=64, rope_dim=64, vocab=64))
    om = O.OracleModel(w)
    dm = DecodeModel(ctx, to_device(w), batch=1)
    om32 = O.OracleModel(w)
    x0 = make_x_pattern_prefill(16, 256)
    ref, _ = om.prefill_ubatch(np.zeros(16, np.int32), 0, x_f16=x0)
    ref32 = om32.prefill_ubatch_f32(None, 0, x_f16=x0)
    got = host(dm.prefill(None, 0, x_f16=dev(x0)))
    ctx.finish()
    check_ubatch_logits(got, ref, "reference test data vs GPU-kernel oracle")
    check_ubatch_logits(got, ref32, "reference test data vs test CPU oracle")
    slot = 2 * 64 // 32 * 34
    for l in range(2):
        for idx in (0, 1):
            for o, tag in ((om, "f16"), (om32, "f32")):
                check_ring(host(dm.rings[l][idx]), o.rings[l][idx], 16 * slot, l,
                           f"layer {l} {'KV'[idx]} vs {tag} oracle")


QWEN_NOBIAS = dict(n_layers=2, embd=512, ffn=1024, head_count=4, head_count_kv=2, head_dim=128,
                   vocab=776, rope_dim=128, rope_mode=1, eps=1e-6, rope_base=1e6,
                   attn_softcap=0.0, bias=False)
LLAMA_NOBIAS = dict(n_layers=3, embd=384, ffn=1024, head_count=6, head_count_kv=2, head_dim=64,
                    vocab=1000, rope_dim=64, rope_mode=0, eps=1e-5, rope_base=5e5,
                    attn_softcap=0.0, bias=False)


@pytest.mark.parametrize("cfg,splits", [(QWEN_NOBIAS, [200, 57]), (LLAMA_NOBIAS, [64, 1, 31])],
                         ids=["qwen2-shape", "llama-shape"])
def test_prefill_ubatch_matches_prefill_oracle(ctx, cfg, splits):
    """Seeded models (benchmark distributions), several ubatches continuing the same rings, then
    one decode position from each side's own rings (forward_token on both)."""
    import torch
    from sulimo_b200.model import DecodeModel
    from sulimo_b200.synthetic import make_model_numpy, to_device
    w = make_model_numpy(cfg, seed=11, kv_capacity=512)
    om, om32 = O.OracleModel(w), O.OracleModel(w)
    dm = DecodeModel(ctx, to_device(w), batch=1)
    n_total = sum(splits)
    toks = np.random.default_rng(13).integers(0, cfg["vocab"], n_total + 1).astype(np.int32)
    start = 0
    for n in splits:
        ref, _ = om.prefill_ubatch(toks[start:start + n], start, threads=8)
        ref32 = om32.prefill_ubatch_f32(toks[start:start + n], start, threads=8)
        got = host(dm.prefill(torch.from_numpy(toks[start:start + n].copy()).cuda(), start))
        ctx.finish()
        start += n
        check_ubatch_logits(got, ref, f"ubatch ending at {start} vs GPU-kernel oracle")
        check_ubatch_logits(got, ref32, f"ubatch ending at {start} vs test CPU oracle")
    slot = cfg["head_count_kv"] * cfg["head_dim"] // 32 * 34
    for l in range(cfg["n_layers"]):
        for idx in (0, 1):
            for o, tag in ((om, "f16"), (om32, "f32")):
                check_ring(host(dm.rings[l][idx]), o.rings[l][idx], n_total * slot, l,
                           f"layer {l} {'KV'[idx]} vs {tag} oracle")
    ref = om.forward_token(int(toks[n_total]), n_total)
    got = dm.forward_token(torch.from_numpy(toks[n_total:n_total + 1].copy()).cuda(), n_total)
    ctx.finish()
    check_ubatch_logits(host(got)[:cfg["vocab"]], ref, "decode after prefill")


QWEN_SMALL = dict(n_layers=2, embd=256, ffn=512, head_count=4, head_count_kv=2, head_dim=64,
                  vocab=512, rope_dim=64, rope_mode=1, eps=1e-6, rope_base=1e6, attn_softcap=0.0,
                  bias=True)
LLAMA_SMALL = dict(n_layers=2, embd=384, ffn=1024, head_count=6, head_count_kv=2, head_dim=128,
                   vocab=1000, rope_dim=128, rope_mode=0, eps=1e-5, rope_base=5e5,
                   attn_softcap=0.0, bias=False)


def check_logits(got, ref, where):
    assert np.isfinite(got).all(), where
    assert rel_l2(got, ref) <= 4e-2, (where, rel_l2(got, ref))
    top = np.argsort(ref)[-2:]
    if (ref[top[1]] - ref[top[0]]) / max(abs(ref[top[1]]), 1e-6) > 5e-2:
        assert int(np.argmax(got)) == int(top[1]), where


# ragged for the prefill's fused projections: ffn 576 leaves the gated gate/up GEMM's last CTA
# pair half empty, embd 320 the o / down tiles ragged, q width 320 (not a multiple of 128) keeps
# q/k/v on separate GEMMs next to the fused o / down / gate-up paths
QWEN_RAGGED = dict(n_layers=2, embd=320, ffn=576, head_count=5, head_count_kv=1, head_dim=64,
                   vocab=304, rope_dim=64, rope_mode=1, eps=1e-6, rope_base=1e6, attn_softcap=0.0,
                   bias=True)


@pytest.mark.parametrize("cfg,splits", [(QWEN_SMALL, [37]), (LLAMA_SMALL, [20, 45]),
                                        (QWEN_RAGGED, [45, 70])],
                         ids=["qwen2-one-ubatch", "llama-two-ubatches", "ragged-two-ubatches"])
def test_prefill_ubatch_then_decode_matches_cpu_prefill(ctx, cfg, splits):
    import torch
    from sulimo_b200.model import DecodeModel
    from sulimo_b200.synthetic import make_model_numpy, to_device
    w = make_model_numpy(cfg, seed=3, kv_capacity=128)
    om = O.OracleModel(w)
    dm = DecodeModel(ctx, to_device(w), batch=1)
    n_total = sum(splits)
    toks = np.random.default_rng(5).integers(0, cfg["vocab"], n_total + 1).astype(np.int32)
    ref = None
    for p in range(n_total):
        ref = om.forward_token(int(toks[p]), p)
    start = 0
    got = None
    for n in splits:
        got = dm.prefill(torch.from_numpy(toks[start:start + n].copy()).cuda(), start)
        start += n
    ctx.finish()
    check_logits(host(got), ref, "prefill last token")
    slot = cfg["head_count_kv"] * cfg["head_dim"] // 32 * 34
    nbytes = n_total * slot   # positions 0 .. n_total-1 are ring slots 0 .. n_total-1
    for l in range(cfg["n_layers"]):
        for idx in (0, 1):
            g = O.dequantize_q8_0_to_f32(host(dm.rings[l][idx])[:nbytes], nbytes // 34)
            r = O.dequantize_q8_0_to_f32(om.rings[l][idx][:nbytes], nbytes // 34)
            assert rel_l2(g, r) <= 4e-2, (l, idx, rel_l2(g, r))
    # one decode step after the prefill, both sides continuing from their own rings
    ref = om.forward_token(int(toks[n_total]), n_total)
    got = dm.forward_token(torch.from_numpy(toks[n_total:n_total + 1].copy()).cuda(), n_total)
    ctx.finish()
    check_logits(host(got)[:cfg["vocab"]], ref, "decode after prefill")


def test_prefill_rejects_overflowing_ring(ctx):
    import torch
    from sulimo_b200.model import DecodeModel
    from sulimo_b200.synthetic import make_model_numpy, to_device
    w = make_model_numpy(QWEN_SMALL, seed=1, kv_capacity=16)
    dm = DecodeModel(ctx, to_device(w), batch=1)
    with pytest.raises(sb.SulimoError) as e:
        dm.prefill(torch.zeros(10, dtype=torch.int32, device="cuda"), start_pos=8)
    assert e.value.kind == "InvalidArgument"
