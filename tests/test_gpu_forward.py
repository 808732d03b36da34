"""GPU parity of a whole decode position (sulimo_cuda_forward_token) against the oracle's
restatement of forward_token (crates/sulimo-engine/src/forward_pass.rs:190-417) on small seeded
models of the supported architectures: Qwen2 (Neox RoPE, QKV biases), Llama (Norm RoPE) and
Gemma 2 (embedding scale, (1 + w) norms, post-attention / post-FFN norms, GeGLU, attention and
final logit soft-capping).

Tolerance: the GEMVs are bit-exact with the AVX2 kernel, but RMSNorm's sum of squares is a tree
(the reference adds eight AVX2 lanes sequentially) and RoPE / SiLU / softmax use CUDA's powf,
sinf, cosf, expf, so activations differ by float rounding; an occasional Q8_0 re-rounding of an
activation follows.  Bars: logits rel-L2 <= 5e-3 at every position, the same greedy token
wherever the oracle's top-2 logits are 1e-3 (relative) apart, and the K/V rings within
rel-L2 1e-2 after dequantization."""
import numpy as np
import pytest

import oracle.ffi as O
from helpers import rel_l2

pytestmark = pytest.mark.gpu

QWEN_SMALL = dict(n_layers=2, embd=256, ffn=512, head_count=4, head_count_kv=2, head_dim=64,
                  vocab=512, rope_dim=64, rope_mode=1, eps=1e-6, rope_base=1e6, attn_softcap=0.0,
                  bias=True)
GEMMA2_SMALL = dict(n_layers=2, embd=256, ffn=512, head_count=4, head_count_kv=2, head_dim=128,
                    vocab=640, rope_dim=128, rope_mode=1, eps=1e-6, rope_base=1e4,
                    attn_softcap=50.0, bias=False, arch=1, final_softcap=30.0)
LLAMA_SMALL = dict(n_layers=3, embd=384, ffn=1024, head_count=6, head_count_kv=2, head_dim=128,
                   vocab=1000, rope_dim=128, rope_mode=0, eps=1e-5, rope_base=5e5,
                   attn_softcap=0.0, bias=False)


def deq_ring(ring_u8):
    nb = ring_u8.size // 34
    return O.dequantize_q8_0_to_f32(ring_u8, nb)


def check_step(got, ref, where):
    assert np.isfinite(got).all(), where
    assert rel_l2(got, ref) <= 5e-3, (where, rel_l2(got, ref))
    top = np.argsort(ref)[-2:]
    margin = (ref[top[1]] - ref[top[0]]) / max(abs(ref[top[1]]), 1e-6)
    if margin > 1e-3:
        assert int(np.argmax(got)) == int(top[1]), where


@pytest.mark.parametrize("cfg", [QWEN_SMALL, LLAMA_SMALL, GEMMA2_SMALL],
                         ids=["qwen2", "llama", "gemma2"])
def test_forward_token_matches_oracle(ctx, cfg):
    import torch
    from sulimo_b200.model import DecodeModel
    from sulimo_b200.synthetic import make_model_numpy, to_device
    w = make_model_numpy(cfg, seed=7, kv_capacity=32)
    om = O.OracleModel(w)
    dm = DecodeModel(ctx, to_device(w), batch=1)
    toks = [3, 77, 120, 5, 400, 9, 250, 31, 8, 100]
    for pos, t in enumerate(toks):
        ref = om.forward_token(t, pos)
        tk = torch.tensor([t], dtype=torch.int32, device="cuda")
        got = dm.forward_token(tk, pos).cpu().numpy()
        ctx.finish()
        check_step(got, ref, f"pos {pos}")
    for l in range(cfg["n_layers"]):
        for which, idx in (("k", 0), ("v", 1)):
            g = deq_ring(dm.rings[l][idx].cpu().numpy())
            r = deq_ring(om.rings[l][idx])
            assert rel_l2(g, r) <= 1e-2, (l, which)


@pytest.mark.parametrize("cfg", [QWEN_SMALL, GEMMA2_SMALL], ids=["qwen2", "gemma2"])
def test_forward_token_batch_of_sequences(ctx, cfg):
    """Three sequences at once: each matches its own oracle run; greedy argmax on the device."""
    import torch
    from sulimo_b200.model import DecodeModel
    from sulimo_b200.synthetic import make_model_numpy, to_device
    w = make_model_numpy(cfg, seed=9, kv_capacity=16)
    oms = [O.OracleModel(w) for _ in range(3)]
    dm = DecodeModel(ctx, to_device(w), batch=3)
    toks = np.array([[1, 2, 3], [50, 60, 70], [500, 7, 64], [11, 12, 13]], np.int32)
    for pos in range(toks.shape[0]):
        tk = torch.from_numpy(toks[pos]).cuda()
        got = dm.forward_token(tk, pos).cpu().numpy().reshape(3, -1)
        nxt = dm.greedy().cpu().numpy()
        ctx.finish()
        for s in range(3):
            ref = oms[s].forward_token(int(toks[pos, s]), pos)
            check_step(got[s], ref, f"seq {s} pos {pos}")
            assert nxt[s] == int(np.argmax(got[s]))


def test_forward_token_rejects_context_beyond_ring(ctx):
    import torch
    import sulimo_b200 as sb
    from sulimo_b200.model import DecodeModel
    from sulimo_b200.synthetic import make_model_numpy, to_device
    w = make_model_numpy(QWEN_SMALL, seed=1, kv_capacity=8)
    dm = DecodeModel(ctx, to_device(w), batch=1)
    tk = torch.zeros(1, dtype=torch.int32, device="cuda")
    with pytest.raises(sb.SulimoError) as e:
        dm.forward_token(tk, 8)   # context 9 > 8 ring slots
    assert e.value.kind == "InvalidArgument"


def test_gemma2_prefill_ubatch_rejected(ctx):
    """The reference's GPU ubatch (prefill.rs:337-566) has no Gemma 2 steps; this one refuses a
    Gemma 2 model instead of computing something else, and forward_token serves it."""
    import torch
    import sulimo_b200 as sb
    from sulimo_b200.model import DecodeModel
    from sulimo_b200.synthetic import make_model_numpy, to_device
    w = make_model_numpy(GEMMA2_SMALL, seed=3, kv_capacity=16)
    dm = DecodeModel(ctx, to_device(w), batch=1)
    with pytest.raises(sb.SulimoError) as e:
        dm.prefill(torch.tensor([1, 2, 3], dtype=torch.int32, device="cuda"))
    from sulimo_b200 import capi
    assert e.value.status == capi.EINVAL
