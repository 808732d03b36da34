"""Seeded synthetic models with the layer structure of the reference's Llama / Qwen2 / Gemma 2 decode path
(no checkpoints are available offline).  Distributions follow the measurement plan:
Q4_0 weights d = f16(|N(0,1)|*0.02) with nibbles uniform in 0..15 (SoA layout), norms
1 + 0.1*N(0,1) (Gemma 2 stores w with the norm weighting 1 + w, so w = 0.1*N(0,1)), QKV biases
N(0,0.02) where the architecture has them.

`make_model_numpy` builds small models for the parity tests (numpy, fed to both the oracle
and the GPU); `make_model_torch` builds full-size ones directly on the GPU for the benchmark.
"""
import numpy as np

LLAMA_3B = dict(n_layers=28, embd=3072, ffn=8192, head_count=24, head_count_kv=8, head_dim=128,
                vocab=128256, rope_dim=128, rope_mode=0, eps=1e-5, rope_base=500000.0,
                attn_softcap=0.0, bias=False)
# Gemma 2 structure (forward_pass.rs:190-417 with arch = Gemma2): Neox RoPE, (1 + w) norms,
# post-attention / post-FFN norms, GeGLU, attention and final logit soft-capping.
GEMMA2_2B = dict(n_layers=26, embd=2304, ffn=9216, head_count=8, head_count_kv=4, head_dim=256,
                 vocab=256000, rope_dim=256, rope_mode=1, eps=1e-6, rope_base=10000.0,
                 attn_softcap=50.0, bias=False, arch=1, final_softcap=30.0)
QWEN_1_5B = dict(n_layers=28, embd=1536, ffn=8960, head_count=12, head_count_kv=2, head_dim=128,
                 vocab=151936, rope_dim=128, rope_mode=1, eps=1e-6, rope_base=1000000.0,
                 attn_softcap=0.0, bias=True)

_MATS = ("wq", "wk", "wv", "wo", "wg", "wu", "wd")


def mat_shapes(cfg):
    E, F = cfg["embd"], cfg["ffn"]
    qd = cfg["head_count"] * cfg["head_dim"]
    kvd = cfg["head_count_kv"] * cfg["head_dim"]
    return dict(wq=(qd, E), wk=(kvd, E), wv=(kvd, E), wo=(E, qd), wg=(F, E), wu=(F, E),
                wd=(E, F))


def _q4_np(rng, rows, cols):
    nb = rows * cols // 32
    d = (np.abs(rng.standard_normal(nb, dtype=np.float32)) * np.float32(0.02)).astype(np.float16)
    return d.view(np.uint16).copy(), rng.integers(0, 256, nb * 16, dtype=np.uint8)


def make_model_numpy(cfg, seed=0, kv_capacity=64):
    """Small model as numpy arrays: {"cfg", "tok", "out", "out_norm", "layers": [...]}."""
    cfg = dict(cfg, kv_capacity=kv_capacity)
    gemma = cfg.get("arch", 0) == 1
    rng = np.random.default_rng(seed)
    E = cfg["embd"]
    qd = cfg["head_count"] * cfg["head_dim"]
    kvd = cfg["head_count_kv"] * cfg["head_dim"]
    shapes = mat_shapes(cfg)
    tok = _q4_np(rng, cfg["vocab"], E)
    layers = []
    for _ in range(cfg["n_layers"]):
        L = {name: _q4_np(rng, *shapes[name]) for name in _MATS}
        L["attn_norm"] = (1.0 + 0.1 * rng.standard_normal(E)).astype(np.float32)
        L["ffn_norm"] = (1.0 + 0.1 * rng.standard_normal(E)).astype(np.float32)
        if cfg["bias"]:
            L["bq"] = (0.02 * rng.standard_normal(qd)).astype(np.float32)
            L["bk"] = (0.02 * rng.standard_normal(kvd)).astype(np.float32)
            L["bv"] = (0.02 * rng.standard_normal(kvd)).astype(np.float32)
        else:
            L["bq"] = L["bk"] = L["bv"] = None
        if gemma:
            L["attn_norm"] = (L["attn_norm"] - 1.0).astype(np.float32)
            L["ffn_norm"] = (L["ffn_norm"] - 1.0).astype(np.float32)
            L["post_attn_norm"] = (0.1 * rng.standard_normal(E)).astype(np.float32)
            L["post_ffn_norm"] = (0.1 * rng.standard_normal(E)).astype(np.float32)
        layers.append(L)
    out_norm = (1.0 + 0.1 * rng.standard_normal(E)).astype(np.float32)
    if gemma:
        out_norm = (out_norm - 1.0).astype(np.float32)
    return dict(cfg=cfg, tok=tok, out=tok, out_norm=out_norm, layers=layers)


def to_device(w):
    """numpy model -> the same model as CUDA torch tensors (scales as int16 bit patterns)."""
    import torch

    def t(a):
        if a is None:
            return None
        if a.dtype == np.uint16:
            a = a.view(np.int16)
        return torch.from_numpy(np.ascontiguousarray(a)).cuda()

    layers = []
    for L in w["layers"]:
        D = {name: (t(L[name][0]), t(L[name][1])) for name in _MATS}
        for name in ("attn_norm", "ffn_norm", "bq", "bk", "bv"):
            D[name] = t(L[name])
        for name in ("post_attn_norm", "post_ffn_norm"):
            D[name] = t(L.get(name))
        layers.append(D)
    tok = (t(w["tok"][0]), t(w["tok"][1]))
    return dict(cfg=w["cfg"], tok=tok, out=tok, out_norm=t(w["out_norm"]), layers=layers)


def make_model_torch(cfg, seed=0, kv_capacity=4096):
    """Full-size model generated on the GPU (same distributions, torch's RNG)."""
    import torch
    cfg = dict(cfg, kv_capacity=kv_capacity)
    g = torch.Generator(device="cuda")
    g.manual_seed(seed)
    E = cfg["embd"]
    qd = cfg["head_count"] * cfg["head_dim"]
    kvd = cfg["head_count_kv"] * cfg["head_dim"]
    shapes = mat_shapes(cfg)

    def q4(rows, cols):
        nb = rows * cols // 32
        d = (torch.randn(nb, device="cuda", generator=g).abs() * 0.02).half().view(torch.int16)
        q = torch.randint(0, 256, (nb * 16,), device="cuda", dtype=torch.uint8, generator=g)
        return d, q

    def vec(n, mean, std):
        return mean + std * torch.randn(n, device="cuda", generator=g)

    tok = q4(cfg["vocab"], E)
    layers = []
    for _ in range(cfg["n_layers"]):
        L = {name: q4(*shapes[name]) for name in _MATS}
        L["attn_norm"], L["ffn_norm"] = vec(E, 1.0, 0.1), vec(E, 1.0, 0.1)
        if cfg["bias"]:
            L["bq"], L["bk"], L["bv"] = vec(qd, 0.0, 0.02), vec(kvd, 0.0, 0.02), vec(kvd, 0.0, 0.02)
        else:
            L["bq"] = L["bk"] = L["bv"] = None
        if cfg.get("arch", 0) == 1:
            L["attn_norm"], L["ffn_norm"] = L["attn_norm"] - 1.0, L["ffn_norm"] - 1.0
            L["post_attn_norm"], L["post_ffn_norm"] = vec(E, 0.0, 0.1), vec(E, 0.0, 0.1)
        layers.append(L)
    out_norm = vec(E, 1.0, 0.1)
    if cfg.get("arch", 0) == 1:
        out_norm = out_norm - 1.0
    return dict(cfg=cfg, tok=tok, out=tok, out_norm=out_norm, layers=layers)


def weight_bytes(cfg):
    """Q4_0 weight bytes read per decode step (layers + the vocab projection)."""
    per = sum(r * c // 32 * 18 for r, c in mat_shapes(cfg).values())
    return cfg["n_layers"] * per + cfg["vocab"] * cfg["embd"] // 32 * 18
