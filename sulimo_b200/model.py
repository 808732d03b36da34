"""Host mirror of the reference's decode loop over the C ABI: a model's device tensors, its
per-sequence Q8_0 K/V rings and the scratch of sulimo_cuda_forward_token
(crates/sulimo-engine/src/forward_pass.rs:190-417, ScratchBuffers :150-186, KvCache
crates/sulimo-core/src/kv_cache.rs:27-155).  `batch` independent sequences advance together.
"""
import ctypes as C

import sulimo_b200 as sb
from sulimo_b200 import capi

_MATS = ("wq", "wk", "wv", "wo", "wg", "wu", "wd")


class _LayerDesc(C.Structure):
    _fields_ = [(n, C.c_void_p) for n in (
        "attn_norm", "ffn_norm", "bq", "bk", "bv",
        "wq_scales", "wq_quants", "wk_scales", "wk_quants", "wv_scales", "wv_quants",
        "wo_scales", "wo_quants", "wg_scales", "wg_quants", "wu_scales", "wu_quants",
        "wd_scales", "wd_quants", "k_ring", "v_ring", "post_attn_norm", "post_ffn_norm")]


class _ModelDesc(C.Structure):
    _fields_ = [("n_layers", C.c_int), ("embd", C.c_int), ("ffn", C.c_int),
                ("head_count", C.c_int), ("head_count_kv", C.c_int), ("head_dim", C.c_int),
                ("vocab", C.c_int), ("rope_dim", C.c_int), ("rope_mode", C.c_int),
                ("eps", C.c_float), ("rope_base", C.c_float), ("attn_softcap", C.c_float),
                ("kv_capacity", C.c_size_t), ("kv_seq_stride", C.c_size_t),
                ("tok_scales", C.c_void_p), ("tok_quants", C.c_void_p),
                ("out_scales", C.c_void_p), ("out_quants", C.c_void_p),
                ("out_norm", C.c_void_p), ("layers", C.POINTER(_LayerDesc)),
                ("arch", C.c_int), ("final_softcap", C.c_float)]


def _p(t):
    return None if t is None else t.data_ptr()


class DecodeModel:
    """Device model + `batch` sequences' rings + scratch (all allocated once)."""

    def __init__(self, ctx, w, batch=1):
        import torch
        self.ctx, self.w, self.batch = ctx, w, batch
        cfg = self.cfg = w["cfg"]
        cap = cfg["kv_capacity"]
        slot = cfg["head_count_kv"] * cfg["head_dim"] // 32 * 34
        self.seq_stride = cap * slot
        self.rings = [(torch.zeros(batch * cap * slot, dtype=torch.uint8, device="cuda"),
                       torch.zeros(batch * cap * slot, dtype=torch.uint8, device="cuda"))
                      for _ in range(cfg["n_layers"])]
        layers = (_LayerDesc * cfg["n_layers"])()
        for i, (L, (kr, vr)) in enumerate(zip(w["layers"], self.rings)):
            e = layers[i]
            for name in ("attn_norm", "ffn_norm", "bq", "bk", "bv"):
                setattr(e, name, _p(L[name]))
            for name in ("post_attn_norm", "post_ffn_norm"):
                setattr(e, name, _p(L.get(name)))
            for name in _MATS:
                setattr(e, name + "_scales", _p(L[name][0]))
                setattr(e, name + "_quants", _p(L[name][1]))
            e.k_ring, e.v_ring = _p(kr), _p(vr)
        self.layers = layers
        d = _ModelDesc()
        for k in ("n_layers", "embd", "ffn", "head_count", "head_count_kv", "head_dim", "vocab",
                  "rope_dim", "rope_mode", "eps", "rope_base", "attn_softcap"):
            setattr(d, k, cfg[k])
        d.kv_capacity, d.kv_seq_stride = cap, self.seq_stride
        d.tok_scales, d.tok_quants = _p(w["tok"][0]), _p(w["tok"][1])
        d.out_scales, d.out_quants = _p(w["out"][0]), _p(w["out"][1])
        d.out_norm = _p(w["out_norm"])
        d.layers = layers
        d.arch = cfg.get("arch", 0)
        d.final_softcap = cfg.get("final_softcap", 0.0)
        self.desc = d
        self._desc_ptr = C.cast(C.pointer(d), C.c_void_p)
        nbytes = capi.load().sulimo_cuda_forward_scratch_bytes(self._desc_ptr, batch)
        if nbytes == 0:
            raise sb.SulimoError(capi.EINVAL, "sulimo_cuda_forward_scratch_bytes",
                                 "invalid model description")
        self.scratch = torch.empty(nbytes, dtype=torch.uint8, device="cuda")
        self.logits = torch.empty(batch * cfg["vocab"], dtype=torch.float32, device="cuda")
        self.next_tokens = torch.empty(batch, dtype=torch.int32, device="cuda")

    def forward_token(self, tokens, pos, logits=None):
        """logits [batch*vocab] for device int32 tokens[batch] at position pos."""
        out = self.logits if logits is None else logits
        capi.call("sulimo_cuda_forward_token", self.ctx.handle, self._desc_ptr, _p(tokens),
                  self.batch, pos, _p(out), _p(self.scratch), self.scratch.numel())
        return out

    def prefill(self, tokens, start_pos=0, logits=None, x_f16=None):
        """One prefill ubatch of len(tokens) tokens (device int32) of sequence 0 at positions
        start_pos..; returns the last token's logits [vocab] (execute_prefill_ubatch).  With
        x_f16 (device f16 [n][embd]) the caller supplies the embeddings instead of tokens."""
        import torch
        if x_f16 is not None:
            n = x_f16.numel() // self.cfg["embd"]
        else:
            n = tokens.numel()
        need = capi.load().sulimo_cuda_prefill_scratch_bytes(self._desc_ptr, n)
        if need == 0:
            raise sb.SulimoError(capi.EINVAL, "sulimo_cuda_prefill_scratch_bytes",
                                 "invalid model description")
        if getattr(self, "pscratch", None) is None or self.pscratch.numel() < need:
            self.pscratch = torch.empty(need, dtype=torch.uint8, device="cuda")
        out = self.logits[:self.cfg["vocab"]] if logits is None else logits
        if x_f16 is not None:
            capi.call("sulimo_cuda_prefill_ubatch_x", self.ctx.handle, self._desc_ptr, _p(x_f16),
                      n, start_pos, _p(out), _p(self.pscratch), self.pscratch.numel())
        else:
            capi.call("sulimo_cuda_prefill_ubatch", self.ctx.handle, self._desc_ptr, _p(tokens),
                      n, start_pos, _p(out), _p(self.pscratch), self.pscratch.numel())
        return out

    def greedy(self, logits=None):
        """Device int32 argmax of each sequence's logits (the greedy sampler's pick)."""
        lg = self.logits if logits is None else logits
        capi.call("sulimo_cuda_argmax_rows", self.ctx.handle, _p(lg), self.batch,
                  self.cfg["vocab"], _p(self.next_tokens))
        return self.next_tokens

    def ring_bytes(self, layer, which="k"):
        return self.rings[layer][0 if which == "k" else 1]
