"""sulimo_b200 — B200 (sm_100a) backend for Sulimo's quantized-matmul hot path.

The product is the C-ABI library libsulimo_cuda.so (include/sulimo_cuda.h) with hand-written
sm_100a kernels.  This module is a thin host mirror of the reference's backend operator surface
(crates/sulimo-ocl/src/{program,buffer,gemm,prefill,waiter}.rs and crates/sulimo-cpu/src/avx2.rs)
over that C ABI, used by the tests and bench.py.  Tensor arguments are CUDA torch tensors (or
raw device pointers as ints); torch only supplies device memory and streams.
"""
from . import capi
from .capi import (ACT_F16, ACT_F32, GGML_F16, GGML_F32, GGML_Q4_0, OUT_F16, OUT_F32,
                   SulimoError)

__all__ = [
    "CudaContext", "SulimoError", "gemm_q4_0_f16", "logits_final", "dispatch_matvec_q4_0_q8_0",
    "block_sums_q4_0_q8_0", "quantize_f32_to_q8_0", "kv_store_q8_0", "dequantize_q4_0_rows",
    "causal_gqa_decode", "causal_gqa_attention_prefill", "live_buffer_count", "unshard_rows", "OUT_F16", "OUT_F32", "ACT_F16",
    "ACT_F32", "GGML_F32", "GGML_F16", "GGML_Q4_0", "dispatch_matvec_f32", "dispatch_matvec_f16",
    "apply_matvec",
]


def _ptr(t):
    if t is None:
        return None
    if isinstance(t, int):
        return t
    if hasattr(t, "data_ptr"):
        if not t.is_cuda:
            raise ValueError("tensor arguments must live on the GPU")
        if not t.is_contiguous():
            raise ValueError("tensor arguments must be contiguous")
        return t.data_ptr()
    raise TypeError(f"expected a CUDA tensor or a device pointer, got {type(t)}")


class CudaContext:
    """One device + one stream (OclContext, crates/sulimo-ocl/src/program.rs:79-94)."""

    def __init__(self, device=0, stream=None):
        import ctypes as C
        h = C.c_void_p()
        capi.call("sulimo_cuda_ctx_create", device, C.byref(h))
        self.handle = h.value
        self.device = device
        if stream is not None:
            self.set_stream(stream)

    def set_stream(self, stream):
        """Launch on the caller's stream (a torch.cuda.Stream or a raw cudaStream_t)."""
        raw = getattr(stream, "cuda_stream", stream)
        capi.call("sulimo_cuda_ctx_set_stream", self.handle, raw)

    @property
    def stream(self):
        return capi.load().sulimo_cuda_ctx_get_stream(self.handle)

    @property
    def launch_count(self):
        return capi.load().sulimo_cuda_ctx_launch_count(self.handle)

    def finish(self):
        """Blocks until the stream drains; raises on a device-side error (OclContext::finish)."""
        capi.call("sulimo_cuda_ctx_synchronize", self.handle)

    # ---- library-owned device buffers (OclBuffer, crates/sulimo-ocl/src/buffer.rs) ----
    def alloc(self, size):
        """A device buffer of `size` bytes (a cudaMalloc base); returns its handle."""
        import ctypes as C
        h = C.c_void_p()
        capi.call("sulimo_cuda_buffer_alloc", self.handle, size, C.byref(h))
        return h.value

    def write(self, buf, data, off=0):
        """Host bytes / numpy array -> buffer at byte offset `off`."""
        import numpy as np
        a = np.frombuffer(data, np.uint8) if isinstance(data, (bytes, bytearray)) else \
            np.ascontiguousarray(data).view(np.uint8).ravel()
        capi.call("sulimo_cuda_buffer_write", buf, off, a.ctypes.data, a.nbytes)

    def read(self, buf, out, off=0):
        """Buffer bytes at `off` -> the numpy array `out` (its nbytes)."""
        capi.call("sulimo_cuda_buffer_read", buf, off, out.ctypes.data, out.nbytes)
        return out

    @staticmethod
    def device_ptr(buf):
        return capi.load().sulimo_cuda_buffer_device_ptr(buf)

    @staticmethod
    def free(buf):
        capi.call("sulimo_cuda_buffer_free", buf)

    def close(self):
        if self.handle:
            capi.load().sulimo_cuda_ctx_destroy(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def live_buffer_count():
    return capi.load().sulimo_cuda_live_buffer_count()


def gemm_q4_0_f16(ctx, scales, quants, x, out, m, k, n, out_dtype=OUT_F16):
    """enqueue_gemm_q4_0_f16 (crates/sulimo-ocl/src/prefill.rs:69-105): out[n][m] = x[n][k] W^T."""
    capi.call("sulimo_cuda_gemm_q4_0_f16", ctx.handle, _ptr(scales), _ptr(quants), _ptr(x),
              _ptr(out), m, k, n, out_dtype)


def gemm_q4_0_f16_exact(ctx, scales, quants, x, out, m, k, n, out_dtype=OUT_F16):
    """gemm_q4_0_f16 with every weight d*(q-8) carried exactly (two f16 parts, twice the MMAs):
    the products are the reference's, only the fp32 summation order differs."""
    capi.call("sulimo_cuda_gemm_q4_0_f16_exact", ctx.handle, _ptr(scales), _ptr(quants), _ptr(x),
              _ptr(out), m, k, n, out_dtype)


def logits_final(ctx, x_all, scales, quants, logits, vocab, embd, token_idx):
    """enqueue_logits_final (prefill.rs:300-330)."""
    capi.call("sulimo_cuda_logits_final", ctx.handle, _ptr(x_all), _ptr(scales), _ptr(quants),
              _ptr(logits), vocab, embd, token_idx)


def dispatch_matvec_q4_0_q8_0(ctx, w_scales, w_quants, x_q8, rows, cols, out, batch=1,
                              static_weights=False):
    """dispatch_matvec_q4_0_q8_0 (crates/sulimo-cpu/src/avx2.rs:17-37), AVX2-bit-exact.
    static_weights: the weights are not written by the previous kernel on the stream (model
    parameters), so the launch may start streaming them before that kernel finishes."""
    name = "sulimo_cuda_gemv_q4_0_q8_0_static" if static_weights else "sulimo_cuda_gemv_q4_0_q8_0"
    capi.call(name, ctx.handle, _ptr(w_scales), _ptr(w_quants), _ptr(x_q8), rows, cols, batch,
              _ptr(out))


def dispatch_matvec_f32(ctx, w, x, rows, cols, out, batch=1):
    """dispatch_matvec_f32 (crates/sulimo-cpu/src/avx2.rs:72-85), AVX2-bit-exact."""
    capi.call("sulimo_cuda_matvec_f32", ctx.handle, _ptr(w), _ptr(x), rows, cols, batch, _ptr(out))


def dispatch_matvec_f16(ctx, w_f16, x, rows, cols, out, batch=1):
    """dispatch_matvec_f16 (crates/sulimo-cpu/src/avx2.rs:88-104), AVX2-bit-exact."""
    capi.call("sulimo_cuda_matvec_f16", ctx.handle, _ptr(w_f16), _ptr(x), rows, cols, batch,
              _ptr(out))


def apply_matvec(ctx, ggml_type, w0, w1, x_q8, x_f32, rows, cols, out, batch=1):
    """apply_matvec (crates/sulimo-engine/src/forward_pass.rs:509-527): Q4_0 tensors (w0 scales,
    w1 quants) against x_q8, F32 / F16 tensors (w0) against x_f32."""
    capi.call("sulimo_cuda_apply_matvec", ctx.handle, ggml_type, _ptr(w0), _ptr(w1), _ptr(x_q8),
              _ptr(x_f32), rows, cols, batch, _ptr(out))


def matvec_q4_0_q8_0_fast(ctx, w_scales, w_quants, x_q8, rows, cols, out, batch=1,
                          static_weights=False):
    """Fast mode of dispatch_matvec_q4_0_q8_0: the reference's exact integer block sums, fp32
    partials over 8 block residues per row combined in a fixed tree (not the AVX2 add order;
    equal to fp32 rounding, deterministic).  The decode step's matvec."""
    capi.call("sulimo_cuda_gemv_q4_0_q8_0_fast", ctx.handle, _ptr(w_scales), _ptr(w_quants),
              _ptr(x_q8), rows, cols, batch, _ptr(out), 1 if static_weights else 0)


def block_sums_q4_0_q8_0(ctx, w_quants, x_q8, rows, cols, out):
    capi.call("sulimo_cuda_block_sums_q4_0_q8_0", ctx.handle, _ptr(w_quants), _ptr(x_q8), rows,
              cols, _ptr(out))


def quantize_f32_to_q8_0(ctx, src, dst, n=None):
    """quantize_f32_to_q8_0 (crates/sulimo-core/src/kv_cache.rs:162-192), byte-exact."""
    if n is None:
        n = src.numel()
    capi.call("sulimo_cuda_quantize_q8_0", ctx.handle, _ptr(src), _ptr(dst), n)


def kv_store_q8_0(ctx, act, kv, start_pos, capacity, blocks_per_pos, n, act_dtype=None):
    """enqueue_kv_store (prefill.rs:176-205) / KvCache::store_key (kv_cache.rs:93-110)."""
    if act_dtype is None:
        import torch
        act_dtype = ACT_F16 if act.dtype == torch.float16 else ACT_F32
    capi.call("sulimo_cuda_kv_store_q8_0", ctx.handle, _ptr(act), act_dtype, _ptr(kv), start_pos,
              capacity, blocks_per_pos, n)


def dequantize_q4_0_rows(ctx, scales, quants, cols, row_ids, out, out_dtype=OUT_F32):
    """dequantize_q4_0_soa (repack.rs:107-131) / lookup_token_embedding_f16 (scheduler.rs:329)."""
    capi.call("sulimo_cuda_dequantize_q4_0_rows", ctx.handle, _ptr(scales), _ptr(quants), cols,
              _ptr(row_ids), row_ids.numel(), _ptr(out), out_dtype)


def unshard_rows(ctx, gathered, out, world, m_tokens, fs, f):
    """Shard-major all-gather result [world][m_tokens][fs] -> row-major [m_tokens][f]."""
    capi.call("sulimo_cuda_unshard_rows", ctx.handle, _ptr(gathered), _ptr(out), world, m_tokens,
              fs, f, gathered.element_size())


def causal_gqa_attention_prefill(ctx, q, k_ring, v_ring, start_pos, capacity, n, head_count,
                                 head_count_kv, head_dim, out):
    """causal_gqa_attention_prefill (kernels/prefill.cl:120-237): q fp32 [n][H][hd] -> out f16."""
    capi.call("sulimo_cuda_attn_prefill_q8_0", ctx.handle, _ptr(q), _ptr(k_ring), _ptr(v_ring),
              start_pos, capacity, n, head_count, head_count_kv, head_dim, _ptr(out))


def causal_gqa_decode(ctx, q, k_ring, v_ring, capacity, context_len, head_count, head_count_kv,
                      head_dim, out, batch=1, seq_stride_bytes=0, softcap=0.0):
    """causal_gqa_decode_scalar_ext (crates/sulimo-cpu/src/scalar.rs:287-359) over the ring."""
    capi.call("sulimo_cuda_attn_decode_q8_0", ctx.handle, _ptr(q), _ptr(k_ring), _ptr(v_ring),
              seq_stride_bytes, capacity, context_len, head_count, head_count_kv, head_dim, batch,
              float(softcap), _ptr(out))
