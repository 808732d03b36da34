/*
 * sulimo_oracle.h — CPU restatement of Sulimo's quantized-matmul hot path.
 *
 * TEST INFRASTRUCTURE ONLY.  This library is the checker that the CUDA
 * kernels of sulimo_b200 are compared against, and the CPU baseline that
 * bench.py times beside them.  Nothing in the product path (the C-ABI
 * library libsulimo_cuda.so and the sulimo_b200 package) links or calls it.
 *
 * Every function restates one function of the reference (a Rust workspace
 * with OpenCL C kernels; paths below are relative to the reference repository
 * root) and cites the lines it follows.  Pinning: the reference's Rust crates
 * cannot be built without a Rust toolchain, but its OpenCL C kernels
 * (kernels/gemm_q4_0.cl, kernels/prefill.cl) compile unchanged for the host
 * (oracle/_ref via oracle/ref_build.py); the GEMM, KV store, logits, the
 * prefill kernels and the whole prefill ubatch here are bit-identical to them
 * (tests/test_ref_pinning.py, fixture tests/golden/ref_ocl.npz).  The CPU
 * decode path (AVX2 matvec, Q8_0, attention, forward_token) is pinned by the
 * reference's own unit tests re-expressed here (tests/test_oracle.py) and by
 * an exact-arithmetic second restatement (tests/golden/exact_ref.py).
 *
 * Numeric conventions carried over from Rust:
 *   - no FMA contraction (the library is built with -ffp-contract=off);
 *   - f32 -> f16 is IEEE round-to-nearest-even (the `half` crate 2.7.1),
 *     done here with the F16C instruction VCVTPS2PH;
 *   - f32::round is roundf (half away from zero); `as i8` after clamp;
 *   - f32::exp/powf/sin/cos/sqrt are glibc's expf/powf/sinf/cosf/sqrtf.
 */
#ifndef SULIMO_ORACLE_H
#define SULIMO_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- f16 helpers (half 2.7.1 semantics) ---- */
uint16_t oracle_f32_to_f16(float x);
float oracle_f16_to_f32(uint16_t h);
void oracle_f32_to_f16_array(const float* src, uint16_t* dst, size_t n);
void oracle_f16_to_f32_array(const uint16_t* src, float* dst, size_t n);

/* ---- Q4_0 repack / dequant (crates/sulimo-core/src/repack.rs) ---- */
/* returns number of blocks, or -1 (InvalidAosLength) / -2 / -3 (buffer too small) */
long oracle_repack_q4_0_aos_to_soa(const uint8_t* src_aos, size_t src_len,
                                   uint8_t* dst_scales, size_t scales_len,
                                   uint8_t* dst_quants, size_t quants_len);
void oracle_dequantize_q4_0_aos(const uint8_t* src_aos, size_t num_blocks, float* dst);
void oracle_dequantize_q4_0_soa(const uint8_t* scales, const uint8_t* quants,
                                size_t num_blocks, float* dst);
/* f16 dequant of one embedding row (crates/sulimo-engine/src/scheduler.rs:329-374) */
void oracle_lookup_token_embedding_f16(const uint8_t* scales, const uint8_t* quants,
                                       size_t embd_dim, uint32_t token_id, uint16_t* out_f16);

/* ---- Q8_0 (crates/sulimo-core/src/kv_cache.rs) ---- */
void oracle_quantize_f32_to_q8_0(const float* src, size_t n, uint8_t* dst_q8);
void oracle_dequantize_q8_0_to_f32(const uint8_t* src_q8, size_t num_blocks, float* dst);
/* kv_store_q8_0 (kernels/prefill.cl:72-116) fed by the CPU quantizer: f16 activations
 * [n][blocks_per_pos*32] into ring slots (start_pos+t) % capacity. */
void oracle_kv_store_q8_0(const uint16_t* act_f16, uint8_t* kv, size_t start_pos,
                          size_t capacity, size_t blocks_per_pos, size_t n);
/* KvCache::store_key/store_value (kv_cache.rs:93-110): f32 vector into slot pos % capacity */
void oracle_kv_store_f32(const float* vec, uint8_t* kv, size_t pos, size_t capacity,
                         size_t blocks_per_pos);

/* ---- Q4_0 x Q8_0 dot / matvec (crates/sulimo-cpu/src/{scalar,avx2}.rs) ---- */
float oracle_vec_dot_q4_0_q8_0_scalar(const uint8_t* w_scales, const uint8_t* w_quants,
                                      const uint8_t* x_q8, size_t num_blocks);
void oracle_matvec_q4_0_q8_0_scalar(const uint8_t* w_scales, const uint8_t* w_quants,
                                    const uint8_t* x_q8, size_t rows, size_t cols, float* out);
float oracle_vec_dot_q4_0_q8_0_avx2(const uint8_t* w_scales, const uint8_t* w_quants,
                                    const uint8_t* x_q8, size_t num_blocks);
void oracle_matvec_q4_0_q8_0_avx2(const uint8_t* w_scales, const uint8_t* w_quants,
                                  const uint8_t* x_q8, size_t rows, size_t cols, float* out);
/* Same as above over a contiguous row range, on `threads` POSIX threads (harness
 * partitioning for the CPU baseline; each row is computed exactly as above). */
void oracle_matvec_q4_0_q8_0_avx2_mt(const uint8_t* w_scales, const uint8_t* w_quants,
                                     const uint8_t* x_q8, size_t rows, size_t cols, float* out,
                                     int threads);
/* Raw F32 / F16 weight matvecs (apply_matvec's other branches, forward_pass.rs:509-527):
 * AVX2 kernels avx2.rs:259-331 (same intrinsics, same order) and scalar.rs:228-251. */
void oracle_matvec_f32_avx2(const float* w, const float* x, size_t rows, size_t cols, float* out);
void oracle_matvec_f16_avx2(const uint16_t* w, const float* x, size_t rows, size_t cols,
                            float* out);
void oracle_matvec_f32_scalar(const float* w, const float* x, size_t rows, size_t cols,
                              float* out);
void oracle_matvec_f16_scalar(const uint16_t* w, const float* x, size_t rows, size_t cols,
                              float* out);
/* Integer per-block sums: out[r*nb+b] = sum_i (w_i-8)*x_i (exact i32). */
void oracle_block_sums_q4_0_q8_0(const uint8_t* w_scales, const uint8_t* w_quants,
                                 const uint8_t* x_q8, size_t rows, size_t cols, int32_t* out);

/* ---- Prefill GEMM (crates/sulimo-ocl/src/gemm.rs:106-147) ---- */
void oracle_gemm_q4_0_f16_scalar_reference(const uint16_t* scales, const uint8_t* quants,
                                           const uint16_t* x, size_t m, size_t k, size_t n,
                                           uint16_t* out);
/* same arithmetic, fp32 result (logits_f16_output, kernels/prefill.cl:269-308) */
void oracle_gemm_q4_0_f16_scalar_f32out(const uint16_t* scales, const uint8_t* quants,
                                        const uint16_t* x, size_t m, size_t k, size_t n,
                                        float* out, int threads);
/* Reference CPU prefill of n tokens through one Q4_0 projection (engine.rs:287-318 ->
 * forward_token -> quantize_f32_to_q8_0 + matvec_q4_0_q8_0_avx2), fp32 activations in. */
void oracle_cpu_prefill_projection(const uint8_t* w_scales, const uint8_t* w_quants,
                                   const float* x, size_t m, size_t k, size_t n, float* out,
                                   int threads);

/* ---- small ops (crates/sulimo-cpu/src/{scalar,avx2}.rs) ---- */
void oracle_rmsnorm_scalar(const float* x, const float* w, size_t len, float eps, float* out);
void oracle_rmsnorm_avx2(const float* x, const float* w, size_t len, float eps, float* out);
void oracle_rope_head_scalar(float* vec, size_t pos, size_t rope_dim, float freq_base, int mode);
void oracle_softmax_scalar(float* x, size_t n);
void oracle_swiglu_scalar(const float* gate, const float* up, float* out, size_t n);

/* ---- decode attention (crates/sulimo-cpu/src/scalar.rs:287-359) ----
 * k_ring / v_ring: one layer's ring, capacity slots of (head_count_kv*head_dim/32)*34 bytes.
 * Position p reads slot p % capacity (KvCache::key_ptr, kv_cache.rs:114-119).
 * scores_buf must hold context_len floats.  softcap <= 0 means none. */
void oracle_causal_gqa_decode(const float* q, const uint8_t* k_ring, const uint8_t* v_ring,
                              size_t capacity, size_t context_len, size_t head_count,
                              size_t head_count_kv, size_t head_dim, float* scores_buf,
                              float* out, float softcap);

/* ---- one decode position through the whole model (forward_token,
 * crates/sulimo-engine/src/forward_pass.rs:190-417), Llama / Qwen2 / Gemma 2 paths: RMSNorm (AVX2),
 * Q8_0 activations, AVX2 matvecs, optional QKV biases, RoPE (Norm / Neox), Q8_0 ring store,
 * causal GQA decode, SwiGLU, residual adds, final norm and the vocab projection. */
typedef struct oracle_layer {
    const float *attn_norm, *ffn_norm;  /* [embd] */
    const float *bq, *bk, *bv;          /* biases or NULL */
    const uint8_t *wq_s, *wq_q, *wk_s, *wk_q, *wv_s, *wv_q, *wo_s, *wo_q;
    const uint8_t *wg_s, *wg_q, *wu_s, *wu_q, *wd_s, *wd_q;
    uint8_t *k_ring, *v_ring;           /* capacity slots of kv_dim/32 Q8_0 blocks */
    const float *post_attn_norm, *post_ffn_norm;  /* Gemma 2's post norms, or NULL */
} oracle_layer;

typedef struct oracle_model {
    int n_layers, embd, ffn, head_count, head_count_kv, head_dim, vocab, rope_dim, rope_mode;
    float eps, rope_base, attn_softcap;
    size_t kv_capacity;
    const uint8_t *tok_s, *tok_q; /* token_embd [vocab][embd] Q4_0 SoA */
    const uint8_t *out_s, *out_q; /* output [vocab][embd] Q4_0 SoA (tied: same pointers) */
    const float* out_norm;
    const oracle_layer* layers;
    int arch;            /* ORACLE_ARCH_DEFAULT (Llama / Qwen2) or ORACLE_ARCH_GEMMA2 */
    float final_softcap; /* final logit soft-capping (Gemma 2), <= 0: none */
} oracle_model;

#define ORACLE_ARCH_DEFAULT 0
#define ORACLE_ARCH_GEMMA2 1

/* rmsnorm_gemma_avx2 (avx2.rs:236-268), geglu_scalar (scalar.rs:77-89), logit_softcap_scalar
 * (scalar.rs:63-71) */
void oracle_rmsnorm_gemma_avx2(const float* x, const float* w, size_t len, float eps, float* out);
void oracle_geglu_scalar(const float* gate, const float* up, float* out, size_t n);
void oracle_logit_softcap_scalar(float* v, size_t n, float cap);

/* logits [vocab] for `token` at position `pos` (context pos+1); stores K/V at pos. */
void oracle_forward_token(const oracle_model* m, uint32_t token, size_t pos, float* logits);


/* ---- GPU prefill ubatch on f16 storage (crates/sulimo-ocl/src/prefill.rs:337-566 over the
 * kernels of kernels/prefill.cl): every activation is f16 between kernels, as in the
 * reference.  x: [n][embd] f16 embeddings in, residual stream out; writes ring slots
 * (start_pos+t) % kv_capacity; logits[vocab] of the last token.  No QKV bias (the reference's
 * GPU ubatch applies none).  Requires head_count*head_dim == embd.  0 or -1. */
void oracle_rmsnorm_f16(const uint16_t* x, const float* w, uint16_t* out, size_t D, float eps,
                        size_t N);
void oracle_rope_f16(uint16_t* vec, size_t head_count, size_t head_dim, size_t rope_dim,
                     float freq_base, int mode, size_t start_pos, size_t N);
void oracle_attention_prefill_f16(const uint16_t* q, const uint8_t* k_ring, const uint8_t* v_ring,
                                  uint16_t* out, size_t start_pos, size_t capacity,
                                  size_t head_count, size_t head_count_kv, size_t head_dim,
                                  size_t N);
void oracle_silu_mul_f16(const uint16_t* gate, const uint16_t* up, uint16_t* out, size_t n);
void oracle_add_f16(uint16_t* a, const uint16_t* b, size_t n);
int oracle_prefill_ubatch(const oracle_model* m, uint16_t* x, size_t start_pos, size_t n,
                          float* logits, int threads);
/* The CPU oracle of the reference's prefill test (crates/sulimo-ocl/tests/test_prefill.rs:
 * 583-800): fp32 residual, f16 GEMM inputs and outputs, scalar RMSNorm / RoPE / Q8_0 store /
 * causal decode attention per token, fp32 final norm; QKV biases added when present.  x_f16
 * [n][embd] is not modified.  0 or -1. */
int oracle_prefill_ubatch_f32(const oracle_model* m, const uint16_t* x_f16, size_t start_pos,
                              size_t n, float* logits, int threads);

#ifdef __cplusplus
}
#endif
#endif
