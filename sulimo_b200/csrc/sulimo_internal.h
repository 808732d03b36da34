// sulimo_internal.h — host-side context and kernel launchers shared by the .cu files.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

#include <atomic>
#include <string>
#include <utility>

#include "../../include/sulimo_cuda.h"

struct sulimo_ctx {
    int device = 0;
    int num_sms = 0;
    cudaStream_t own_stream = nullptr;
    cudaStream_t stream = nullptr;  // the stream launches go to (own or caller's)
    int* d_error = nullptr;         // device error word (0 = none)
    void* workspace = nullptr;      // attention partials
    size_t workspace_bytes = 0;
    void* argmax_scratch = nullptr;  // greedy argmax partials + per-row counters (zero at rest)
    size_t argmax_bytes = 0;
    unsigned* attn_counters = nullptr;  // decode attention merge counters (zero at rest)
    void* q8_stage = nullptr;  // staged activations of the batched fast matvec (C-ABI inputs)
    size_t q8_stage_bytes = 0;
    std::atomic<uint64_t> launches{0};
};

namespace sulimo {

// One "done" bit per device (device index mod 64) for per-device, idempotent set-up such as
// cudaFuncSetAttribute.  Atomic, so host threads driving different devices may test and set
// it concurrently; two threads that both see the bit clear both do the (idempotent) set-up.
struct DeviceBits {
    std::atomic<uint64_t> bits{0};
    bool test(int device) const {
        return (bits.load(std::memory_order_acquire) >> (device & 63)) & 1;
    }
    void set(int device) { bits.fetch_or(1ull << (device & 63), std::memory_order_release); }
};

// Launches a kernel with programmatic stream serialization: it may begin (prologue, TMEM
// allocation, barrier setup) while the previous kernel of the stream drains, and orders its
// global accesses after that kernel with griddepcontrol.wait.
template <typename... Params, typename... Args>
cudaError_t launch_pdl(void (*kernel)(Params...), dim3 grid, dim3 block, size_t smem,
                       cudaStream_t stream, Args&&... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

// Thread-local error message + status helper.
int set_error(int status, const std::string& msg);
int check_cuda(cudaError_t e, const char* what);
// Grows ctx->workspace to at least `bytes` (synchronizes the stream first if it must grow).
int ensure_workspace(sulimo_ctx* ctx, size_t bytes);

// cuTensorMapEncodeTiled resolved through the runtime's driver entry point.
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                  const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                  const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                  CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
EncodeTiledFn get_encode_tiled();
// Encodes a tiled tensor map of rank 2 or 3: dims and box innermost first, `strides` = byte
// strides of dims 1.. (rank-1 entries); interleave none, L2 promotion 256B, zero OOB fill.
int encode_tensor_map(CUtensorMap* map, CUtensorMapDataType dt, const void* base, int rank,
                      const uint64_t* dims, const uint64_t* strides, const uint32_t* box,
                      CUtensorMapSwizzle swz);

// Launchers (return SULIMO_* status; argument checks done by the C-ABI layer).
// Tile plan of the CTA-pair prefill GEMM (gemm_q4_0_pair.cu).
struct PairPlan {
    int bn, splits, iters_per_split, stages, grid_x, grid_y;
    uint32_t smem;
};
PairPlan gemm_pair_plan(int m, int k, int n, int max_pairs);
// Weight matrices stacked along M for one pair GEMM: matrix g from row start[g] (a multiple of
// 128), rows[g] rows, block scales scales[g].
struct PairSegs {
    const uint16_t* scales[3];
    int start[3];
    int rows[3];
};
// One matrix of a stacked GEMM: Q4_0 SoA weights of `rows` rows.
struct GemmSeg {
    const void* scales;
    const void* quants;
    int rows;
};
// Whether the pair GEMM takes these matrices stacked (every one but the last a multiple of 128
// rows, the stack wide enough for the pair kernel).
bool gemm_stacked_applies(const GemmSeg* segs, int nseg, int k, int n);
// The pair GEMM of f16 activations x [n][k] against the stacked matrices, as fp32 split-K
// partials [*splits][n][sum of rows] in ctx->workspace (*partials); the caller sums them.
int launch_gemm_pair_stacked(sulimo_ctx* ctx, const GemmSeg* segs, int nseg, const void* x, int k,
                             int n, const float** partials, int* splits);
// Whether the gated pair GEMM takes rows x k weights and n tokens.
bool gemm_gated_applies(int rows, int k, int n);
// silu(x W_gate^T) * (x W_up^T) as f16 out [n][rows] in one pair GEMM (no split-K): CTA 0 of a
// pair computes the gate rows, CTA 1 the same up rows, and they exchange halves of the tile.
int launch_gemm_pair_gated(sulimo_ctx* ctx, const GemmSeg& gate, const GemmSeg& up,
                           const void* x, int k, int n, void* out);
bool gemm_uses_pair(int m, int k, int n);
int launch_gemm_pair(sulimo_ctx* ctx, const void* scales, const void* quants, const void* x,
                     void* out, int m, int k, int n, int out_dtype, int x_row_stride,
                     int x_row_offset);
// Ordered sum of split-K fp32 partials ws[splits][nm] into f16 / f32 out (one launch).
int launch_splitk_reduce(sulimo_ctx* ctx, const float* ws, void* out, size_t nm, int splits,
                         bool out_f32);
// exact: the exact-weight form (hi + lo f16 parts of every weight; one-CTA kernel).
int launch_gemm_q4_0_f16(sulimo_ctx* ctx, const void* scales, const void* quants, const void* x,
                         void* out, int m, int k, int n, int out_dtype, int x_row_stride,
                         int x_row_offset, bool exact = false);
// Row-sharded GEMM with the all-gather in the epilogue (see gemm_q4_0_tc.cu): stores this rank's
// [n][m_local] result at column col0 of every rank's row-major Y (row pitch f_total elements,
// out_bases[r] mapped in this process) and adds one per CTA to every rank's counter.
int launch_gemm_allgather(sulimo_ctx* ctx, const void* scales, const void* quants, const void* x,
                          int m_local, int m_valid, int k, int n, int out_dtype,
                          void* const* out_bases, size_t f_total, size_t col0,
                          unsigned* const* flags, unsigned* const* release, int world, int rank,
                          unsigned epoch, unsigned* tiles_out);
int launch_wait_counter(sulimo_ctx* ctx, const unsigned* flag, unsigned target);
// Where a decode-step producer writes its Q8_0 activations (row = sequence, K values per row):
//   aos:   the reference's block array [rows][K/32][34], or null;
//   codes / aux: the staged form the batched tensor-core matvec reads (gemv_mma_q4_0_q8_0.cu),
//          or null: codes [rows8][K] i8 (rows8 = rows rounded up to 8) and per block
//          aux [rows8 / 8][K/32][8] = {d as f32 bits (the f16 value), 0x4B400000 - 8 * sum(q)}
//          (the second word seeds the matvec's integer accumulator).
struct Q8Out {
    uint8_t* aos;
    int8_t* codes;
    int2* aux;
    int K;
};
// Bytes of the staged form for `batch` rows of K values, and its two arrays inside `base`.
size_t q8_staged_bytes(int batch, int K);
Q8Out q8_staged_view(void* base, int batch, int K);
// Q8_0 block arrays [batch][K/32][34] -> the staged form (one launch).
int launch_q8_stage(sulimo_ctx* ctx, const void* x_q8, int batch, int K, const Q8Out& dst);
int launch_gemv_q4_0_q8_0(sulimo_ctx* ctx, const void* w_scales, const void* w_quants,
                          const void* x_q8, int rows, int cols, int batch, float* out);
// One matrix of a grouped decode GEMV (all of a group share K and the activations).
struct GemvMatSrc {
    const void* scales;
    const void* quants;
    float* out;
    int rows;
};
// Streams 1..3 matrices in one launch (the exact AVX2-order GEMV); *handled is false when the
// streaming form does not apply and the caller must launch each matrix on its own.
// static_weights: the caller guarantees the weights are not written by the previous kernel of
// the stream, so the first weight tiles may be fetched before the programmatic-launch wait.
int launch_gemv_group(sulimo_ctx* ctx, const GemvMatSrc* src, int count, const void* x_q8,
                      int cols, int batch, bool* handled, bool static_weights);
// launch_gemv_q4_0_q8_0 for a decode step's static weights (see launch_gemv_group).
int launch_gemv_static(sulimo_ctx* ctx, const void* w_scales, const void* w_quants,
                       const void* x_q8, int rows, int cols, int batch, float* out);
// Fast-mode matvec (exact integer block sums, fp32 partials over 8 block residues combined in a
// fixed tree; not the AVX2 add order) for 1..3 matrices sharing x_q8; falls back to the exact
// kernel when its layout conditions do not hold.
int launch_gemv_fast_group(sulimo_ctx* ctx, const GemvMatSrc* src, int count, const void* x_q8,
                           int cols, int batch, bool static_weights);
// Batched fast-mode matvec on the tensor cores (gemv_mma_q4_0_q8_0.cu) for 1..3 matrices
// sharing staged activations x (Q8Out codes / aux); gemv_mma_applies tells whether the shape and
// layout qualify (K a multiple of 256, 16-byte aligned quants and scales).
bool gemv_mma_applies(const GemvMatSrc* src, int count, int cols, int batch, int num_sms);
// Sequences from which the fast matvec takes the tensor-core form.
constexpr int GEMV_MMA_MIN_BATCH = 2;
int launch_gemv_mma_group(sulimo_ctx* ctx, const GemvMatSrc* src, int count, const Q8Out& x,
                          int cols, int batch, bool static_weights);
// Activation producer folded into the fast matvec's prologue (every CTA recomputes the vector
// from L2 after the launch's dependency wait; the quantization is quantize_f32_to_q8_0):
//   GEMV_PRO_NORM: v = a + b (b may be null), written to a_out by the CTAs of column 0 when
//                  a_out is set; x = quantize((v * 1/sqrt(mean(v^2) + eps)) * w)
// a, b, a_out: [batch][cols] f32, 16-byte aligned; a_out never aliases a or b.  Batch 1 and
// cols <= 4096 (the vector is held in registers, one L2 round trip).
enum { GEMV_PRO_Q8 = 0, GEMV_PRO_NORM = 1 };
struct GemvPrologue {
    int mode;
    const float* a;
    const float* b;
    const float* w;
    float* a_out;
    float eps;
};
// Whether launch_gemv_fast_fused handles this shape (else the caller runs the producer kernel
// and launch_gemv_fast_group / the exact matvec).
bool gemv_fast_fused_ok(const GemvMatSrc* src, int count, int cols, int batch,
                        const GemvPrologue& pro);
int launch_gemv_fast_fused(sulimo_ctx* ctx, const GemvMatSrc* src, int count,
                           const GemvPrologue& pro, int cols, int batch, bool static_weights);
int launch_matvec_dense(sulimo_ctx* ctx, int wtype, const void* w, const float* x, int rows,
                        int cols, int batch, float* out);
int launch_block_sums(sulimo_ctx* ctx, const void* w_quants, const void* x_q8, int rows, int cols,
                      int32_t* out);
int launch_quantize_q8_0(sulimo_ctx* ctx, const float* src, void* dst, size_t n);
int launch_kv_store_q8_0(sulimo_ctx* ctx, const void* act, int act_dtype, void* kv,
                         size_t start_pos, size_t capacity, size_t blocks_per_pos, size_t n);
// Dequantisation output modes: SULIMO_OUT_F16 / SULIMO_OUT_F32 (DEQUANT_F32) as in the C ABI,
// and DEQUANT_F16_WIDE (the f16-rounded weight stored as f32; internal).
enum { DEQUANT_F16 = SULIMO_OUT_F16, DEQUANT_F32 = SULIMO_OUT_F32, DEQUANT_F16_WIDE = 2 };
int launch_dequant_rows(sulimo_ctx* ctx, const void* scales, const void* quants, int cols,
                        const int32_t* row_ids, int count, void* out, int out_dtype);
// Decode attention merge counters per context: [sequence][cluster rank], up to the batch limit.
constexpr size_t ATTN_COUNTERS = (size_t)65536 * 8;
// The tensor-core decode attention (attn_decode_mma.cu).  *used = false (and nothing launched)
// when the geometry or the workspace does not fit it; the caller then runs the scalar kernels.
int launch_attn_decode_mma(sulimo_ctx* ctx, const float* q, const void* k_ring,
                           const void* v_ring, size_t seq_stride, size_t capacity,
                           size_t context_len, int head_count, int head_count_kv, int head_dim,
                           int batch, float softcap, float* out, float* partials,
                           size_t partial_bytes, const Q8Out& out_q8,
                           bool* used, size_t static_before = 0);
size_t attn_decode_mma_partial_bytes(size_t ctx_len, size_t capacity, int H, int Hkv, int HD,
                                     int batch, int num_sms, size_t seq_stride, const void* k,
                                     const void* v);
int launch_attn_decode(sulimo_ctx* ctx, const float* q, const void* k_ring, const void* v_ring,
                       size_t seq_stride, size_t capacity, size_t context_len, int head_count,
                       int head_count_kv, int head_dim, int batch, float softcap, float* out,
                       float* partials, size_t partial_bytes, const Q8Out* out_q8 = nullptr,
                       size_t static_before = 0);
int launch_unshard_rows(sulimo_ctx* ctx, const void* gathered, void* out, int world,
                        int m_tokens, size_t fs, size_t f, int elem_size);
size_t forward_scratch_bytes(const sulimo_model_desc* m, int batch);
int launch_forward_token(sulimo_ctx* ctx, const sulimo_model_desc* m, const int32_t* tokens,
                         int batch, size_t pos, float* logits, void* scratch);
int launch_argmax_rows(sulimo_ctx* ctx, const float* x, int rows, int cols, int32_t* out);
size_t prefill_scratch_bytes(const sulimo_model_desc* m, int n);
// tokens != nullptr: embeddings looked up on the device (f16-rounded, as the reference's
// lookup_token_embedding_f16); else x_f16 [n][embd] holds them (the reference's scratch.x).
int launch_prefill_ubatch(sulimo_ctx* ctx, const sulimo_model_desc* m, const int32_t* tokens,
                          const void* x_f16, int n, size_t start_pos, float* logits,
                          void* scratch);
// repack_context's arithmetic (scheduler.rs:316-326) and the device-side repack + re-prefill.
void repack_context_plan(size_t n_past, size_t capacity, size_t* sys_len, size_t* recent_len);
int launch_repack_context(sulimo_ctx* ctx, const sulimo_model_desc* m, const int32_t* past,
                          size_t n_past, int32_t* new_tokens, int ubatch, float* logits,
                          void* scratch, size_t* new_pos);
int launch_repack_q4_0(sulimo_ctx* ctx, const void* src_aos, size_t nblocks, void* dst_scales,
                       void* dst_quants);
// tcgen05 form of the prefill attention (attn_prefill_tc.cu) and whether it applies.
bool attn_prefill_tc_applies(const float* q, const void* k_ring, const void* v_ring,
                             size_t capacity, int Hkv, int hd, const void* out);
int launch_attn_prefill_tc(sulimo_ctx* ctx, const float* q, const void* k_ring,
                           const void* v_ring, size_t start_pos, size_t capacity, int n_tok,
                           int H, int Hkv, int hd, void* out);
int launch_attn_prefill(sulimo_ctx* ctx, const float* q, const void* k_ring, const void* v_ring,
                        size_t start_pos, size_t capacity, int n_tok, int H, int Hkv, int hd,
                        void* out);
// Workspace bytes (and split count) the attention entry point will use for this geometry.
size_t attn_decode_partial_bytes(size_t context_len, size_t capacity, int head_count,
                                 int head_count_kv, int head_dim, int batch, int num_sms,
                                 size_t seq_stride, const void* k, const void* v,
                                 int* splits_out);
// Smallest split count the per-head partial kernel accepts (<= 256 positions per split) and
// that kernel's own preferred count.
void attn_decode_split_range(size_t context_len, int head_count_kv, int batch, int num_sms,
                             int* min_splits, int* default_splits);
// Decode attention with a caller-chosen split count and partials buffer (which must hold
// batch * head_count * splits * (head_dim + 2) floats).
int launch_attn_decode_with_splits(sulimo_ctx* ctx, const float* q, const void* k_ring,
                                   const void* v_ring, size_t seq_stride, size_t capacity,
                                   size_t context_len, int head_count, int head_count_kv,
                                   int head_dim, int batch, float softcap, float* out,
                                   float* partials, int splits);

}  // namespace sulimo
