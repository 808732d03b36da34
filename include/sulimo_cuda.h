/*
 * sulimo_cuda.h — C ABI of the B200 (sm_100a) backend for Sulimo's quantized-matmul hot path.
 *
 * This is the drop-in boundary a `sulimo-cuda` Rust crate binds through FFI in place of the
 * `sulimo-ocl` (OpenCL prefill) and `sulimo-cpu` (AVX2 decode) backends.  Every entry point
 * names the reference interface it replaces (paths relative to the reference repository).
 *
 * Conventions
 *   - Plain pointers and sizes only.  Tensor pointers are DEVICE pointers (cudaMalloc'd or
 *     obtained from sulimo_cuda_buffer_device_ptr) unless a parameter says "host".
 *   - Weight format is the reference's Q4_0 SoA arena layout (crates/sulimo-core/src/repack.rs:
 *     45-81): `scales` = rows*(cols/32) little-endian f16, `quants` = rows*(cols/32)*16 bytes,
 *     row r / block b at index r*(cols/32)+b; weight i<16 is the low nibble of qs[i], i>=16 the
 *     high nibble of qs[i-16]; value (nibble-8)*d.
 *   - Activation / KV format is Q8_0 (crates/sulimo-core/src/kv_cache.rs:11-15): 34-byte blocks
 *     [f16 d][32 x i8].
 *   - Every call returns an int status (SULIMO_OK == 0).  Shape violations that the reference
 *     turns into a panic (assert!) return SULIMO_EINVAL here; nothing aborts the process.
 *     sulimo_cuda_last_error() returns a thread-local message for the last failure.
 *   - Kernels are enqueued on the context's stream and return without waiting, like the
 *     reference's enqueue_* functions; sulimo_cuda_ctx_synchronize / sulimo_cuda_event_wait
 *     are the waits.  A kernel whose bounded internal wait ran out records a device error that
 *     the next synchronize returns as SULIMO_EDEVICE.
 */
#ifndef SULIMO_CUDA_H
#define SULIMO_CUDA_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* The library is built with hidden visibility; everything declared here is exported. */
#if defined(__GNUC__)
#pragma GCC visibility push(default)
#endif

/* Status codes — map the variants of OclError (crates/sulimo-ocl/src/program.rs:26-40). */
enum {
    SULIMO_OK = 0,
    SULIMO_EINVAL = 1,   /* bad shape / argument (reference: assert! panics)            */
    SULIMO_ENODEV = 2,   /* no usable sm_100 device (OclError::DeviceNotFound)          */
    SULIMO_EOOM = 3,     /* device allocation failed                                    */
    SULIMO_ELAUNCH = 4,  /* CUDA launch / driver error (OclError::Driver)               */
    SULIMO_ETIMEOUT = 5, /* host wait deadline passed                                   */
    SULIMO_ENCCL = 6,    /* NCCL error in a sharded call                                */
    SULIMO_EALIGN = 7,   /* pointer / size alignment violated (OclError::ZeroCopyViolation) */
    SULIMO_EDEVICE = 8   /* a kernel reported a device-side error (OclError::ExecutionFailed) */
};

/* Output element types for the prefill GEMM. */
enum { SULIMO_OUT_F16 = 0, SULIMO_OUT_F32 = 1 };
/* Tensor types of the reference's loader (GgmlType, crates/sulimo-core/src/gguf.rs:118-122).  */
enum { SULIMO_GGML_F32 = 0, SULIMO_GGML_F16 = 1, SULIMO_GGML_Q4_0 = 2 };
/* Activation element types. */
enum { SULIMO_ACT_F16 = 0, SULIMO_ACT_F32 = 1 };

typedef struct sulimo_ctx sulimo_ctx;
typedef struct sulimo_buf sulimo_buf;
typedef struct sulimo_event sulimo_event;

/* ---------------------------------------------------------------------------------------- */
/* Errors / version                                                                          */
/* ---------------------------------------------------------------------------------------- */
const char* sulimo_cuda_last_error(void);
const char* sulimo_cuda_version(void);

/* ---------------------------------------------------------------------------------------- */
/* Context — replaces OclContext::new / get_or_init / finish                                 */
/* (crates/sulimo-ocl/src/program.rs:79-94).  One context = one device + one stream.          */
/* ---------------------------------------------------------------------------------------- */
int sulimo_cuda_ctx_create(int device, sulimo_ctx** out);
int sulimo_cuda_ctx_destroy(sulimo_ctx* ctx);
/* Wait for all work on the context stream; returns SULIMO_EDEVICE if a kernel flagged an error. */
int sulimo_cuda_ctx_synchronize(sulimo_ctx* ctx);
/* Launch on the caller's cudaStream_t (e.g. a framework's current stream) instead of the
 * context's own non-blocking stream.  NULL selects the CUDA legacy default stream; keep the
 * value of sulimo_cuda_ctx_get_stream() from before the switch to return to the own stream. */
int sulimo_cuda_ctx_set_stream(sulimo_ctx* ctx, void* cuda_stream);
void* sulimo_cuda_ctx_get_stream(sulimo_ctx* ctx);
int sulimo_cuda_ctx_device(sulimo_ctx* ctx);
/* Launches issued by this library since the context was created (a kernel-count probe). */
uint64_t sulimo_cuda_ctx_launch_count(sulimo_ctx* ctx);
/* Bytes of device memory the context has allocated for itself on demand (the attention      */
/* workspace and the argmax partials; caller-owned buffers excluded) — a memory diagnostic    */
/* in the spirit of active_cl_mem_count (crates/sulimo-ocl/src/buffer.rs:21).                 */
size_t sulimo_cuda_ctx_workspace_bytes(sulimo_ctx* ctx);

/* ---------------------------------------------------------------------------------------- */
/* Buffers — replace OclBuffer::from_host_ptr / map_read / Drop / active_cl_mem_count        */
/* (crates/sulimo-ocl/src/buffer.rs:21-161).  The reference wraps host arena memory          */
/* zero-copy; a B200 is discrete, so a buffer owns device memory and from_host copies the    */
/* host bytes in.  The host alignment contract is kept: host_ptr 4096-aligned and size a     */
/* multiple of 64 when `strict_arena` is set (else SULIMO_EALIGN).                           */
/* ---------------------------------------------------------------------------------------- */
int sulimo_cuda_buffer_from_host(sulimo_ctx* ctx, const void* host_ptr, size_t size,
                                 int read_only, int strict_arena, sulimo_buf** out);
int sulimo_cuda_buffer_alloc(sulimo_ctx* ctx, size_t size, sulimo_buf** out);
int sulimo_cuda_buffer_write(sulimo_buf* buf, size_t offset, const void* host_src, size_t n);
int sulimo_cuda_buffer_read(sulimo_buf* buf, size_t offset, void* host_dst, size_t n);
void* sulimo_cuda_buffer_device_ptr(sulimo_buf* buf);
size_t sulimo_cuda_buffer_size(sulimo_buf* buf);
int sulimo_cuda_buffer_free(sulimo_buf* buf);
/* Number of live buffers (active_cl_mem_count, buffer.rs:21-23). */
size_t sulimo_cuda_live_buffer_count(void);

/* ---------------------------------------------------------------------------------------- */
/* Events — replace wait_event_zero_spin (crates/sulimo-ocl/src/waiter.rs:39-82).            */
/* The wait blocks in the driver (cudaEventBlockingSync, no spinning) up to timeout_ns       */
/* (0 = no deadline) and returns SULIMO_ETIMEOUT instead of hanging.                         */
/* ---------------------------------------------------------------------------------------- */
int sulimo_cuda_event_record(sulimo_ctx* ctx, sulimo_event** out);
int sulimo_cuda_event_wait(sulimo_event* ev, uint64_t timeout_ns);
int sulimo_cuda_event_free(sulimo_event* ev);

/* ---------------------------------------------------------------------------------------- */
/* Prefill GEMM — replaces enqueue_gemm_q4_0_f16 (crates/sulimo-ocl/src/prefill.rs:69-105)   */
/* and gemm_q4_0_f16 (crates/sulimo-ocl/src/gemm.rs:28-102), kernels                          */
/* gemm_q4_0_f16_{portable,intel} (kernels/gemm_q4_0.cl:13-130).                             */
/*   out[t][r] = sum_b d[r][b] * sum_i x[t][32b+i] * (q[r][b][i]-8),  t < n, r < m            */
/* m = output features (rows of W), k = input channels, n = tokens; x is [n][k] f16 row-major,*/
/* out is [n][m] f16 (SULIMO_OUT_F16, as the reference) or f32 (SULIMO_OUT_F32, the          */
/* logits_f16_output form, kernels/prefill.cl:269-308).  Requires k % 32 == 0 and            */
/* m % 8 == 0 (the reference's asserts, gemm.rs:39-40); x, out and quants 16-byte aligned.    */
/* Tensor cores compute with B operand f16(d*(q-8)) (one RNE rounding per weight) and fp32   */
/* accumulation.  The weights are read as static: the kernel may start loading scales and    */
/* quants while the previous kernel of the context's stream still runs, if that kernel lets   */
/* its dependents launch early (griddepcontrol.launch_dependents); none of this library's     */
/* kernels that write Q4_0 weights does (sulimo_cuda_repack_q4_0_aos_to_soa).                  */
/* ---------------------------------------------------------------------------------------- */
int sulimo_cuda_gemm_q4_0_f16(sulimo_ctx* ctx, const void* scales, const void* quants,
                              const void* x, void* out, int m, int k, int n, int out_dtype);

/* Exact-weight prefill GEMM — the same operation and arguments as sulimo_cuda_gemm_q4_0_f16  */
/* (the reference's gemm_q4_0_f16, gemm.rs:28-102, and its scalar oracle gemm.rs:106-147),    */
/* with every weight d*(q-8) carried exactly into the tensor cores as two f16 parts            */
/* hi = f16(d*(q-8)) and lo = f16(d*(q-8) - hi), so each product equals the reference's and    */
/* only the fp32 summation order differs (the bar of crates/sulimo-ocl/tests/test_gemm.rs:    */
/* 207-214).  Twice the tensor work of sulimo_cuda_gemm_q4_0_f16.                             */
int sulimo_cuda_gemm_q4_0_f16_exact(sulimo_ctx* ctx, const void* scales, const void* quants,
                                    const void* x, void* out, int m, int k, int n,
                                    int out_dtype);

/* Last-token logits — replaces enqueue_logits_final (prefill.rs:300-330): fp32 logits of    */
/* token row `token_idx` of x_all [*, embd] against a [vocab][embd] Q4_0 matrix.             */
int sulimo_cuda_logits_final(sulimo_ctx* ctx, const void* x_all, const void* scales,
                             const void* quants, float* logits, int vocab, int embd,
                             int token_idx);

/* ---------------------------------------------------------------------------------------- */
/* Decode GEMV — replaces dispatch_matvec_q4_0_q8_0 (crates/sulimo-cpu/src/avx2.rs:17-37)     */
/* with matvec_q4_0_q8_0_avx2 / vec_dot_q4_0_q8_0_avx2 (avx2.rs:113-189).                    */
/* x_q8 holds `batch` Q8_0 vectors of cols/32 blocks each; out is [batch][rows] f32.         */
/* The result is bit-identical to the AVX2 kernel: eight fp32 lanes per row accumulate       */
/* fma(float(lane_sum), d_w*d_x, acc) over blocks in order and are reduced with hsum_256's   */
/* add tree (avx2.rs:333-342).  Requires cols % 32 == 0.                                     */
/* ---------------------------------------------------------------------------------------- */
int sulimo_cuda_gemv_q4_0_q8_0(sulimo_ctx* ctx, const void* w_scales, const void* w_quants,
                               const void* x_q8, int rows, int cols, int batch, float* out);

/* Same result as sulimo_cuda_gemv_q4_0_q8_0 for weights that the previous kernel on the stream */
/* does not write (a decode step's model parameters): the first weight tiles are fetched before */
/* the launch's wait on the previous kernel, so back-to-back matvecs overlap their weight       */
/* streams.  The activations are always read after the wait.                                    */
int sulimo_cuda_gemv_q4_0_q8_0_static(sulimo_ctx* ctx, const void* w_scales,
                                      const void* w_quants, const void* x_q8, int rows, int cols,
                                      int batch, float* out);

/* Fast mode of the same matvec (exact_mode = 0 of the entry above): the integer block sums are the      */
/* reference's, exact; each row's blocks are split over 8 fp32 partial sums (block index mod 8) */
/* combined as ((p0+p1)+(p2+p3))+((p4+p5)+(p6+p7)), so the result differs from the AVX2 add   */
/* order only by fp32 rounding and is deterministic for a given shape.  This is the form the   */
/* decode step (sulimo_cuda_forward_token) streams its weights with.  static_weights != 0: the */
/* weights are not written by the previous kernel on the stream (see the _static entry).       */
int sulimo_cuda_gemv_q4_0_q8_0_fast(sulimo_ctx* ctx, const void* w_scales, const void* w_quants,
                                    const void* x_q8, int rows, int cols, int batch, float* out,
                                    int static_weights);

/* Raw F32 / F16 weight matvecs — replace dispatch_matvec_f32 / dispatch_matvec_f16           */
/* (crates/sulimo-cpu/src/avx2.rs:72-104; AVX2 kernels :259-331): w [rows][cols] (f32, or f16  */
/* little-endian bytes), x [batch][cols] fp32, out [batch][rows] fp32; bit-identical to the     */
/* AVX2 kernels (eight FMA lanes per row in column order, the hsum_256 tree, then the tail     */
/* columns multiply-then-add).  Any cols >= 1.                                                 */
int sulimo_cuda_matvec_f32(sulimo_ctx* ctx, const float* w, const float* x, int rows, int cols,
                           int batch, float* out);
int sulimo_cuda_matvec_f16(sulimo_ctx* ctx, const void* w_f16, const float* x, int rows,
                           int cols, int batch, float* out);

/* apply_matvec (crates/sulimo-engine/src/forward_pass.rs:509-527): routes by tensor type.     */
/* SULIMO_GGML_Q4_0: w0 = scales, w1 = quants, x_q8 the Q8_0 activations (the AVX2-order       */
/* matvec, sulimo_cuda_gemv_q4_0_q8_0); SULIMO_GGML_F32 / F16: w0 = the raw weights, w1 unused, */
/* x_f32 the fp32 activations (sulimo_cuda_matvec_f32 / _f16).  Any other type: SULIMO_EINVAL. */
int sulimo_cuda_apply_matvec(sulimo_ctx* ctx, int ggml_type, const void* w0, const void* w1,
                             const void* x_q8, const float* x_f32, int rows, int cols, int batch,
                             float* out);

/* Integer per-block sums (debug / parity entry): out[b][r*(cols/32)+j] = sum_i (w_i-8)*x_i, */
/* the i32 `block_sum` of vec_dot_q4_0_q8_0_scalar (crates/sulimo-cpu/src/scalar.rs:189-199). */
int sulimo_cuda_block_sums_q4_0_q8_0(sulimo_ctx* ctx, const void* w_quants, const void* x_q8,
                                     int rows, int cols, int32_t* out);

/* ---------------------------------------------------------------------------------------- */
/* Q8_0 quantize — replaces quantize_f32_to_q8_0 (crates/sulimo-core/src/kv_cache.rs:162-192).*/
/* n % 32 == 0; byte-identical output.                                                        */
/* ---------------------------------------------------------------------------------------- */
int sulimo_cuda_quantize_q8_0(sulimo_ctx* ctx, const float* src, void* dst_q8, size_t n);

/* Q8_0 ring store — replaces enqueue_kv_store (crates/sulimo-ocl/src/prefill.rs:176-205,     */
/* kernel kv_store_q8_0, kernels/prefill.cl:72-116) and KvCache::store_key/store_value        */
/* (kv_cache.rs:93-110).  act is [n][blocks_per_pos*32] (f16 or f32); token t goes to ring    */
/* slot (start_pos+t) % capacity.  Bytes are identical to quantize_f32_to_q8_0 of the         */
/* activations widened to f32.                                                               */
int sulimo_cuda_kv_store_q8_0(sulimo_ctx* ctx, const void* act, int act_dtype, void* kv_ring,
                              size_t start_pos, size_t capacity, size_t blocks_per_pos,
                              size_t n);

/* Q4_0 row dequant — dequantize_q4_0_soa (crates/sulimo-core/src/repack.rs:107-131) for      */
/* `count` rows starting at `row0` of a [rows][cols] tensor; f32 out (bit-exact) or f16 out   */
/* (lookup_token_embedding_f16, crates/sulimo-engine/src/scheduler.rs:329-357).              */
int sulimo_cuda_dequantize_q4_0_rows(sulimo_ctx* ctx, const void* scales, const void* quants,
                                     int cols, const int32_t* row_ids, int count, void* out,
                                     int out_dtype);

/* Row-sharded projection layout (multi-GPU; the reference is single-device, the sharding of  */
/* its Q4_0 projections follows the SoA layout: rows [r*fs, r*fs+fs) of a [F][K] tensor are    */
/* the contiguous scales/quants subranges r*fs*(K/32) .. ).  `gathered` is the shard-major     */
/* result of an all-gather, [world][m_tokens][fs] elements of `elem_size` (2 = f16, 4 = f32)  */
/* bytes, shard world-1 holding F - (world-1)*fs valid rows; `out` receives the row-major     */
/* [m_tokens][F] layout of the single-device GEMM (gemm_q4_0_f16's out).                       */
int sulimo_cuda_unshard_rows(sulimo_ctx* ctx, const void* gathered, void* out, int world,
                             int m_tokens, size_t fs, size_t f, int elem_size);

/* ---- multi-GPU: the row-sharded projection with the all-gather fused into the GEMM --------- */
/* CUDA IPC of a library buffer (a cudaMalloc base): 64-byte handle out; another process opens  */
/* it with sulimo_cuda_ipc_open (peer access enabled) and closes it with sulimo_cuda_ipc_close.  */
int sulimo_cuda_ipc_handle(sulimo_buf* buf, void* handle_out);
int sulimo_cuda_ipc_open(sulimo_ctx* ctx, const void* handle, void** dev_ptr_out);
int sulimo_cuda_ipc_close(sulimo_ctx* ctx, void* dev_ptr);

/* This rank's rows [col0, col0 + m_local) of a Q4_0 [F][k] projection (m_local rows computed,  */
/* the first m_valid of them stored) for n tokens of x [n][k] f16, written straight into every  */
/* rank's row-major result Y[n][f_total] (out_bases: host array of `world` device pointers      */
/* valid in this process, i.e. opened IPC mappings) over NVLink, then one arrival per CTA added */
/* to every rank's counter (flags: host array of `world` device pointers).  *tiles_out = CTAs   */
/* of this launch.  A rank's Y is complete once its counter has grown by the sum of all ranks' */
/* CTAs: sulimo_cuda_wait_counter.  No split-K.  (The reference runs on one device; this is     */
/* the row-sharded form of enqueue_gemm_q4_0_f16, crates/sulimo-ocl/src/prefill.rs:69-105.)    */
/* Release handshake: `epoch` numbers the calls (1, 2, ... on every rank, modulo 2^32, never   */
/* 0) and release[r] is rank r's release word (a 4-byte device word, zero before the first     */
/* call).  The kernel sets this rank's word to `epoch` once the work enqueued on this          */
/* context's stream before the call has completed, and stores into rank r's Y only after       */
/* rank r's word has reached `epoch` (bounded wait, then SULIMO_EDEVICE).  So a rank's readers */
/* of the previous Y, enqueued on its stream before its next call, finish before any peer      */
/* overwrites it.                                                                              */
int sulimo_cuda_gemm_q4_0_f16_allgather(sulimo_ctx* ctx, const void* scales, const void* quants,
                                        const void* x, int m_local, int m_valid, int k, int n,
                                        int out_dtype, void* const* out_bases, size_t f_total,
                                        size_t col0, unsigned* const* flags,
                                        unsigned* const* release, int world, int rank,
                                        unsigned epoch, unsigned* tiles_out);

/* Enqueues a bounded wait (one thread; SULIMO_EDEVICE at the next synchronize after ~2 s)     */
/* until *flag (device) reaches `target` (modulo 2^32 arithmetic).                             */
int sulimo_cuda_wait_counter(sulimo_ctx* ctx, const unsigned* flag, unsigned target);

/* ---------------------------------------------------------------------------------------- */
/* Whole decode position — replaces forward_token                                            */
/* (crates/sulimo-engine/src/forward_pass.rs:190-417; its Llama, Qwen2 and Gemma 2 branches)  */
/* for a batch of independent sequences at the same position.  All pointers are device       */
/* pointers except `layers` (a host array of n_layers entries).  Weights are Q4_0 SoA (scales, */
/* quants), norms and biases f32 (biases may be NULL), each sequence has its own Q8_0 K and V  */
/* ring per layer: sequence s's ring starts kv_seq_stride bytes after sequence s-1's.          */
/* Gemma 2 (arch = SULIMO_ARCH_GEMMA2): embeddings scaled by sqrt(embd), every RMSNorm        */
/* weighted by (1 + w) (rmsnorm_gemma), the attention and FFN outputs RMS-normalized by        */
/* post_attn_norm / post_ffn_norm before their residual adds (layers without them add as the  */
/* other architectures do), GeGLU instead of SwiGLU, logits soft-capped by final_softcap       */
/* (<= 0: none); attn_softcap as for every architecture.                                      */
typedef struct sulimo_layer_desc {
    const void *attn_norm, *ffn_norm, *bq, *bk, *bv;
    const void *wq_scales, *wq_quants, *wk_scales, *wk_quants, *wv_scales, *wv_quants;
    const void *wo_scales, *wo_quants, *wg_scales, *wg_quants, *wu_scales, *wu_quants;
    const void *wd_scales, *wd_quants;
    void *k_ring, *v_ring;
    const void *post_attn_norm, *post_ffn_norm; /* [embd] f32 (Gemma 2) or NULL */
} sulimo_layer_desc;

#define SULIMO_ARCH_DEFAULT 0 /* Llama / Qwen2 */
#define SULIMO_ARCH_GEMMA2 1

typedef struct sulimo_model_desc {
    int n_layers, embd, ffn, head_count, head_count_kv, head_dim, vocab, rope_dim;
    int rope_mode; /* 0 = Norm (Llama), 1 = Neox (Qwen2, Gemma 2) */
    float eps, rope_base, attn_softcap;
    size_t kv_capacity, kv_seq_stride;
    const void *tok_scales, *tok_quants; /* token_embd [vocab][embd] */
    const void *out_scales, *out_quants; /* output [vocab][embd] (tied: token_embd) */
    const float* out_norm;
    const sulimo_layer_desc* layers;
    int arch;            /* SULIMO_ARCH_DEFAULT or SULIMO_ARCH_GEMMA2 */
    float final_softcap; /* final logit soft-capping (Gemma 2); <= 0: none */
} sulimo_model_desc;

/* Bytes of device scratch sulimo_cuda_forward_token needs for `batch` sequences (the          */
/* reference's ScratchBuffers, forward_pass.rs:150-186: allocated once, no per-token alloc).  */
size_t sulimo_cuda_forward_scratch_bytes(const sulimo_model_desc* model, int batch);

/* logits[batch][vocab] (fp32) for tokens[batch] (device int32) at position `pos` (context     */
/* pos+1); stores each sequence's K/V at ring slot pos % kv_capacity.                         */
int sulimo_cuda_forward_token(sulimo_ctx* ctx, const sulimo_model_desc* model,
                              const int32_t* tokens, int batch, size_t pos, float* logits,
                              void* scratch, size_t scratch_bytes);

/* Bytes of device scratch sulimo_cuda_prefill_ubatch needs for ubatches of up to n tokens.    */
size_t sulimo_cuda_prefill_scratch_bytes(const sulimo_model_desc* model, int n);

/* One prefill ubatch — replaces execute_prefill_ubatch (crates/sulimo-ocl/src/prefill.rs:     */
/* 337-566): tokens[n] (device int32) at positions start_pos .. start_pos+n-1 of ONE sequence  */
/* (kv_seq_stride unused), K/V stored into the rings, logits[vocab] (fp32) of the last token   */
/* (enqueue_logits_final, prefill.rs:300-330).  Requires start_pos + n <= kv_capacity.        */
/* The embeddings are the f16 rows of lookup_token_embedding_f16 (scheduler.rs:329-374), as   */
/* the reference's engine writes them (engine.rs:249-256).  Unlike the reference's GPU ubatch  */
/* this one applies the QKV biases (as forward_token does) and keeps the residual stream in    */
/* fp32; the GEMM activations are f16 like the reference's.  Like the reference's GPU ubatch, */
/* it has no Gemma 2 steps: a Gemma 2 model is rejected (SULIMO_EINVAL) and prefills through  */
/* sulimo_cuda_forward_token per token, as the reference's CPU prefill does.                   */
int sulimo_cuda_prefill_ubatch(sulimo_ctx* ctx, const sulimo_model_desc* model,
                               const int32_t* tokens, int n, size_t start_pos, float* logits,
                               void* scratch, size_t scratch_bytes);

/* The same ubatch for a caller that has written the embeddings itself — the reference's      */
/* contract exactly (execute_prefill_ubatch reads them from scratch.x, prefill.rs:337-566):     */
/* x_f16 [n][embd] f16 on the device (8-byte aligned), not modified.                          */
int sulimo_cuda_prefill_ubatch_x(sulimo_ctx* ctx, const sulimo_model_desc* model,
                                 const void* x_f16, int n, size_t start_pos, float* logits,
                                 void* scratch, size_t scratch_bytes);

/* Context repack on capacity overflow — replaces repack_context (crates/sulimo-engine/src/     */
/* scheduler.rs:316-326) and the re-prefill that follows it (engine.rs:226-239), on the device: */
/* the plan keeps the first sys_len = min(clamp(capacity/8, 4, 64), n_past) tokens and the last */
/* recent_len = min(capacity/2, n_past - sys_len); the entry point gathers those tokens of      */
/* past_tokens[n_past] (device int32) into new_tokens (device, not overlapping), re-prefills    */
/* them from position 0 in ubatches of at most `ubatch` tokens (sulimo_cuda_prefill_ubatch;     */
/* scratch >= sulimo_cuda_prefill_scratch_bytes(model, ubatch)), leaves the last token's logits */
/* in logits[vocab] and the new position (sys_len + recent_len) in *new_pos_out.  No host round */
/* trip: the counts are functions of n_past and kv_capacity.                                   */
void sulimo_cuda_repack_context_plan(size_t n_past, size_t capacity, size_t* sys_len,
                                     size_t* recent_len);
int sulimo_cuda_repack_context(sulimo_ctx* ctx, const sulimo_model_desc* model,
                               const int32_t* past_tokens, size_t n_past, int32_t* new_tokens,
                               int ubatch, float* logits, void* scratch, size_t scratch_bytes,
                               size_t* new_pos_out);

/* GGUF Q4_0 blocks to the SoA layout on the device — replaces repack_q4_0_aos_to_soa           */
/* (crates/sulimo-core/src/repack.rs:45-81): src_aos = src_len bytes of 18-byte blocks          */
/* [d: f16][qs: 16 B] (device, 2-byte aligned), dst_scales[nb] f16 (2-byte aligned),             */
/* dst_quants[nb][16] (16-byte aligned); *num_blocks_out = nb.  The reference's errors:         */
/* src_len % 18 != 0 (InvalidAosLength), scales_len < 2 nb (ScalesBufferTooSmall), quants_len  */
/* < 16 nb (QuantsBufferTooSmall) -> SULIMO_EINVAL.                                             */
int sulimo_cuda_repack_q4_0_aos_to_soa(sulimo_ctx* ctx, const void* src_aos, size_t src_len,
                                       void* dst_scales, size_t scales_len, void* dst_quants,
                                       size_t quants_len, size_t* num_blocks_out);

/* Causal GQA prefill attention over one layer's Q8_0 ring — replaces                          */
/* causal_gqa_attention_prefill (kernels/prefill.cl:120-237, enqueue_attention_prefill):       */
/* q [n][head_count][head_dim] fp32 (after RoPE; the reference passes f16), token t at         */
/* position start_pos + t attends to positions 0 .. start_pos + t (slot p % capacity);         */
/* out [n][head_count][head_dim] f16.  head_dim 64 or 128.  When the (128-token tile, head)    */
/* pairs are fewer than the SMs, a tile's keys are split over several CTAs whose partials      */
/* live in the context workspace (grown, after a stream synchronisation, on first need) and    */
/* are combined by a second kernel.                                                           */
int sulimo_cuda_attn_prefill_q8_0(sulimo_ctx* ctx, const float* q, const void* k_ring,
                                  const void* v_ring, size_t start_pos, size_t capacity, int n,
                                  int head_count, int head_count_kv, int head_dim, void* out);

/* Greedy pick: out[r] = first index of the maximum of row r of x[rows][cols].                */
int sulimo_cuda_argmax_rows(sulimo_ctx* ctx, const float* x, int rows, int cols, int32_t* out);

/* ---------------------------------------------------------------------------------------- */
/* Decode attention — replaces causal_gqa_decode_scalar_ext                                   */
/* (crates/sulimo-cpu/src/scalar.rs:287-359) over the KvCache ring (kv_cache.rs:114-128).     */
/* q: [batch][head_count][head_dim] f32; out: same shape.  Sequence s reads its K/V rings at  */
/* k_ring + s*seq_stride_bytes (v likewise); position p reads slot p % capacity; positions    */
/* 0..context_len-1 are attended.  softcap <= 0 disables soft-capping.  Split-K over the      */
/* context (partial max/sum/output in the context workspace, combined by a second kernel).    */
/* ---------------------------------------------------------------------------------------- */
int sulimo_cuda_attn_decode_q8_0(sulimo_ctx* ctx, const float* q, const void* k_ring,
                                 const void* v_ring, size_t seq_stride_bytes, size_t capacity,
                                 size_t context_len, int head_count, int head_count_kv,
                                 int head_dim, int batch, float softcap, float* out);

/* Decode attention that allocates nothing.  No counterpart in the reference: it exists for
 * callers that must not allocate device memory — a decode loop held to a no-allocation rule
 * per token (the reference's CPU decode makes zero heap allocations), or a host that plans all
 * device memory up front from a fixed budget.  Same arguments and results as
 * sulimo_cuda_attn_decode_q8_0, but the split-K partials live in a fixed 2 MiB array compiled
 * into the library (reserved on every GPU that loads it, until the process exits) instead of
 * the context workspace.  Limit: batch * head_count * ceil(context_len / 256) * (head_dim + 2)
 * <= 524288 floats, else SULIMO_EINVAL; within the limit the split count is reduced to fit.
 * The first call on a device looks up the array's device address (cudaGetSymbolAddress) and
 * caches it; make that first call before any stream capture.  All calls share the array and it
 * keeps the last call's contents (every call overwrites the part it reads, so nothing needs
 * clearing); calls that overlap on the GPU — different streams or contexts of one device —
 * race on it and must be serialized by the caller. */
int sulimo_cuda_attn_decode_q8_0_noalloc(sulimo_ctx* ctx, const float* q, const void* k_ring,
                                         const void* v_ring, size_t seq_stride_bytes,
                                         size_t capacity, size_t context_len, int head_count,
                                         int head_count_kv, int head_dim, int batch,
                                         float softcap, float* out);

#if defined(__GNUC__)
#pragma GCC visibility pop
#endif

#ifdef __cplusplus
}
#endif
#endif /* SULIMO_CUDA_H */
