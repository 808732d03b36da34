/*
 * sulimo_oracle.c — CPU restatement of Sulimo's quantized-matmul hot path.
 *
 * TEST INFRASTRUCTURE ONLY (the checker and the timed CPU baseline); the
 * product library never links it.  Each function cites the reference lines
 * (paths relative to the reference repository root) it restates.  Built with
 * -O2 -mavx2 -mfma -mf16c -ffp-contract=off so that, like the Rust reference,
 * no multiply-add is fused unless the reference calls an FMA intrinsic.
 */
#include "sulimo_oracle.h"

#include <immintrin.h>
#include <math.h>
#include <stdlib.h>
#include <pthread.h>
#include <string.h>

/* ------------------------------------------------------------------ */
/* f16 <-> f32 (half 2.7.1: IEEE binary16, round-to-nearest-even)      */
/* ------------------------------------------------------------------ */
uint16_t oracle_f32_to_f16(float x) {
    return (uint16_t)_cvtss_sh(x, _MM_FROUND_TO_NEAREST_INT);
}

float oracle_f16_to_f32(uint16_t h) { return _cvtsh_ss(h); }

void oracle_f32_to_f16_array(const float* src, uint16_t* dst, size_t n) {
    for (size_t i = 0; i < n; i++) dst[i] = oracle_f32_to_f16(src[i]);
}

void oracle_f16_to_f32_array(const uint16_t* src, float* dst, size_t n) {
    for (size_t i = 0; i < n; i++) dst[i] = oracle_f16_to_f32(src[i]);
}

static inline float le_f16(const uint8_t* p) {
    return oracle_f16_to_f32((uint16_t)(p[0] | ((uint16_t)p[1] << 8)));
}

/* ------------------------------------------------------------------ */
/* Q4_0 repack / dequant                                               */
/* ------------------------------------------------------------------ */

/* repack_q4_0_aos_to_soa — crates/sulimo-core/src/repack.rs:45-81 */
long oracle_repack_q4_0_aos_to_soa(const uint8_t* src_aos, size_t src_len,
                                   uint8_t* dst_scales, size_t scales_len,
                                   uint8_t* dst_quants, size_t quants_len) {
    if (src_len % 18 != 0) return -1;
    size_t nb = src_len / 18;
    if (scales_len < nb * 2) return -2;
    if (quants_len < nb * 16) return -3;
    for (size_t b = 0; b < nb; b++) {
        memcpy(dst_scales + b * 2, src_aos + b * 18, 2);
        memcpy(dst_quants + b * 16, src_aos + b * 18 + 2, 16);
    }
    return (long)nb;
}

/* dequantize_q4_0_aos — repack.rs:84-104 */
void oracle_dequantize_q4_0_aos(const uint8_t* src_aos, size_t num_blocks, float* dst) {
    for (size_t b = 0; b < num_blocks; b++) {
        const uint8_t* blk = src_aos + b * 18;
        float scale = le_f16(blk);
        const uint8_t* qs = blk + 2;
        for (int i = 0; i < 16; i++) {
            int v0 = (qs[i] & 0x0F) - 8;
            int v1 = (qs[i] >> 4) - 8;
            dst[b * 32 + i] = (float)v0 * scale;
            dst[b * 32 + i + 16] = (float)v1 * scale;
        }
    }
}

/* dequantize_q4_0_soa — repack.rs:107-131 */
void oracle_dequantize_q4_0_soa(const uint8_t* scales, const uint8_t* quants,
                                size_t num_blocks, float* dst) {
    for (size_t b = 0; b < num_blocks; b++) {
        float scale = le_f16(scales + b * 2);
        const uint8_t* qs = quants + b * 16;
        for (int i = 0; i < 16; i++) {
            int v0 = (qs[i] & 0x0F) - 8;
            int v1 = (qs[i] >> 4) - 8;
            dst[b * 32 + i] = (float)v0 * scale;
            dst[b * 32 + i + 16] = (float)v1 * scale;
        }
    }
}

/* lookup_token_embedding_f16 — crates/sulimo-engine/src/scheduler.rs:329-357.
 * `d * f16::from_f32(q)` in half 2.7.1 is f16(f32(d) * f32(q)), one RNE rounding. */
void oracle_lookup_token_embedding_f16(const uint8_t* scales, const uint8_t* quants,
                                       size_t embd_dim, uint32_t token_id, uint16_t* out_f16) {
    size_t bpr = embd_dim / 32;
    const uint8_t* rs = scales + (size_t)token_id * bpr * 2;
    const uint8_t* rq = quants + (size_t)token_id * bpr * 16;
    for (size_t b = 0; b < bpr; b++) {
        float d = le_f16(rs + b * 2);
        const uint8_t* q = rq + b * 16;
        for (int i = 0; i < 16; i++) {
            int lo = (q[i] & 0x0F) - 8;
            int hi = ((q[i] >> 4) & 0x0F) - 8;
            out_f16[b * 32 + i] = oracle_f32_to_f16(d * oracle_f16_to_f32(oracle_f32_to_f16((float)lo)));
            out_f16[b * 32 + 16 + i] =
                oracle_f32_to_f16(d * oracle_f16_to_f32(oracle_f32_to_f16((float)hi)));
        }
    }
}

/* ------------------------------------------------------------------ */
/* Q8_0                                                                */
/* ------------------------------------------------------------------ */

/* quantize_f32_to_q8_0 — crates/sulimo-core/src/kv_cache.rs:162-192 */
void oracle_quantize_f32_to_q8_0(const float* src, size_t n, uint8_t* dst_q8) {
    size_t nb = n / 32;
    for (size_t b = 0; b < nb; b++) {
        const float* s = src + b * 32;
        uint8_t* d8 = dst_q8 + b * 34;
        float max_abs = 0.0f;
        for (int i = 0; i < 32; i++) {
            float a = fabsf(s[i]);
            if (a > max_abs) max_abs = a;
        }
        float d = max_abs / 127.0f;
        uint16_t dh = oracle_f32_to_f16(d);
        d8[0] = (uint8_t)(dh & 0xFF);
        d8[1] = (uint8_t)(dh >> 8);
        float id = (d != 0.0f) ? 1.0f / d : 0.0f;
        for (int i = 0; i < 32; i++) {
            float q = roundf(s[i] * id);
            /* f32::clamp(-128, 127) then `as i8` (saturating; NaN -> 0) */
            if (q != q) q = 0.0f;
            if (q < -128.0f) q = -128.0f;
            if (q > 127.0f) q = 127.0f;
            d8[2 + i] = (uint8_t)(int8_t)q;
        }
    }
}

/* dequantize_q8_0_to_f32 — kv_cache.rs:195-208 */
void oracle_dequantize_q8_0_to_f32(const uint8_t* src_q8, size_t num_blocks, float* dst) {
    for (size_t b = 0; b < num_blocks; b++) {
        const uint8_t* blk = src_q8 + b * 34;
        float scale = le_f16(blk);
        for (int i = 0; i < 32; i++) dst[b * 32 + i] = (float)(int8_t)blk[2 + i] * scale;
    }
}

/* kv_store_q8_0 — kernels/prefill.cl:72-116, checked against the CPU quantizer exactly as
 * crates/sulimo-ocl/tests/test_prefill.rs:126-150 does (f16 activations widened to f32). */
void oracle_kv_store_q8_0(const uint16_t* act_f16, uint8_t* kv, size_t start_pos,
                          size_t capacity, size_t blocks_per_pos, size_t n) {
    size_t bytes_per_pos = blocks_per_pos * 34;
    float blk[32];
    for (size_t t = 0; t < n; t++) {
        size_t ring = (start_pos + t) % capacity;
        for (size_t b = 0; b < blocks_per_pos; b++) {
            for (int i = 0; i < 32; i++)
                blk[i] = oracle_f16_to_f32(act_f16[(t * blocks_per_pos + b) * 32 + i]);
            oracle_quantize_f32_to_q8_0(blk, 32, kv + ring * bytes_per_pos + b * 34);
        }
    }
}

/* KvCache::store_key / store_value — kv_cache.rs:93-110 */
void oracle_kv_store_f32(const float* vec, uint8_t* kv, size_t pos, size_t capacity,
                         size_t blocks_per_pos) {
    size_t ring = pos % capacity;
    oracle_quantize_f32_to_q8_0(vec, blocks_per_pos * 32, kv + ring * blocks_per_pos * 34);
}

/* ------------------------------------------------------------------ */
/* Q4_0 x Q8_0                                                         */
/* ------------------------------------------------------------------ */

/* vec_dot_q4_0_q8_0_scalar — crates/sulimo-cpu/src/scalar.rs:173-205 */
float oracle_vec_dot_q4_0_q8_0_scalar(const uint8_t* w_scales, const uint8_t* w_quants,
                                      const uint8_t* x_q8, size_t num_blocks) {
    float total = 0.0f;
    for (size_t b = 0; b < num_blocks; b++) {
        float ws = le_f16(w_scales + b * 2);
        float xs = le_f16(x_q8 + b * 34);
        float d = ws * xs;
        const uint8_t* wq = w_quants + b * 16;
        const uint8_t* xq = x_q8 + b * 34 + 2;
        int32_t bs = 0;
        for (int i = 0; i < 16; i++) {
            int w0 = (wq[i] & 0x0F) - 8;
            int w1 = (wq[i] >> 4) - 8;
            int x0 = (int8_t)xq[i];
            int x1 = (int8_t)xq[i + 16];
            bs += w0 * x0 + w1 * x1;
        }
        total += (float)bs * d;
    }
    return total;
}

/* matvec_q4_0_q8_0_scalar — scalar.rs:208-225 */
void oracle_matvec_q4_0_q8_0_scalar(const uint8_t* w_scales, const uint8_t* w_quants,
                                    const uint8_t* x_q8, size_t rows, size_t cols, float* out) {
    size_t nb = cols / 32;
    for (size_t r = 0; r < rows; r++)
        out[r] = oracle_vec_dot_q4_0_q8_0_scalar(w_scales + r * nb * 2, w_quants + r * nb * 16,
                                                 x_q8, nb);
}

/* hsum_256 — crates/sulimo-cpu/src/avx2.rs:333-342 */
static inline float hsum_256(__m256 v) {
    __m128 hi = _mm256_extractf128_ps(v, 1);
    __m128 lo = _mm256_castps256_ps128(v);
    __m128 sum128 = _mm_add_ps(lo, hi);
    __m128 shuf = _mm_movehdup_ps(sum128);
    __m128 sums = _mm_add_ps(sum128, shuf);
    __m128 shuf2 = _mm_movehl_ps(sums, sums);
    __m128 fin = _mm_add_ss(sums, shuf2);
    return _mm_cvtss_f32(fin);
}

/* vec_dot_q4_0_q8_0_avx2 — avx2.rs:113-164; same intrinsics in the same order. */
float oracle_vec_dot_q4_0_q8_0_avx2(const uint8_t* w_scales, const uint8_t* w_quants,
                                    const uint8_t* x_q8, size_t num_blocks) {
    __m256 acc = _mm256_setzero_ps();
    for (size_t b = 0; b < num_blocks; b++) {
        float w_scale = le_f16(w_scales + b * 2);
        float x_scale = le_f16(x_q8 + b * 34);
        float d = w_scale * x_scale;

        __m128i w128 = _mm_loadu_si128((const __m128i*)(w_quants + b * 16));
        __m128i mask_low = _mm_set1_epi8(0x0F);
        __m128i eight = _mm_set1_epi8(8);
        __m128i w_low = _mm_sub_epi8(_mm_and_si128(w128, mask_low), eight);
        __m128i w_high = _mm_sub_epi8(_mm_and_si128(_mm_srli_epi16(w128, 4), mask_low), eight);
        __m256i w256 = _mm256_set_m128i(w_high, w_low);

        __m256i x256 = _mm256_loadu_si256((const __m256i*)(x_q8 + b * 34 + 2));

        __m256i w_lo_16 = _mm256_cvtepi8_epi16(_mm256_extracti128_si256(w256, 0));
        __m256i w_hi_16 = _mm256_cvtepi8_epi16(_mm256_extracti128_si256(w256, 1));
        __m256i x_lo_16 = _mm256_cvtepi8_epi16(_mm256_extracti128_si256(x256, 0));
        __m256i x_hi_16 = _mm256_cvtepi8_epi16(_mm256_extracti128_si256(x256, 1));

        __m256i prod_lo = _mm256_madd_epi16(w_lo_16, x_lo_16);
        __m256i prod_hi = _mm256_madd_epi16(w_hi_16, x_hi_16);
        __m256i sum32 = _mm256_add_epi32(prod_lo, prod_hi);
        __m256 sum_ps = _mm256_cvtepi32_ps(sum32);

        __m256 d_vec = _mm256_set1_ps(d);
        acc = _mm256_fmadd_ps(sum_ps, d_vec, acc);
    }
    return hsum_256(acc);
}

/* matvec_q4_0_q8_0_avx2 — avx2.rs:172-189 (dispatch_matvec_q4_0_q8_0, avx2.rs:17-37,
 * selects this on any AVX2+FMA host). */
void oracle_matvec_q4_0_q8_0_avx2(const uint8_t* w_scales, const uint8_t* w_quants,
                                  const uint8_t* x_q8, size_t rows, size_t cols, float* out) {
    size_t nb = cols / 32;
    for (size_t r = 0; r < rows; r++)
        out[r] = oracle_vec_dot_q4_0_q8_0_avx2(w_scales + r * nb * 2, w_quants + r * nb * 16,
                                               x_q8, nb);
}

typedef struct {
    const uint8_t* ws;
    const uint8_t* wq;
    const uint8_t* x;
    size_t r0, r1, cols;
    float* out;
} mv_job;

static void* mv_worker(void* arg) {
    mv_job* j = (mv_job*)arg;
    size_t nb = j->cols / 32;
    for (size_t r = j->r0; r < j->r1; r++)
        j->out[r] = oracle_vec_dot_q4_0_q8_0_avx2(j->ws + r * nb * 2, j->wq + r * nb * 16, j->x, nb);
    return NULL;
}

void oracle_matvec_q4_0_q8_0_avx2_mt(const uint8_t* w_scales, const uint8_t* w_quants,
                                     const uint8_t* x_q8, size_t rows, size_t cols, float* out,
                                     int threads) {
    if (threads <= 1) {
        oracle_matvec_q4_0_q8_0_avx2(w_scales, w_quants, x_q8, rows, cols, out);
        return;
    }
    if (threads > 256) threads = 256;
    pthread_t tid[256];
    mv_job jobs[256];
    size_t per = (rows + (size_t)threads - 1) / (size_t)threads;
    int started = 0;
    for (int t = 0; t < threads; t++) {
        size_t r0 = (size_t)t * per, r1 = r0 + per;
        if (r0 >= rows) break;
        if (r1 > rows) r1 = rows;
        jobs[t] = (mv_job){w_scales, w_quants, x_q8, r0, r1, cols, out};
        if (pthread_create(&tid[t], NULL, mv_worker, &jobs[t]) != 0) {
            mv_worker(&jobs[t]);
            tid[t] = 0;
        }
        started = t + 1;
    }
    for (int t = 0; t < started; t++)
        if (tid[t]) pthread_join(tid[t], NULL);
}

/* Integer per-block Q4_0 x Q8_0 sums — the `block_sum` of scalar.rs:189-199, which equals the
 * sum of the eight i32 lanes of `sum32` in avx2.rs:146-155. */
void oracle_block_sums_q4_0_q8_0(const uint8_t* w_scales, const uint8_t* w_quants,
                                 const uint8_t* x_q8, size_t rows, size_t cols, int32_t* out) {
    (void)w_scales;
    size_t nb = cols / 32;
    for (size_t r = 0; r < rows; r++)
        for (size_t b = 0; b < nb; b++) {
            const uint8_t* wq = w_quants + (r * nb + b) * 16;
            const uint8_t* xq = x_q8 + b * 34 + 2;
            int32_t bs = 0;
            for (int i = 0; i < 16; i++) {
                bs += ((wq[i] & 0x0F) - 8) * (int8_t)xq[i] + ((wq[i] >> 4) - 8) * (int8_t)xq[i + 16];
            }
            out[r * nb + b] = bs;
        }
}

/* ------------------------------------------------------------------ */
/* Prefill GEMM                                                        */
/* ------------------------------------------------------------------ */

/* One output of gemm_q4_0_f16_scalar_reference — crates/sulimo-ocl/src/gemm.rs:115-142 */
static inline float gemm_dot(const uint16_t* scales, const uint8_t* quants, const float* xr,
                             size_t row_m, size_t nbr) {
    float acc = 0.0f;
    size_t off = row_m * nbr;
    for (size_t b = 0; b < nbr; b++) {
        float d = oracle_f16_to_f32(scales[off + b]);
        const uint8_t* q = quants + (off + b) * 16;
        const float* xs = xr + b * 32;
        float bsum = 0.0f;
        for (int i = 0; i < 16; i++) {
            float ql = (float)((q[i] & 0x0F) - 8);
            float qh = (float)(((q[i] >> 4) & 0x0F) - 8);
            bsum += xs[i] * ql + xs[16 + i] * qh;
        }
        acc += bsum * d;
    }
    return acc;
}

/* gemm_q4_0_f16_scalar_reference — gemm.rs:106-147: out[n][m] = f16(acc) */
void oracle_gemm_q4_0_f16_scalar_reference(const uint16_t* scales, const uint8_t* quants,
                                           const uint16_t* x, size_t m, size_t k, size_t n,
                                           uint16_t* out) {
    size_t nbr = k / 32;
    float* xr = (float*)__builtin_alloca(k * sizeof(float));
    for (size_t t = 0; t < n; t++) {
        for (size_t i = 0; i < k; i++) xr[i] = oracle_f16_to_f32(x[t * k + i]);
        for (size_t r = 0; r < m; r++) out[t * m + r] = oracle_f32_to_f16(gemm_dot(scales, quants, xr, r, nbr));
    }
}

typedef struct {
    const uint16_t* scales;
    const uint8_t* quants;
    const uint16_t* x;
    size_t m, k, n, t0, t1;
    float* out;
} gemm_job;

static void* gemm_worker(void* arg) {
    gemm_job* j = (gemm_job*)arg;
    size_t nbr = j->k / 32;
    float* xr = (float*)__builtin_alloca(j->k * sizeof(float));
    for (size_t t = j->t0; t < j->t1; t++) {
        for (size_t i = 0; i < j->k; i++) xr[i] = oracle_f16_to_f32(j->x[t * j->k + i]);
        for (size_t r = 0; r < j->m; r++) j->out[t * j->m + r] = gemm_dot(j->scales, j->quants, xr, r, nbr);
    }
    return NULL;
}

/* Same arithmetic with fp32 results (logits_f16_output, kernels/prefill.cl:269-308, and the
 * test oracle of crates/sulimo-ocl/tests/test_prefill.rs:781-800).  Token rows are split across
 * `threads` POSIX threads; each output is computed exactly as gemm_dot. */
void oracle_gemm_q4_0_f16_scalar_f32out(const uint16_t* scales, const uint8_t* quants,
                                        const uint16_t* x, size_t m, size_t k, size_t n,
                                        float* out, int threads) {
    if (threads < 1) threads = 1;
    if (threads > 256) threads = 256;
    pthread_t tid[256];
    gemm_job jobs[256];
    size_t per = (n + (size_t)threads - 1) / (size_t)threads;
    int started = 0;
    for (int t = 0; t < threads; t++) {
        size_t t0 = (size_t)t * per, t1 = t0 + per;
        if (t0 >= n) break;
        if (t1 > n) t1 = n;
        jobs[t] = (gemm_job){scales, quants, x, m, k, n, t0, t1, out};
        if (threads == 1 || pthread_create(&tid[t], NULL, gemm_worker, &jobs[t]) != 0) {
            gemm_worker(&jobs[t]);
            tid[t] = 0;
        }
        started = t + 1;
    }
    for (int t = 0; t < started; t++)
        if (tid[t]) pthread_join(tid[t], NULL);
}

/* CPU prefill of one projection: per token, quantize_f32_to_q8_0 then the AVX2 matvec, as
 * forward_token does for every prompt token when prefill runs on the CPU
 * (crates/sulimo-engine/src/engine.rs:287-318, forward_pass.rs:227-247). */
typedef struct {
    const uint8_t* ws;
    const uint8_t* wq;
    const float* x;
    size_t m, k, t0, t1;
    float* out;
} pf_job;

static void* pf_worker(void* arg) {
    pf_job* j = (pf_job*)arg;
    size_t nb = j->k / 32;
    uint8_t* q8 = (uint8_t*)__builtin_alloca(nb * 34);
    for (size_t t = j->t0; t < j->t1; t++) {
        oracle_quantize_f32_to_q8_0(j->x + t * j->k, j->k, q8);
        oracle_matvec_q4_0_q8_0_avx2(j->ws, j->wq, q8, j->m, j->k, j->out + t * j->m);
    }
    return NULL;
}

void oracle_cpu_prefill_projection(const uint8_t* w_scales, const uint8_t* w_quants,
                                   const float* x, size_t m, size_t k, size_t n, float* out,
                                   int threads) {
    if (threads < 1) threads = 1;
    if (threads > 256) threads = 256;
    pthread_t tid[256];
    pf_job jobs[256];
    size_t per = (n + (size_t)threads - 1) / (size_t)threads;
    int started = 0;
    for (int t = 0; t < threads; t++) {
        size_t t0 = (size_t)t * per, t1 = t0 + per;
        if (t0 >= n) break;
        if (t1 > n) t1 = n;
        jobs[t] = (pf_job){w_scales, w_quants, x, m, k, t0, t1, out};
        if (threads == 1 || pthread_create(&tid[t], NULL, pf_worker, &jobs[t]) != 0) {
            pf_worker(&jobs[t]);
            tid[t] = 0;
        }
        started = t + 1;
    }
    for (int t = 0; t < started; t++)
        if (tid[t]) pthread_join(tid[t], NULL);
}

/* ------------------------------------------------------------------ */
/* small ops                                                           */
/* ------------------------------------------------------------------ */

/* rmsnorm_scalar — crates/sulimo-cpu/src/scalar.rs:23-38 */
void oracle_rmsnorm_scalar(const float* x, const float* w, size_t len, float eps, float* out) {
    float sum_sq = 0.0f;
    for (size_t i = 0; i < len; i++) sum_sq += x[i] * x[i];
    float mean = sum_sq / (float)len;
    float scale = 1.0f / sqrtf(mean + eps);
    for (size_t i = 0; i < len; i++) out[i] = x[i] * scale * w[i];
}

/* rmsnorm_avx2 — crates/sulimo-cpu/src/avx2.rs:197-226 */
void oracle_rmsnorm_avx2(const float* x, const float* w, size_t len, float eps, float* out) {
    size_t chunks = len / 8;
    __m256 ssv = _mm256_setzero_ps();
    for (size_t i = 0; i < chunks; i++) {
        __m256 xv = _mm256_loadu_ps(x + i * 8);
        ssv = _mm256_fmadd_ps(xv, xv, ssv);
    }
    float sum_sq = hsum_256(ssv);
    for (size_t i = chunks * 8; i < len; i++) sum_sq += x[i] * x[i];
    float mean = sum_sq / (float)len;
    float scale = 1.0f / sqrtf(mean + eps);
    __m256 sv = _mm256_set1_ps(scale);
    for (size_t i = 0; i < chunks; i++) {
        __m256 xv = _mm256_loadu_ps(x + i * 8);
        __m256 wv = _mm256_loadu_ps(w + i * 8);
        _mm256_storeu_ps(out + i * 8, _mm256_mul_ps(_mm256_mul_ps(xv, sv), wv));
    }
    for (size_t i = chunks * 8; i < len; i++) out[i] = x[i] * scale * w[i];
}

/* rmsnorm_gemma_avx2 — avx2.rs:236-268: the same sum of squares as rmsnorm_avx2, output
 * (x * scale) * (1 + w) */
void oracle_rmsnorm_gemma_avx2(const float* x, const float* w, size_t len, float eps, float* out) {
    size_t chunks = len / 8;
    __m256 ssv = _mm256_setzero_ps();
    for (size_t i = 0; i < chunks; i++) {
        __m256 xv = _mm256_loadu_ps(x + i * 8);
        ssv = _mm256_fmadd_ps(xv, xv, ssv);
    }
    float sum_sq = hsum_256(ssv);
    for (size_t i = chunks * 8; i < len; i++) sum_sq += x[i] * x[i];
    float mean = sum_sq / (float)len;
    float scale = 1.0f / sqrtf(mean + eps);
    __m256 sv = _mm256_set1_ps(scale);
    __m256 ones = _mm256_set1_ps(1.0f);
    for (size_t i = 0; i < chunks; i++) {
        __m256 xv = _mm256_loadu_ps(x + i * 8);
        __m256 gw = _mm256_add_ps(ones, _mm256_loadu_ps(w + i * 8));
        _mm256_storeu_ps(out + i * 8, _mm256_mul_ps(_mm256_mul_ps(xv, sv), gw));
    }
    for (size_t i = chunks * 8; i < len; i++) out[i] = x[i] * scale * (1.0f + w[i]);
}

/* geglu_scalar — scalar.rs:77-89: out = gelu(gate) * up, gelu the tanh form */
void oracle_geglu_scalar(const float* gate, const float* up, float* out, size_t n) {
    const float sqrt_2_over_pi = 0.7978846f;
    for (size_t i = 0; i < n; i++) {
        float x = gate[i];
        float cube = x * x * x;
        float inner = sqrt_2_over_pi * (x + 0.044715f * cube);
        float gelu_x = 0.5f * x * (1.0f + tanhf(inner));
        out[i] = gelu_x * up[i];
    }
}

/* logit_softcap_scalar — scalar.rs:63-71: v = tanh(v / cap) * cap, in place; cap <= 0: none */
void oracle_logit_softcap_scalar(float* v, size_t n, float cap) {
    if (cap <= 0.0f) return;
    float inv_cap = 1.0f / cap;
    for (size_t i = 0; i < n; i++) v[i] = tanhf(v[i] * inv_cap) * cap;
}

/* rope_head_scalar — scalar.rs:92-130 (no freq_factors); mode 0 = Norm, 1 = Neox */
void oracle_rope_head_scalar(float* vec, size_t pos, size_t rope_dim, float freq_base, int mode) {
    size_t half_dim = rope_dim / 2;
    for (size_t i = 0; i < half_dim; i++) {
        float freq = 1.0f / powf(freq_base, (float)(2 * i) / (float)rope_dim);
        float theta = (float)pos * freq;
        float c = cosf(theta), s = sinf(theta);
        if (mode == 0) {
            float v0 = vec[2 * i], v1 = vec[2 * i + 1];
            vec[2 * i] = v0 * c - v1 * s;
            vec[2 * i + 1] = v0 * s + v1 * c;
        } else {
            float v0 = vec[i], v1 = vec[i + half_dim];
            vec[i] = v0 * c - v1 * s;
            vec[i + half_dim] = v0 * s + v1 * c;
        }
    }
}

/* softmax_scalar — scalar.rs:133-158 */
void oracle_softmax_scalar(float* x, size_t n) {
    if (n == 0) return;
    float mx = x[0];
    for (size_t i = 1; i < n; i++)
        if (x[i] > mx) mx = x[i];
    float sum = 0.0f;
    for (size_t i = 0; i < n; i++) {
        float e = expf(x[i] - mx);
        x[i] = e;
        sum += e;
    }
    if (sum > 0.0f) {
        float inv = 1.0f / sum;
        for (size_t i = 0; i < n; i++) x[i] *= inv;
    }
}

/* swiglu_scalar — scalar.rs:161-170 */
void oracle_swiglu_scalar(const float* gate, const float* up, float* out, size_t n) {
    for (size_t i = 0; i < n; i++) {
        float g = gate[i];
        float silu = g / (1.0f + expf(-g));
        out[i] = silu * up[i];
    }
}

/* causal_gqa_decode_scalar_ext — scalar.rs:287-359, K/V addressed through the ring as
 * KvCache::key_ptr / value_ptr do (kv_cache.rs:114-128). */
void oracle_causal_gqa_decode(const float* q, const uint8_t* k_ring, const uint8_t* v_ring,
                              size_t capacity, size_t context_len, size_t head_count,
                              size_t head_count_kv, size_t head_dim, float* scores_buf,
                              float* out, float softcap) {
    size_t heads_per_kv = head_count / head_count_kv;
    float scale = 1.0f / sqrtf((float)head_dim);
    size_t head_bytes = (head_dim / 32) * 34;
    size_t bytes_per_pos = head_count_kv * head_bytes;
    float* deq = (float*)__builtin_alloca(head_dim * sizeof(float));
    /* the reference's dequant buffer starts zeroed (test_prefill.rs:690, ScratchBuffers); with
     * head_dim < 32 no block is dequantised into it and the zeros are what is read */
    memset(deq, 0, head_dim * sizeof(float));
    for (size_t h = 0; h < head_count; h++) {
        size_t kvh = h / heads_per_kv;
        const float* qh = q + h * head_dim;
        for (size_t p = 0; p < context_len; p++) {
            const uint8_t* kp = k_ring + (p % capacity) * bytes_per_pos + kvh * head_bytes;
            oracle_dequantize_q8_0_to_f32(kp, head_dim / 32, deq);
            float dot = 0.0f;
            for (size_t d = 0; d < head_dim; d++) dot += qh[d] * deq[d];
            float score = dot * scale;
            if (softcap > 0.0f) score = tanhf(score / softcap) * softcap;
            scores_buf[p] = score;
        }
        oracle_softmax_scalar(scores_buf, context_len);
        float* oh = out + h * head_dim;
        for (size_t d = 0; d < head_dim; d++) oh[d] = 0.0f;
        for (size_t p = 0; p < context_len; p++) {
            const uint8_t* vp = v_ring + (p % capacity) * bytes_per_pos + kvh * head_bytes;
            oracle_dequantize_q8_0_to_f32(vp, head_dim / 32, deq);
            float wgt = scores_buf[p];
            for (size_t d = 0; d < head_dim; d++) oh[d] += wgt * deq[d];
        }
    }
}

/* forward_token — crates/sulimo-engine/src/forward_pass.rs:190-417 (Llama / Qwen2 branches):
 * lookup_token_embedding :419-450, apply_rmsnorm :493-507 (dispatch_rmsnorm -> rmsnorm_avx2),
 * quantize_f32_to_q8_0 + apply_matvec :509-527 (dispatch_matvec_q4_0_q8_0 -> avx2), add_bias
 * :452-465, rope_head_scalar per head, KvCache::store_key/value, causal_gqa_decode_scalar_ext
 * with context pos+1, swiglu_scalar, residual adds, final norm + output projection. */
/* apply_rmsnorm — forward_pass.rs:495-507: the Gemma form for ModelArch::Gemma2 */
static void fwd_rmsnorm(const oracle_model* m, const float* x, const float* w, size_t n, float* out) {
    if (m->arch == ORACLE_ARCH_GEMMA2)
        oracle_rmsnorm_gemma_avx2(x, w, n, m->eps, out);
    else
        oracle_rmsnorm_avx2(x, w, n, m->eps, out);
}

void oracle_forward_token(const oracle_model* m, uint32_t token, size_t pos, float* logits) {
    const size_t E = (size_t)m->embd, F = (size_t)m->ffn, hd = (size_t)m->head_dim;
    const size_t qd = (size_t)m->head_count * hd, kvd = (size_t)m->head_count_kv * hd;
    const size_t nbE = E / 32;
    const size_t ctx = pos + 1;
    const int gemma = m->arch == ORACLE_ARCH_GEMMA2;
    float* x = (float*)malloc(E * 4);
    float* h = (float*)malloc(E * 4);
    float* q = (float*)malloc(qd * 4);
    float* k = (float*)malloc(kvd * 4);
    float* v = (float*)malloc(kvd * 4);
    float* att = (float*)malloc(qd * 4);
    float* g = (float*)malloc(F * 4);
    float* u = (float*)malloc(F * 4);
    float* sw = (float*)malloc(F * 4);
    float* dn = (float*)malloc(E * 4);
    float* scores = (float*)malloc(ctx * 4);
    size_t q8n = (qd > E ? qd : E);
    if (F > q8n) q8n = F;
    uint8_t* q8 = (uint8_t*)malloc(q8n / 32 * 34);
    oracle_dequantize_q4_0_soa(m->tok_s + (size_t)token * nbE * 2, m->tok_q + (size_t)token * nbE * 16,
                               nbE, x);
    if (gemma) { /* forward_pass.rs:210-214: x *= sqrt(embd) */
        const float scale = sqrtf((float)E);
        for (size_t i = 0; i < E; i++) x[i] *= scale;
    }
    for (int l = 0; l < m->n_layers; l++) {
        const oracle_layer* L = &m->layers[l];
        fwd_rmsnorm(m, x, L->attn_norm, E, h);
        oracle_quantize_f32_to_q8_0(h, E, q8);
        oracle_matvec_q4_0_q8_0_avx2(L->wq_s, L->wq_q, q8, qd, E, q);
        oracle_matvec_q4_0_q8_0_avx2(L->wk_s, L->wk_q, q8, kvd, E, k);
        oracle_matvec_q4_0_q8_0_avx2(L->wv_s, L->wv_q, q8, kvd, E, v);
        if (L->bq) for (size_t i = 0; i < qd; i++) q[i] += L->bq[i];
        if (L->bk) for (size_t i = 0; i < kvd; i++) k[i] += L->bk[i];
        if (L->bv) for (size_t i = 0; i < kvd; i++) v[i] += L->bv[i];
        for (int hh = 0; hh < m->head_count; hh++)
            oracle_rope_head_scalar(q + hh * hd, pos, (size_t)m->rope_dim, m->rope_base, m->rope_mode);
        for (int hh = 0; hh < m->head_count_kv; hh++)
            oracle_rope_head_scalar(k + hh * hd, pos, (size_t)m->rope_dim, m->rope_base, m->rope_mode);
        oracle_kv_store_f32(k, L->k_ring, pos, m->kv_capacity, kvd / 32);
        oracle_kv_store_f32(v, L->v_ring, pos, m->kv_capacity, kvd / 32);
        oracle_causal_gqa_decode(q, L->k_ring, L->v_ring, m->kv_capacity, ctx,
                                 (size_t)m->head_count, (size_t)m->head_count_kv, hd, scores, att,
                                 m->attn_softcap);
        oracle_quantize_f32_to_q8_0(att, qd, q8);
        oracle_matvec_q4_0_q8_0_avx2(L->wo_s, L->wo_q, q8, E, qd, h);
        if (L->post_attn_norm) { /* forward_pass.rs:330-336: x += rmsnorm(Wo a) * post_attn_norm */
            fwd_rmsnorm(m, h, L->post_attn_norm, E, att);
            for (size_t i = 0; i < E; i++) x[i] += att[i];
        } else {
            for (size_t i = 0; i < E; i++) x[i] += h[i];
        }
        fwd_rmsnorm(m, x, L->ffn_norm, E, h);
        oracle_quantize_f32_to_q8_0(h, E, q8);
        oracle_matvec_q4_0_q8_0_avx2(L->wg_s, L->wg_q, q8, F, E, g);
        oracle_matvec_q4_0_q8_0_avx2(L->wu_s, L->wu_q, q8, F, E, u);
        if (gemma) /* forward_pass.rs:363-368 */
            oracle_geglu_scalar(g, u, sw, F);
        else
            oracle_swiglu_scalar(g, u, sw, F);
        oracle_quantize_f32_to_q8_0(sw, F, q8);
        oracle_matvec_q4_0_q8_0_avx2(L->wd_s, L->wd_q, q8, E, F, dn);
        if (L->post_ffn_norm) { /* forward_pass.rs:379-385 */
            fwd_rmsnorm(m, dn, L->post_ffn_norm, E, h);
            for (size_t i = 0; i < E; i++) x[i] += h[i];
        } else {
            for (size_t i = 0; i < E; i++) x[i] += dn[i];
        }
    }
    fwd_rmsnorm(m, x, m->out_norm, E, h);
    oracle_quantize_f32_to_q8_0(h, E, q8);
    oracle_matvec_q4_0_q8_0_avx2(m->out_s, m->out_q, q8, (size_t)m->vocab, E, logits);
    oracle_logit_softcap_scalar(logits, (size_t)m->vocab, m->final_softcap); /* :411-414 */
    free(x); free(h); free(q); free(k); free(v); free(att); free(g); free(u); free(sw);
    free(dn); free(scores); free(q8);
}

/* ------------------------------------------------------------------ */
/* GPU prefill ubatch on f16 storage                                   */
/* ------------------------------------------------------------------ */
/* The reference's GPU prefill (execute_prefill_ubatch, crates/sulimo-ocl/src/prefill.rs:337-566)
 * keeps every activation in f16 between kernels; each helper below restates one kernel of
 * kernels/prefill.cl on those f16 buffers, with its float operations in source order. */

static inline uint16_t f16r(float x) { return oracle_f32_to_f16(x); }
static inline float f16w(uint16_t h) { return oracle_f16_to_f32(h); }

/* rmsnorm_f16_f32w — kernels/prefill.cl:4-29 */
void oracle_rmsnorm_f16(const uint16_t* x, const float* w, uint16_t* out, size_t D, float eps,
                        size_t N) {
    for (size_t n = 0; n < N; n++) {
        const uint16_t* xr = x + n * D;
        float sum_sq = 0.0f;
        for (size_t i = 0; i < D; i++) {
            float v = f16w(xr[i]);
            sum_sq += v * v;
        }
        float mean = sum_sq / (float)D;
        float scale = 1.0f / sqrtf(mean + eps);
        for (size_t i = 0; i < D; i++) out[n * D + i] = f16r(f16w(xr[i]) * scale * w[i]);
    }
}

/* rope_f16 — kernels/prefill.cl:32-68: the rotation of rope_head_scalar on f16 storage */
void oracle_rope_f16(uint16_t* vec, size_t head_count, size_t head_dim, size_t rope_dim,
                     float freq_base, int mode, size_t start_pos, size_t N) {
    float* tmp = (float*)__builtin_alloca(head_dim * sizeof(float));
    for (size_t n = 0; n < N; n++)
        for (size_t h = 0; h < head_count; h++) {
            uint16_t* hp = vec + (n * head_count + h) * head_dim;
            for (size_t i = 0; i < head_dim; i++) tmp[i] = f16w(hp[i]);
            oracle_rope_head_scalar(tmp, start_pos + n, rope_dim, freq_base, mode);
            for (size_t i = 0; i < rope_dim; i++) hp[i] = f16r(tmp[i]);
        }
}

/* causal_gqa_attention_prefill — kernels/prefill.cl:120-237: scores in fp32 from f16 q and the
 * Q8_0 ring (each K element dequantised as q*d before the product), softmax over positions
 * 0..start_pos+n, then the output accumulated IN F16: out += f16(w * v) per key, per element.
 * The kernel recomputes the identical scores in each of its three passes; they are computed
 * once here. */
void oracle_attention_prefill_f16(const uint16_t* q, const uint8_t* k_ring, const uint8_t* v_ring,
                                  uint16_t* out, size_t start_pos, size_t capacity,
                                  size_t head_count, size_t head_count_kv, size_t head_dim,
                                  size_t N) {
    const size_t hpk = head_count / head_count_kv;
    const float scale = 1.0f / sqrtf((float)head_dim);
    const size_t bph = head_dim / 32, head_bytes = bph * 34;
    const size_t bytes_per_pos = head_count_kv * head_bytes;
    float* scores = (float*)malloc((start_pos + N) * sizeof(float));
    for (size_t n = 0; n < N; n++)
        for (size_t h = 0; h < head_count; h++) {
            const size_t kvh = h / hpk, num_keys = start_pos + n + 1;
            const uint16_t* qh = q + (n * head_count + h) * head_dim;
            float max_score = -1e30f;
            for (size_t p = 0; p < num_keys; p++) {
                const uint8_t* kp = k_ring + (p % capacity) * bytes_per_pos + kvh * head_bytes;
                float dot = 0.0f;
                for (size_t b = 0; b < bph; b++) {
                    const uint8_t* blk = kp + b * 34;
                    float d = le_f16(blk);
                    for (int i = 0; i < 32; i++)
                        dot += f16w(qh[b * 32 + i]) * ((float)(int8_t)blk[2 + i] * d);
                }
                float s = dot * scale;
                scores[p] = s;
                if (s > max_score) max_score = s;
            }
            float sum_exp = 0.0f;
            for (size_t p = 0; p < num_keys; p++) sum_exp += expf(scores[p] - max_score);
            const float inv = (sum_exp > 0.0f) ? (1.0f / sum_exp) : 0.0f;
            uint16_t* oh = out + (n * head_count + h) * head_dim;
            for (size_t i = 0; i < head_dim; i++) oh[i] = 0;
            for (size_t p = 0; p < num_keys; p++) {
                const float wgt = expf(scores[p] - max_score) * inv;
                const uint8_t* vp = v_ring + (p % capacity) * bytes_per_pos + kvh * head_bytes;
                for (size_t b = 0; b < bph; b++) {
                    const uint8_t* blk = vp + b * 34;
                    float d = le_f16(blk);
                    for (int i = 0; i < 32; i++) {
                        float vv = (float)(int8_t)blk[2 + i] * d;
                        uint16_t* o = &oh[b * 32 + i];
                        *o = f16r(f16w(*o) + f16w(f16r(wgt * vv)));
                    }
                }
            }
        }
    free(scores);
}

/* silu_mul_f16 — kernels/prefill.cl:240-253 */
void oracle_silu_mul_f16(const uint16_t* gate, const uint16_t* up, uint16_t* out, size_t n) {
    for (size_t i = 0; i < n; i++) {
        float g = f16w(gate[i]), u = f16w(up[i]);
        float silu = g / (1.0f + expf(-g));
        out[i] = f16r(silu * u);
    }
}

/* add_f16 — kernels/prefill.cl:256-266 */
void oracle_add_f16(uint16_t* a, const uint16_t* b, size_t n) {
    for (size_t i = 0; i < n; i++) a[i] = f16r(f16w(a[i]) + f16w(b[i]));
}

/* One GEMM of the ubatch with f16 results: gemm_q4_0_f16_portable (kernels/gemm_q4_0.cl:13-58),
 * whose arithmetic is gemm_dot's, rounded once to f16. */
static void pf_gemm_f16(const uint8_t* scales, const uint8_t* quants, const uint16_t* x,
                        size_t m, size_t k, size_t n, uint16_t* out, float* tmp, int threads) {
    oracle_gemm_q4_0_f16_scalar_f32out((const uint16_t*)scales, quants, x, m, k, n, tmp, threads);
    oracle_f32_to_f16_array(tmp, out, m * n);
}

/* execute_prefill_ubatch — crates/sulimo-ocl/src/prefill.rs:337-566, step for step (steps 1-14
 * of its body).  x: [n][embd] f16, the ubatch's embeddings on entry (lookup_token_embedding_f16
 * per token, crates/sulimo-engine/src/engine.rs:249-256) and the residual stream on return;
 * K/V go to ring slots (start_pos + t) % kv_capacity; logits[vocab] = the last token's fp32
 * logits.  As in the reference, the o projection is embd x embd (head_count*head_dim == embd)
 * and no QKV bias or softcap is applied.  Returns 0, or -1 for invalid arguments. */
int oracle_prefill_ubatch(const oracle_model* m, uint16_t* x, size_t start_pos, size_t n,
                          float* logits, int threads) {
    if (!m || !x || !logits || n == 0) return -1;
    const size_t E = (size_t)m->embd, F = (size_t)m->ffn, hd = (size_t)m->head_dim;
    const size_t H = (size_t)m->head_count, Hkv = (size_t)m->head_count_kv;
    const size_t qd = H * hd, kvd = Hkv * hd;
    if (qd != E) return -1;
    size_t big = E > F ? E : F;
    uint16_t* h = (uint16_t*)malloc(n * E * 2);
    uint16_t* q = (uint16_t*)malloc(n * qd * 2);
    uint16_t* k = (uint16_t*)malloc(n * kvd * 2);
    uint16_t* v = (uint16_t*)malloc(n * kvd * 2);
    uint16_t* att = (uint16_t*)malloc(n * qd * 2);
    uint16_t* g = (uint16_t*)malloc(n * F * 2);
    uint16_t* u = (uint16_t*)malloc(n * F * 2);
    uint16_t* sw = (uint16_t*)malloc(n * F * 2);
    uint16_t* dn = (uint16_t*)malloc(n * E * 2);
    float* tmp = (float*)malloc(n * big * 4);
    for (int l = 0; l < m->n_layers; l++) {
        const oracle_layer* L = &m->layers[l];
        oracle_rmsnorm_f16(x, L->attn_norm, h, E, m->eps, n);
        pf_gemm_f16(L->wq_s, L->wq_q, h, qd, E, n, q, tmp, threads);
        pf_gemm_f16(L->wk_s, L->wk_q, h, kvd, E, n, k, tmp, threads);
        pf_gemm_f16(L->wv_s, L->wv_q, h, kvd, E, n, v, tmp, threads);
        oracle_rope_f16(q, H, hd, (size_t)m->rope_dim, m->rope_base, m->rope_mode, start_pos, n);
        oracle_rope_f16(k, Hkv, hd, (size_t)m->rope_dim, m->rope_base, m->rope_mode, start_pos, n);
        oracle_kv_store_q8_0(k, L->k_ring, start_pos, m->kv_capacity, kvd / 32, n);
        oracle_kv_store_q8_0(v, L->v_ring, start_pos, m->kv_capacity, kvd / 32, n);
        oracle_attention_prefill_f16(q, L->k_ring, L->v_ring, att, start_pos, m->kv_capacity, H,
                                     Hkv, hd, n);
        pf_gemm_f16(L->wo_s, L->wo_q, att, E, E, n, h, tmp, threads);
        oracle_add_f16(x, h, n * E);
        oracle_rmsnorm_f16(x, L->ffn_norm, h, E, m->eps, n);
        pf_gemm_f16(L->wg_s, L->wg_q, h, F, E, n, g, tmp, threads);
        pf_gemm_f16(L->wu_s, L->wu_q, h, F, E, n, u, tmp, threads);
        oracle_silu_mul_f16(g, u, sw, n * F);
        pf_gemm_f16(L->wd_s, L->wd_q, sw, E, F, n, dn, tmp, threads);
        oracle_add_f16(x, dn, n * E);
    }
    oracle_rmsnorm_f16(x, m->out_norm, h, E, m->eps, n);
    oracle_gemm_q4_0_f16_scalar_f32out((const uint16_t*)m->out_s, m->out_q, h + (n - 1) * E,
                                       (size_t)m->vocab, E, 1, logits, threads);
    free(h); free(q); free(k); free(v); free(att); free(g); free(u); free(sw); free(dn); free(tmp);
    return 0;
}

/* The CPU oracle of the reference's prefill test (crates/sulimo-ocl/tests/test_prefill.rs:
 * 583-800), the reference's own definition of a correct GPU prefill, which its GPU ubatch must
 * match within one Q8_0 step of K/V, cosine 0.99 and the same greedy token (:826-890): an fp32
 * residual stream, rmsnorm_scalar (scalar.rs:23-40) rounded to f16 for each GEMM, f16 GEMM
 * outputs widened to f32, rope_head_scalar in fp32, quantize_f32_to_q8_0 into the ring,
 * causal_gqa_decode_scalar per token, SwiGLU in fp32, and the last token's final norm kept in
 * fp32 for the logits (:781-800).  Positions start at start_pos (the test uses 0) and ring slots
 * are (start_pos + t) % kv_capacity.  QKV biases, when the model has them, are added to the
 * widened projections as forward_token adds them (forward_pass.rs:452-465); the test's Llama
 * model has none.  x_f16: [n][embd] embeddings in; logits[vocab] of the last token.  0 / -1. */
int oracle_prefill_ubatch_f32(const oracle_model* m, const uint16_t* x_f16, size_t start_pos,
                              size_t n, float* logits, int threads) {
    if (!m || !x_f16 || !logits || n == 0) return -1;
    const size_t E = (size_t)m->embd, F = (size_t)m->ffn, hd = (size_t)m->head_dim;
    const size_t H = (size_t)m->head_count, Hkv = (size_t)m->head_count_kv;
    const size_t qd = H * hd, kvd = Hkv * hd;
    const size_t ctx_max = start_pos + n;
    size_t big = qd > F ? qd : F;
    if (E > big) big = E;
    float* x = (float*)malloc(n * E * 4);
    float* hf = (float*)malloc(n * E * 4);
    uint16_t* h16 = (uint16_t*)malloc(n * big * 2);
    float* q = (float*)malloc(n * qd * 4);
    float* k = (float*)malloc(n * kvd * 4);
    float* v = (float*)malloc(n * kvd * 4);
    float* att = (float*)malloc(n * qd * 4);
    float* g = (float*)malloc(n * F * 4);
    float* u = (float*)malloc(n * F * 4);
    float* tmp = (float*)malloc(n * big * 4);
    float* scores = (float*)malloc(ctx_max * 4);
    oracle_f16_to_f32_array(x_f16, x, n * E);
    /* a GEMM with f16 inputs and f16 outputs widened back to f32 (gemm_q4_0_f16_scalar_reference
     * then f16::to_f32) */
#define PF32_GEMM(W_S, W_Q, IN16, ROWS, COLS, OUT)                                              \
    do {                                                                                       \
        oracle_gemm_q4_0_f16_scalar_f32out((const uint16_t*)(W_S), (W_Q), (IN16), (ROWS), (COLS), \
                                           n, tmp, threads);                                   \
        for (size_t i_ = 0; i_ < (size_t)(ROWS) * n; i_++) (OUT)[i_] = f16w(f16r(tmp[i_]));    \
    } while (0)
    for (int l = 0; l < m->n_layers; l++) {
        const oracle_layer* L = &m->layers[l];
        for (size_t t = 0; t < n; t++) oracle_rmsnorm_scalar(x + t * E, L->attn_norm, E, m->eps, hf + t * E);
        oracle_f32_to_f16_array(hf, h16, n * E);
        PF32_GEMM(L->wq_s, L->wq_q, h16, qd, E, q);
        PF32_GEMM(L->wk_s, L->wk_q, h16, kvd, E, k);
        PF32_GEMM(L->wv_s, L->wv_q, h16, kvd, E, v);
        for (size_t t = 0; t < n; t++) {
            if (L->bq) for (size_t i = 0; i < qd; i++) q[t * qd + i] += L->bq[i];
            if (L->bk) for (size_t i = 0; i < kvd; i++) k[t * kvd + i] += L->bk[i];
            if (L->bv) for (size_t i = 0; i < kvd; i++) v[t * kvd + i] += L->bv[i];
            for (size_t hh = 0; hh < H; hh++)
                oracle_rope_head_scalar(q + t * qd + hh * hd, start_pos + t, (size_t)m->rope_dim,
                                        m->rope_base, m->rope_mode);
            for (size_t hh = 0; hh < Hkv; hh++)
                oracle_rope_head_scalar(k + t * kvd + hh * hd, start_pos + t, (size_t)m->rope_dim,
                                        m->rope_base, m->rope_mode);
            oracle_kv_store_f32(k + t * kvd, L->k_ring, start_pos + t, m->kv_capacity, kvd / 32);
            oracle_kv_store_f32(v + t * kvd, L->v_ring, start_pos + t, m->kv_capacity, kvd / 32);
        }
        for (size_t t = 0; t < n; t++)
            oracle_causal_gqa_decode(q + t * qd, L->k_ring, L->v_ring, m->kv_capacity,
                                     start_pos + t + 1, H, Hkv, hd, scores, att + t * qd, 0.0f);
        oracle_f32_to_f16_array(att, h16, n * qd);
        PF32_GEMM(L->wo_s, L->wo_q, h16, E, qd, hf);
        for (size_t i = 0; i < n * E; i++) x[i] += hf[i];
        for (size_t t = 0; t < n; t++) oracle_rmsnorm_scalar(x + t * E, L->ffn_norm, E, m->eps, hf + t * E);
        oracle_f32_to_f16_array(hf, h16, n * E);
        PF32_GEMM(L->wg_s, L->wg_q, h16, F, E, g);
        PF32_GEMM(L->wu_s, L->wu_q, h16, F, E, u);
        oracle_swiglu_scalar(g, u, g, n * F);
        oracle_f32_to_f16_array(g, h16, n * F);
        PF32_GEMM(L->wd_s, L->wd_q, h16, E, F, hf);
        for (size_t i = 0; i < n * E; i++) x[i] += hf[i];
    }
#undef PF32_GEMM
    oracle_rmsnorm_scalar(x + (n - 1) * E, m->out_norm, E, m->eps, hf);
    /* logits from the fp32 final norm (test_prefill.rs:781-800): gemm_dot on f32 inputs */
    const size_t nbr = E / 32;
    for (size_t r = 0; r < (size_t)m->vocab; r++)
        logits[r] = gemm_dot((const uint16_t*)m->out_s, m->out_q, hf, r, nbr);
    free(x); free(hf); free(h16); free(q); free(k); free(v); free(att); free(g); free(u);
    free(tmp); free(scores);
    return 0;
}

/* ------------------------------------------------------------------ */
/* Raw F32 / F16 matvecs (apply_matvec's other branches)               */
/* ------------------------------------------------------------------ */

/* matvec_f32_avx2 — crates/sulimo-cpu/src/avx2.rs:259-280; same intrinsics in the same order */
void oracle_matvec_f32_avx2(const float* w, const float* x, size_t rows, size_t cols,
                            float* out) {
    size_t chunks = cols / 8;
    for (size_t r = 0; r < rows; r++) {
        const float* wr = w + r * cols;
        __m256 acc = _mm256_setzero_ps();
        for (size_t c = 0; c < chunks; c++)
            acc = _mm256_fmadd_ps(_mm256_loadu_ps(wr + c * 8), _mm256_loadu_ps(x + c * 8), acc);
        float sum = hsum_256(acc);
        for (size_t c = chunks * 8; c < cols; c++) sum += wr[c] * x[c];
        out[r] = sum;
    }
}

/* matvec_f16_avx2 — avx2.rs:287-331: F16C widening, same lanes and tree */
void oracle_matvec_f16_avx2(const uint16_t* w, const float* x, size_t rows, size_t cols,
                            float* out) {
    size_t chunks = cols / 8;
    for (size_t r = 0; r < rows; r++) {
        const uint16_t* wr = w + r * cols;
        __m256 acc = _mm256_setzero_ps();
        for (size_t c = 0; c < chunks; c++) {
            __m256 wv = _mm256_cvtph_ps(_mm_loadu_si128((const __m128i*)(wr + c * 8)));
            acc = _mm256_fmadd_ps(wv, _mm256_loadu_ps(x + c * 8), acc);
        }
        float sum = hsum_256(acc);
        for (size_t c = chunks * 8; c < cols; c++) sum += oracle_f16_to_f32(wr[c]) * x[c];
        out[r] = sum;
    }
}

/* matvec_f32_scalar / matvec_f16_scalar — crates/sulimo-cpu/src/scalar.rs:228-251 */
void oracle_matvec_f32_scalar(const float* w, const float* x, size_t rows, size_t cols,
                              float* out) {
    for (size_t r = 0; r < rows; r++) {
        float sum = 0.0f;
        for (size_t c = 0; c < cols; c++) sum += w[r * cols + c] * x[c];
        out[r] = sum;
    }
}

void oracle_matvec_f16_scalar(const uint16_t* w, const float* x, size_t rows, size_t cols,
                              float* out) {
    for (size_t r = 0; r < rows; r++) {
        float sum = 0.0f;
        for (size_t c = 0; c < cols; c++) sum += oracle_f16_to_f32(w[r * cols + c]) * x[c];
        out[r] = sum;
    }
}
