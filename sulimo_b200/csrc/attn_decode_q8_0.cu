// attn_decode_q8_0.cu — single-position causal GQA attention over the Q8_0 KV ring.
//
// Restates causal_gqa_decode_scalar_ext (crates/sulimo-cpu/src/scalar.rs:287-359) with the ring
// addressing of KvCache::key_ptr / value_ptr (crates/sulimo-core/src/kv_cache.rs:114-128):
//   for each query head h (kv head h / (H/Hkv)):
//     score[p] = (q_h . dequant(K[p % cap])) * 1/sqrt(hd)   [optionally tanh soft-capped]
//     w = softmax(score[0..ctx]);  out_h = sum_p w[p] * dequant(V[p % cap])
//
// B200 form (split-K over the context, "flash-decoding"):
//   kernel 1, one CTA per (context split, kv head, sequence): stages the split's K head-rows
//   into shared memory once for all H/Hkv query heads of the group (the scalar reference
//   re-reads them per query head), computes the scores, the split's max m and sum l of
//   exp(score - m), stages V the same way and accumulates sum exp(score-m) * v.  It writes
//   (o[hd], m, l) per (sequence, query head, split) to a workspace.
//   kernel 2 merges the splits: out = sum_s o_s e^{m_s-M} / sum_s l_s e^{m_s-M}.
// Reordered fp32 sums: the result matches the reference within fp32 rounding (the parity
// tests bound the relative L2 error at 2e-3).
#include "sulimo_common.cuh"
#include "sulimo_internal.h"

namespace sulimo {
namespace {

constexpr int ATT_THREADS = 128;
constexpr int ATT_PMAX = 256;  // positions per split
constexpr int ATT_GMAX = 8;    // query heads per kv head

// Shared memory per CTA (dynamic): q[G][HD] f32 | sc[PMAX][NB] f32 | qs[PMAX][NB*32 + 16] i8 |
// e[G][PMAX] f32
template <int HD>
struct AttnLayout {
    static constexpr int NB = HD / 32;
    static constexpr int QS_STRIDE = NB * 32 + 16;  // bytes per staged position (16: bank skew)
    static constexpr size_t q_off = 0;
    static constexpr size_t sc_off = q_off + sizeof(float) * ATT_GMAX * HD;
    static constexpr size_t qs_off = sc_off + sizeof(float) * ATT_PMAX * NB;
    static constexpr size_t e_off = qs_off + (size_t)QS_STRIDE * ATT_PMAX;
    static constexpr size_t bytes = e_off + sizeof(float) * ATT_GMAX * ATT_PMAX;
};

// Copies the head rows of positions [p0, p0+np) of one kv head into shared memory:
// scales -> sc[pos][b] (f32), quants -> qs[pos][b*32 + i] (i8).  2-byte loads: the ring's
// 34-byte blocks are only 2-byte aligned.
template <int HD>
__device__ __forceinline__ void stage_rows(const uint8_t* __restrict__ ring, size_t capacity,
                                           size_t bpp, size_t head_off, size_t p0, int np,
                                           float* sc, uint8_t* qs) {
    using L = AttnLayout<HD>;
    constexpr int W = L::NB * 17;  // u16 words per head row
    for (int it = threadIdx.x; it < np * W; it += ATT_THREADS) {
        const int pos = it / W, w = it - pos * W;
        const int b = w / 17, k = w - b * 17;
        const size_t slot = (p0 + pos) % capacity;
        const uint16_t* src =
            reinterpret_cast<const uint16_t*>(ring + slot * bpp + head_off + (size_t)b * 34);
        const uint16_t v = __ldg(src + k);
        if (k == 0)
            sc[pos * L::NB + b] = f16_bits_to_f32(v);
        else
            *reinterpret_cast<uint16_t*>(qs + pos * L::QS_STRIDE + b * 32 + 2 * (k - 1)) = v;
    }
}

template <int HD>
__global__ void __launch_bounds__(ATT_THREADS)
    attn_decode_partial_kernel(const float* __restrict__ q, const uint8_t* __restrict__ kring,
                               const uint8_t* __restrict__ vring, size_t seq_stride,
                               size_t capacity, size_t ctx_len, int H, int Hkv, int chunk,
                               float sm_scale, float softcap, float* __restrict__ part) {
    using L = AttnLayout<HD>;
    extern __shared__ __align__(16) uint8_t smem[];
    float* sq = reinterpret_cast<float*>(smem + L::q_off);
    float* sc = reinterpret_cast<float*>(smem + L::sc_off);
    uint8_t* qs = smem + L::qs_off;
    float* se = reinterpret_cast<float*>(smem + L::e_off);
    __shared__ float red[ATT_THREADS / 32][ATT_GMAX];

    const int split = blockIdx.x, kvh = blockIdx.y, seq = blockIdx.z;
    const int splits = gridDim.x;
    const int G = H / Hkv;
    const size_t p0 = (size_t)split * chunk;
    const int np = (int)min((size_t)chunk, ctx_len > p0 ? ctx_len - p0 : (size_t)0);
    const size_t hb = (size_t)L::NB * 34;
    const size_t bpp = (size_t)Hkv * hb;
    const size_t head_off = (size_t)kvh * hb;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;

    // query heads of this group
    for (int i = tid; i < G * HD; i += ATT_THREADS)
        sq[i] = q[((size_t)seq * H + (size_t)kvh * G) * HD + i];
    stage_rows<HD>(kring + (size_t)seq * seq_stride, capacity, bpp, head_off, p0, np, sc, qs);
    __syncthreads();

    // ---- scores: one thread per position ----
    for (int pos = tid; pos < np; pos += ATT_THREADS) {
        float dot[ATT_GMAX];
#pragma unroll
        for (int g = 0; g < ATT_GMAX; g++) dot[g] = 0.0f;
        const uint8_t* row = qs + pos * L::QS_STRIDE;
#pragma unroll
        for (int b = 0; b < L::NB; b++) {
            const float s = sc[pos * L::NB + b];
#pragma unroll
            for (int i16 = 0; i16 < 2; i16++) {
                // 16-byte loads: with the 16-byte row skew, 8 lanes hit 8 distinct bank groups
                const uint4 w4 = *reinterpret_cast<const uint4*>(row + b * 32 + i16 * 16);
                const uint32_t ws[4] = {w4.x, w4.y, w4.z, w4.w};
#pragma unroll
                for (int i4 = 0; i4 < 4; i4++) {
#pragma unroll
                    for (int e = 0; e < 4; e++) {
                        const float kv =
                            __fmul_rn((float)(int8_t)((ws[i4] >> (8 * e)) & 0xFF), s);
                        const int d = b * 32 + i16 * 16 + i4 * 4 + e;
#pragma unroll
                        for (int g = 0; g < ATT_GMAX; g++)
                            if (g < G) dot[g] = __fmaf_rn(sq[g * HD + d], kv, dot[g]);
                    }
                }
            }
        }
#pragma unroll
        for (int g = 0; g < ATT_GMAX; g++) {
            if (g < G) {
                float score = __fmul_rn(dot[g], sm_scale);
                if (softcap > 0.0f) score = tanhf(score / softcap) * softcap;
                se[g * ATT_PMAX + pos] = score;
            }
        }
    }
    __syncthreads();

    // ---- split max and sum of exp, per query head ----
    float mloc[ATT_GMAX], lloc[ATT_GMAX];
#pragma unroll
    for (int g = 0; g < ATT_GMAX; g++) {
        if (g >= G) break;
        float m = -INFINITY;
        for (int pos = tid; pos < np; pos += ATT_THREADS) m = fmaxf(m, se[g * ATT_PMAX + pos]);
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, off));
        if (lane == 0) red[warp][g] = m;
    }
    __syncthreads();
#pragma unroll
    for (int g = 0; g < ATT_GMAX; g++) {
        if (g >= G) break;
        float m = red[0][g];
        for (int w = 1; w < ATT_THREADS / 32; w++) m = fmaxf(m, red[w][g]);
        mloc[g] = m;
    }
    __syncthreads();
#pragma unroll
    for (int g = 0; g < ATT_GMAX; g++) {
        if (g >= G) break;
        float l = 0.0f;
        for (int pos = tid; pos < np; pos += ATT_THREADS) {
            const float e = expf(se[g * ATT_PMAX + pos] - mloc[g]);
            se[g * ATT_PMAX + pos] = e;
            l += e;
        }
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) l += __shfl_xor_sync(0xffffffffu, l, off);
        if (lane == 0) red[warp][g] = l;
    }
    __syncthreads();
#pragma unroll
    for (int g = 0; g < ATT_GMAX; g++) {
        if (g >= G) break;
        float l = 0.0f;
        for (int w = 0; w < ATT_THREADS / 32; w++) l += red[w][g];
        lloc[g] = l;
    }

    // ---- V: stage, then one thread per head dimension (groups of threads split positions) ----
    stage_rows<HD>(vring + (size_t)seq * seq_stride, capacity, bpp, head_off, p0, np, sc, qs);
    __syncthreads();
    constexpr int DPT = (HD + ATT_THREADS - 1) / ATT_THREADS;  // dims per thread
    constexpr int GROUPS = (HD >= ATT_THREADS) ? 1 : ATT_THREADS / HD;
    const int grp = tid / (ATT_THREADS / GROUPS);
    const int dt = tid % (ATT_THREADS / GROUPS);
    float o[ATT_GMAX][DPT];
#pragma unroll
    for (int g = 0; g < ATT_GMAX; g++)
#pragma unroll
        for (int k = 0; k < DPT; k++) o[g][k] = 0.0f;
    for (int pos = grp; pos < np; pos += GROUPS) {
#pragma unroll
        for (int k = 0; k < DPT; k++) {
            const int d = dt + k * ATT_THREADS;
            if (d < HD) {
                const int b = d / 32;
                const float v = __fmul_rn((float)(int8_t)qs[pos * L::QS_STRIDE + d], sc[pos * L::NB + b]);
#pragma unroll
                for (int g = 0; g < ATT_GMAX; g++)
                    if (g < G) o[g][k] = __fmaf_rn(se[g * ATT_PMAX + pos], v, o[g][k]);
            }
        }
    }
    // reduce the position groups through shared memory (reuse the score area)
    __syncthreads();
    float* ored = se;  // [GROUPS][G][HD] <= GMAX*PMAX floats
    if (GROUPS > 1) {
#pragma unroll
        for (int g = 0; g < ATT_GMAX; g++)
            if (g < G)
#pragma unroll
                for (int k = 0; k < DPT; k++) {
                    const int d = dt + k * ATT_THREADS;
                    if (d < HD) ored[(grp * G + g) * HD + d] = o[g][k];
                }
        __syncthreads();
    }
    const size_t base = (((size_t)seq * H + (size_t)kvh * G) * splits + split);
    if (grp == 0) {
#pragma unroll
        for (int g = 0; g < ATT_GMAX; g++) {
            if (g >= G) break;
            float* dst = part + (base + (size_t)g * splits) * (HD + 2);
#pragma unroll
            for (int k = 0; k < DPT; k++) {
                const int d = dt + k * ATT_THREADS;
                if (d < HD) {
                    float v = o[g][k];
                    for (int r = 1; r < GROUPS; r++) v += ored[(r * G + g) * HD + d];
                    dst[d] = v;
                }
            }
            if (dt == 0) {
                dst[HD] = np > 0 ? mloc[g] : -INFINITY;
                dst[HD + 1] = np > 0 ? lloc[g] : 0.0f;
            }
        }
    }
}

// One CTA per (query head, sequence); thread d owns output dimension d.
template <int HD>
__global__ void __launch_bounds__(HD < 32 ? 32 : HD)
    attn_decode_combine_kernel(const float* __restrict__ part, int H, int splits,
                               float* __restrict__ out) {
    const int h = blockIdx.x, seq = blockIdx.y, d = threadIdx.x;
    const float* p = part + ((size_t)seq * H + h) * splits * (HD + 2);
    float M = -INFINITY;
    for (int s = 0; s < splits; s++) M = fmaxf(M, p[(size_t)s * (HD + 2) + HD]);
    float Lsum = 0.0f, O = 0.0f;
    for (int s = 0; s < splits; s++) {
        const float* ps = p + (size_t)s * (HD + 2);
        const float m = ps[HD];
        if (m == -INFINITY) continue;
        const float f = expf(m - M);
        Lsum = __fmaf_rn(ps[HD + 1], f, Lsum);
        O = __fmaf_rn(ps[d], f, O);
    }
    out[((size_t)seq * H + h) * HD + d] = Lsum > 0.0f ? O / Lsum : 0.0f;
}

int pick_splits(size_t ctx_len, int Hkv, int batch, int num_sms) {
    size_t min_splits = (ctx_len + ATT_PMAX - 1) / ATT_PMAX;
    if (min_splits < 1) min_splits = 1;
    size_t want = ((size_t)2 * num_sms + (size_t)Hkv * batch - 1) / ((size_t)Hkv * batch);
    size_t max_splits = (ctx_len + 31) / 32;  // keep >= 32 positions per split
    if (max_splits < 1) max_splits = 1;
    size_t s = want < max_splits ? want : max_splits;
    if (s < min_splits) s = min_splits;
    return (int)s;
}

template <int HD>
int launch_hd(sulimo_ctx* ctx, const float* q, const uint8_t* k, const uint8_t* v,
              size_t seq_stride, size_t capacity, size_t ctx_len, int H, int Hkv, int batch,
              float softcap, float* out, float* part, int splits) {
    using L = AttnLayout<HD>;
    const int chunk = (int)((ctx_len + splits - 1) / splits);
    const float sm_scale = 1.0f / sqrtf((float)HD);
    static uint64_t attr_set_mask = 0;  // one bit per device: the attribute is per device
    const uint64_t bit = 1ull << (ctx->device & 63);
    if (!(attr_set_mask & bit)) {
        int st = check_cuda(cudaFuncSetAttribute(attn_decode_partial_kernel<HD>,
                                                 cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                 (int)L::bytes),
                            "attn smem attribute");
        if (st) return st;
        attr_set_mask |= bit;
    }
    dim3 g1(splits, Hkv, batch);
    attn_decode_partial_kernel<HD><<<g1, ATT_THREADS, L::bytes, ctx->stream>>>(
        q, k, v, seq_stride, capacity, ctx_len, H, Hkv, chunk, sm_scale, softcap, part);
    int st = check_cuda(cudaGetLastError(), "attn_decode_partial launch");
    if (st) return st;
    dim3 g2(H, batch);
    attn_decode_combine_kernel<HD><<<g2, HD, 0, ctx->stream>>>(part, H, splits, out);
    ctx->launches += 2;
    return check_cuda(cudaGetLastError(), "attn_decode_combine launch");
}

}  // namespace

void attn_decode_split_range(size_t context_len, int head_count_kv, int batch, int num_sms,
                             int* min_splits, int* default_splits) {
    size_t mn = (context_len + ATT_PMAX - 1) / ATT_PMAX;
    *min_splits = (int)(mn < 1 ? 1 : mn);
    *default_splits = pick_splits(context_len, head_count_kv, batch, num_sms);
}

int launch_attn_decode_with_splits(sulimo_ctx* ctx, const float* q, const void* k_ring,
                                   const void* v_ring, size_t seq_stride, size_t capacity,
                                   size_t context_len, int head_count, int head_count_kv,
                                   int head_dim, int batch, float softcap, float* out,
                                   float* partials, int splits) {
    const uint8_t* k = reinterpret_cast<const uint8_t*>(k_ring);
    const uint8_t* v = reinterpret_cast<const uint8_t*>(v_ring);
    switch (head_dim) {
        case 32: return launch_hd<32>(ctx, q, k, v, seq_stride, capacity, context_len, head_count, head_count_kv, batch, softcap, out, partials, splits);
        case 64: return launch_hd<64>(ctx, q, k, v, seq_stride, capacity, context_len, head_count, head_count_kv, batch, softcap, out, partials, splits);
        case 96: return launch_hd<96>(ctx, q, k, v, seq_stride, capacity, context_len, head_count, head_count_kv, batch, softcap, out, partials, splits);
        case 128: return launch_hd<128>(ctx, q, k, v, seq_stride, capacity, context_len, head_count, head_count_kv, batch, softcap, out, partials, splits);
        case 256: return launch_hd<256>(ctx, q, k, v, seq_stride, capacity, context_len, head_count, head_count_kv, batch, softcap, out, partials, splits);
        default: return set_error(SULIMO_EINVAL, "head_dim must be one of 32, 64, 96, 128, 256");
    }
}

size_t attn_decode_partial_bytes(size_t context_len, int head_count, int head_dim, int batch,
                                 int num_sms, int* splits_out) {
    // head_count_kv only steers the split count; the byte bound uses the worst case (Hkv = 1)
    int splits = pick_splits(context_len, 1, batch, num_sms);
    if (splits_out) *splits_out = splits;
    return (size_t)batch * head_count * splits * (head_dim + 2) * sizeof(float);
}

int launch_attn_decode(sulimo_ctx* ctx, const float* q, const void* k_ring, const void* v_ring,
                       size_t seq_stride, size_t capacity, size_t context_len, int head_count,
                       int head_count_kv, int head_dim, int batch, float softcap, float* out,
                       float* partials, size_t partial_bytes) {
    const int splits = pick_splits(context_len, head_count_kv, batch, ctx->num_sms);
    const size_t need = (size_t)batch * head_count * splits * (head_dim + 2) * sizeof(float);
    if (need > partial_bytes) return set_error(SULIMO_EINVAL, "attention workspace too small");
    const uint8_t* k = reinterpret_cast<const uint8_t*>(k_ring);
    const uint8_t* v = reinterpret_cast<const uint8_t*>(v_ring);
    switch (head_dim) {
        case 32: return launch_hd<32>(ctx, q, k, v, seq_stride, capacity, context_len, head_count, head_count_kv, batch, softcap, out, partials, splits);
        case 64: return launch_hd<64>(ctx, q, k, v, seq_stride, capacity, context_len, head_count, head_count_kv, batch, softcap, out, partials, splits);
        case 96: return launch_hd<96>(ctx, q, k, v, seq_stride, capacity, context_len, head_count, head_count_kv, batch, softcap, out, partials, splits);
        case 128: return launch_hd<128>(ctx, q, k, v, seq_stride, capacity, context_len, head_count, head_count_kv, batch, softcap, out, partials, splits);
        case 256: return launch_hd<256>(ctx, q, k, v, seq_stride, capacity, context_len, head_count, head_count_kv, batch, softcap, out, partials, splits);
        default: return set_error(SULIMO_EINVAL, "head_dim must be one of 32, 64, 96, 128, 256");
    }
}

}  // namespace sulimo
