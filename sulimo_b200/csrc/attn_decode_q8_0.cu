// attn_decode_q8_0.cu — single-position causal GQA attention over the Q8_0 KV ring.
//
// Restates causal_gqa_decode_scalar_ext (crates/sulimo-cpu/src/scalar.rs:287-359) with the ring
// addressing of KvCache::key_ptr / value_ptr (crates/sulimo-core/src/kv_cache.rs:114-128):
//   for each query head h (kv head h / (H/Hkv)):
//     score[p] = (q_h . dequant(K[p % cap])) * 1/sqrt(hd)   [optionally tanh soft-capped]
//     w = softmax(score[0..ctx]);  out_h = sum_p w[p] * dequant(V[p % cap])
//
// B200 form (split-K over the context, "flash-decoding"), two kernels:
//   kernel 1 computes, per (sequence, query head, context split), the split's max score m, the
//   sum l of exp(score - m) and o = sum exp(score - m) * v, into a workspace.  K/V are read once
//   for all H/Hkv query heads of a kv head (the scalar reference re-reads them per query head).
//   Two forms:
//     slot form (default): one CTA per (split, sequence) covering all kv heads; its positions
//       are contiguous ring slots fetched with two bulk copies (exact bytes);
//     per-head form (ring wrap, unaligned rings, too few splits for the slot form's shared
//       memory): one CTA per (split, kv head, sequence), K/V rows staged by TMA tensor copies
//       or, when the rows are not 16-byte aligned, by 2-byte loads.
//   kernel 2 merges the splits: out = sum_s o_s e^{m_s-M} / sum_s l_s e^{m_s-M}.
// Reordered fp32 sums: the result matches the reference within fp32 rounding (the parity
// tests bound the relative L2 error at 2e-3).
#include <string.h>

#include "sulimo_common.cuh"
#include "sulimo_internal.h"

namespace sulimo {
namespace {

constexpr int ATT_THREADS = 128;
constexpr int ATT_PMAX = 256;  // positions per split
constexpr int ATT_GMAX = 8;    // query heads per kv head
constexpr int ATT_SMEM_SLACK = 128;  // room to align the dynamic region to 128 bytes

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
    // TMA staging: the head row of NB*34 bytes starts at a 2-byte aligned offset; the copy
    // starts at the 16-byte boundary below it and is BOXW bytes wide (<= 14 bytes of lead-in).
    static constexpr int HB = NB * 34;
    static constexpr int BOXW = ((HB + 14 + 15) / 16) * 16;
    static constexpr size_t raw_off = (bytes + 127) / 128 * 128;
    __host__ __device__ static size_t raw_bytes(int chunk) { return ((size_t)chunk * BOXW + 127) / 128 * 128; }
    __host__ __device__ static size_t tma_bytes(int chunk) { return raw_off + 2 * raw_bytes(chunk) + 16; }
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

// Same repacking as stage_rows, from a TMA tile in shared memory: position pos of the tile is
// the raw row at raw + pos*BOXW, the head's bytes start `off` bytes into it.
template <int HD>
__device__ __forceinline__ void repack_rows(const uint8_t* raw, int off, int np, float* sc,
                                            uint8_t* qs) {
    using L = AttnLayout<HD>;
    constexpr int W = L::NB * 17;
    for (int it = threadIdx.x; it < np * W; it += ATT_THREADS) {
        const int pos = it / W, w = it - pos * W;
        const int b = w / 17, k = w - b * 17;
        const uint16_t v =
            *reinterpret_cast<const uint16_t*>(raw + (size_t)pos * L::BOXW + off + b * 34 + 2 * k);
        if (k == 0)
            sc[pos * L::NB + b] = f16_bits_to_f32(v);
        else
            *reinterpret_cast<uint16_t*>(qs + pos * L::QS_STRIDE + b * 32 + 2 * (k - 1)) = v;
    }
}

// Sign-extended byte I of w as an exact float: prmt replicates the byte's sign into the upper
// bytes, and 1.5*2^23 + v (|v| < 2^22) has an integer ulp, so one add/subtract converts exactly.
template <int I>
__device__ __forceinline__ float s8_to_f32(uint32_t w) {
    constexpr uint32_t sel = (uint32_t)I | ((0x8u | I) << 4) | ((0x8u | I) << 8) | ((0x8u | I) << 12);
    const int v = (int)prmt(w, 0u, sel);
    return __fsub_rn(__int_as_float(0x4B400000 + v), 12582912.0f);
}

__device__ __forceinline__ float int_to_f32_exact(int v) {
    return __fsub_rn(__int_as_float(0x4B400000 + v), 12582912.0f);
}

template <int HD, int G, bool TMA>
__global__ void __launch_bounds__(ATT_THREADS)
    attn_decode_partial_kernel(const float* __restrict__ q, const uint8_t* __restrict__ kring,
                               const uint8_t* __restrict__ vring, size_t seq_stride,
                               size_t capacity, size_t ctx_len, int H, int Hkv, int chunk,
                               float sm_scale, float softcap, float* __restrict__ part,
                               const __grid_constant__ CUtensorMap tmap_k,
                               const __grid_constant__ CUtensorMap tmap_v, int* __restrict__ err) {
    pdl_launch_dependents();
    pdl_wait_prerequisites();
    using L = AttnLayout<HD>;
    extern __shared__ __align__(16) uint8_t smem_raw[];
    // The dynamic region follows the static `red` array, so its base is only 16-byte aligned;
    // TMA destinations need 128 bytes: align explicitly (the launch adds ATT_SMEM_SLACK).
    uint8_t* smem = smem_raw + ((128u - (smem_u32(smem_raw) & 127u)) & 127u);
    float* sq = reinterpret_cast<float*>(smem + L::q_off);
    float* sc = reinterpret_cast<float*>(smem + L::sc_off);
    uint8_t* qs = smem + L::qs_off;
    float* se = reinterpret_cast<float*>(smem + L::e_off);
    __shared__ float red[ATT_THREADS / 32][G];

    const int split = blockIdx.x, kvh = blockIdx.y, seq = blockIdx.z;
    const int splits = gridDim.x;
    const size_t p0 = (size_t)split * chunk;
    const int np = (int)min((size_t)chunk, ctx_len > p0 ? ctx_len - p0 : (size_t)0);
    const size_t hb = (size_t)L::NB * 34;
    const size_t bpp = (size_t)Hkv * hb;
    const size_t head_off = (size_t)kvh * hb;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;

    uint8_t* raw_k = smem + L::raw_off;
    uint8_t* raw_v = raw_k + L::raw_bytes(chunk);
    uint64_t* bar = reinterpret_cast<uint64_t*>(raw_v + L::raw_bytes(chunk));
    const int x0 = (int)(head_off & ~(size_t)15), off = (int)(head_off & 15);
    if (TMA) {
        // both tiles are requested up front; V lands while the scores are computed
        if (tid == 0) {
            mbar_init(&bar[0], 1);
            mbar_init(&bar[1], 1);
            fence_barrier_init();
        }
        __syncthreads();
        if (tid == 0) {
            mbar_arrive_expect_tx(&bar[0], (uint32_t)(chunk * L::BOXW));
            tma_load_3d(raw_k, &tmap_k, x0, (int)p0, seq, &bar[0]);
            mbar_arrive_expect_tx(&bar[1], (uint32_t)(chunk * L::BOXW));
            tma_load_3d(raw_v, &tmap_v, x0, (int)p0, seq, &bar[1]);
        }
    }
    // query heads of this group (unrolled: the loads of a batch issue before its stores)
#pragma unroll 4
    for (int i = tid; i < G * HD; i += ATT_THREADS)
        sq[i] = q[((size_t)seq * H + (size_t)kvh * G) * HD + i];
    if (TMA) {
        const bool ok = mbar_wait_bounded(&bar[0], 0, err, nullptr);
        repack_rows<HD>(raw_k, off, ok ? np : 0, sc, qs);
    } else {
        stage_rows<HD>(kring + (size_t)seq * seq_stride, capacity, bpp, head_off, p0, np, sc, qs);
    }
    __syncthreads();

    // ---- scores: one thread per position; the block scale is applied to each block's sum ----
    for (int pos = tid; pos < np; pos += ATT_THREADS) {
        float dot[G];
#pragma unroll
        for (int g = 0; g < G; g++) dot[g] = 0.0f;
        const uint8_t* row = qs + pos * L::QS_STRIDE;
#pragma unroll
        for (int b = 0; b < L::NB; b++) {
            float blk[G];
#pragma unroll
            for (int g = 0; g < G; g++) blk[g] = 0.0f;
#pragma unroll
            for (int i16 = 0; i16 < 2; i16++) {
                // 16-byte loads: with the 16-byte row skew, 8 lanes hit 8 distinct bank groups
                const uint4 w4 = *reinterpret_cast<const uint4*>(row + b * 32 + i16 * 16);
                const uint32_t ws[4] = {w4.x, w4.y, w4.z, w4.w};
#pragma unroll
                for (int i4 = 0; i4 < 4; i4++) {
                    const float k0 = s8_to_f32<0>(ws[i4]), k1 = s8_to_f32<1>(ws[i4]);
                    const float k2 = s8_to_f32<2>(ws[i4]), k3 = s8_to_f32<3>(ws[i4]);
                    const int d = b * 32 + i16 * 16 + i4 * 4;
#pragma unroll
                    for (int g = 0; g < G; g++) {
                        const float4 qv = *reinterpret_cast<const float4*>(sq + g * HD + d);
                        blk[g] = __fmaf_rn(qv.x, k0, blk[g]);
                        blk[g] = __fmaf_rn(qv.y, k1, blk[g]);
                        blk[g] = __fmaf_rn(qv.z, k2, blk[g]);
                        blk[g] = __fmaf_rn(qv.w, k3, blk[g]);
                    }
                }
            }
            const float s = sc[pos * L::NB + b];
#pragma unroll
            for (int g = 0; g < G; g++) dot[g] = __fmaf_rn(blk[g], s, dot[g]);
        }
#pragma unroll
        for (int g = 0; g < G; g++) {
            float score = __fmul_rn(dot[g], sm_scale);
            if (softcap > 0.0f) score = tanhf(score / softcap) * softcap;
            se[g * ATT_PMAX + pos] = score;
        }
    }
    __syncthreads();

    // ---- split max and sum of exp, per query head ----
    float mloc[G], lloc[G];
#pragma unroll
    for (int g = 0; g < G; g++) {
        float m = -INFINITY;
        for (int pos = tid; pos < np; pos += ATT_THREADS) m = fmaxf(m, se[g * ATT_PMAX + pos]);
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
        if (lane == 0) red[warp][g] = m;
    }
    __syncthreads();
#pragma unroll
    for (int g = 0; g < G; g++) {
        float m = red[0][g];
        for (int w = 1; w < ATT_THREADS / 32; w++) m = fmaxf(m, red[w][g]);
        mloc[g] = m;
    }
    __syncthreads();
#pragma unroll
    for (int g = 0; g < G; g++) {
        float l = 0.0f;
        for (int pos = tid; pos < np; pos += ATT_THREADS) {
            const float e = expf(se[g * ATT_PMAX + pos] - mloc[g]);
            se[g * ATT_PMAX + pos] = e;
            l += e;
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) l += __shfl_xor_sync(0xffffffffu, l, o);
        if (lane == 0) red[warp][g] = l;
    }
    __syncthreads();
#pragma unroll
    for (int g = 0; g < G; g++) {
        float l = 0.0f;
        for (int w = 0; w < ATT_THREADS / 32; w++) l += red[w][g];
        lloc[g] = l;
    }

    // ---- V: stage, then one thread per head dimension (groups of threads split positions) ----
    if (TMA) {
        const bool ok = mbar_wait_bounded(&bar[1], 0, err, nullptr);
        repack_rows<HD>(raw_v, off, ok ? np : 0, sc, qs);
    } else {
        stage_rows<HD>(vring + (size_t)seq * seq_stride, capacity, bpp, head_off, p0, np, sc, qs);
    }
    __syncthreads();
    constexpr int DPT = (HD + ATT_THREADS - 1) / ATT_THREADS;  // dims per thread
    constexpr int GROUPS = (HD >= ATT_THREADS) ? 1 : ATT_THREADS / HD;
    const int grp = tid / (ATT_THREADS / GROUPS);
    const int dt = tid % (ATT_THREADS / GROUPS);
    float o[G][DPT];
#pragma unroll
    for (int g = 0; g < G; g++)
#pragma unroll
        for (int k = 0; k < DPT; k++) o[g][k] = 0.0f;
    for (int pos = grp; pos < np; pos += GROUPS) {
#pragma unroll
        for (int k = 0; k < DPT; k++) {
            const int d = dt + k * ATT_THREADS;
            if (d < HD) {
                const int b = d / 32;
                const float v = __fmul_rn(
                    int_to_f32_exact((int)*reinterpret_cast<const int8_t*>(qs + pos * L::QS_STRIDE + d)),
                    sc[pos * L::NB + b]);
#pragma unroll
                for (int g = 0; g < G; g++) o[g][k] = __fmaf_rn(se[g * ATT_PMAX + pos], v, o[g][k]);
            }
        }
    }
    // reduce the position groups through shared memory (reuse the score area)
    __syncthreads();
    float* ored = se;  // [GROUPS][G][HD] <= GMAX*PMAX floats
    if (GROUPS > 1) {
#pragma unroll
        for (int g = 0; g < G; g++)
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
        for (int g = 0; g < G; g++) {
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

// ---------------------------------------------------------------------------------------------
// Slot form: one CTA per (context split, sequence) covering ALL kv heads.  Positions
// p0..p0+np-1 of a ring are np contiguous slots, so K and V arrive with one bulk copy each
// (exactly the algorithmic bytes, no tensor map).  Used when the context does not wrap the
// ring and the slot size is a multiple of 16 bytes (Qwen2.5-1.5B: 272 B, Llama-3.2-3B: 1088 B).
//   scores : item (position, kv head) split over adjacent lanes, one 32-dim Q8_0 block each
//            (G dot products read in place with 2-byte loads: 34-byte blocks are 2-byte
//            aligned; times the block scale), summed across the lane group by shuffles;
//   softmax: one warp per (kv head, query head) row over the split's positions;
//   V      : weights pre-multiplied by V's block scales, item (kv head, dim) accumulates
//            sum_pos w[g][pos][b] * v_int[pos][d] for the G query heads.
// Threads per CTA: the phases' serial latency, not bytes, bounds the kernel, so a grid of at
// most one CTA per SM (one sequence) runs 1024 threads; larger grids (several sequences) run
// 256 so that two CTAs share an SM (measured on config 4: batch 1 1.39 -> 1.28 ms per step
// with 1024, batch 8 5.18 -> 5.54 ms with 1024 everywhere).
constexpr int SLOT_THREADS_WIDE = 1024;
constexpr int SLOT_THREADS_NARROW = 256;
constexpr size_t SLOT_SMEM_MAX = 200 * 1024;

// Query row of a kv head in shared memory: [G][NB][34] floats (each 32-dim block padded to 34,
// so the NB lanes of one score item read different banks) and the row itself padded to
// 8 (mod 32) words, so 8 kv heads x 4 blocks of float2 reads take the minimum 2 wavefronts.
__host__ __device__ constexpr int slot_qrow(int G, int NB) {
    return G * NB * 34 + (8 - (G * NB * 34) % 32 + 32) % 32;
}

template <int HD, int G>
struct SlotLayout {
    static constexpr int NB = HD / 32;
    static constexpr int HB = NB * 34;
    static constexpr int QROW = slot_qrow(G, NB);
    __host__ __device__ static size_t raw_bytes(int chunk, int Hkv) {
        return ((size_t)chunk * Hkv * HB + 127) / 128 * 128;
    }
    __host__ __device__ static size_t q_off(int chunk, int Hkv) { return 2 * raw_bytes(chunk, Hkv); }
    __host__ __device__ static size_t e_off(int chunk, int Hkv) {
        return q_off(chunk, Hkv) + (size_t)Hkv * QROW * 4;
    }
    __host__ __device__ static size_t w_off(int chunk, int Hkv) {  // [Hkv][G][chunk][NB]
        return e_off(chunk, Hkv) + (size_t)Hkv * G * chunk * 4;
    }
    __host__ __device__ static size_t stat_off(int chunk, int Hkv) {  // m, l per row
        return w_off(chunk, Hkv) + (size_t)Hkv * G * chunk * NB * 4;
    }
    __host__ __device__ static size_t bar_off(int chunk, int Hkv) {
        return (stat_off(chunk, Hkv) + (size_t)Hkv * G * 8 + 15) / 16 * 16;
    }
    static size_t bytes(int chunk, int Hkv) { return bar_off(chunk, Hkv) + 16 + 128; }
};

// two sign-extended bytes of a little-endian 16-bit word, as exact floats
__device__ __forceinline__ void s8x2_to_f32(uint32_t w, float& lo, float& hi) {
    lo = __fsub_rn(__int_as_float(0x4B400000 + (int)prmt(w, 0u, 0x8880)), 12582912.0f);
    hi = __fsub_rn(__int_as_float(0x4B400000 + (int)prmt(w, 0u, 0x9991)), 12582912.0f);
}

template <int HD, int G, int SLOT_THREADS>
__global__ void __launch_bounds__(SLOT_THREADS)
    attn_decode_slots_kernel(const float* __restrict__ q, const uint8_t* __restrict__ kring,
                             const uint8_t* __restrict__ vring, size_t seq_stride,
                             size_t ctx_len, int H, int Hkv, int chunk, float sm_scale,
                             float softcap, float* __restrict__ part, int* __restrict__ err) {
    pdl_launch_dependents();
    pdl_wait_prerequisites();
    using L = SlotLayout<HD, G>;
    extern __shared__ __align__(16) uint8_t smem_raw[];
    uint8_t* smem = smem_raw + ((128u - (smem_u32(smem_raw) & 127u)) & 127u);
    uint8_t* raw_k = smem;
    uint8_t* raw_v = smem + L::raw_bytes(chunk, Hkv);
    float* sq = reinterpret_cast<float*>(smem + L::q_off(chunk, Hkv));
    float* se = reinterpret_cast<float*>(smem + L::e_off(chunk, Hkv));
    float* sw = reinterpret_cast<float*>(smem + L::w_off(chunk, Hkv));
    float* stat = reinterpret_cast<float*>(smem + L::stat_off(chunk, Hkv));
    uint64_t* bar = reinterpret_cast<uint64_t*>(smem + L::bar_off(chunk, Hkv));

    const int split = blockIdx.x, seq = blockIdx.y, splits = gridDim.x;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const size_t bpp = (size_t)Hkv * L::HB;
    const size_t p0 = (size_t)split * chunk;
    const int np = (int)min((size_t)chunk, ctx_len > p0 ? ctx_len - p0 : (size_t)0);
    const int rows = Hkv * G;

    if (tid == 0) {
        mbar_init(&bar[0], 1);
        mbar_init(&bar[1], 1);
        fence_barrier_init();
    }
    __syncthreads();
    if (tid == 0 && np > 0) {
        const uint32_t bytes = (uint32_t)(np * bpp);
        mbar_arrive_expect_tx(&bar[0], bytes);
        bulk_load(raw_k, kring + (size_t)seq * seq_stride + p0 * bpp, bytes, &bar[0]);
        mbar_arrive_expect_tx(&bar[1], bytes);
        bulk_load(raw_v, vring + (size_t)seq * seq_stride + p0 * bpp, bytes, &bar[1]);
    }
    // query rows, kv head major, blocks padded.  The loads of a batch are all issued before
    // the first shared-memory store (one L2 round trip per 4 * SLOT_THREADS float4).
    {
        const float4* q4 = reinterpret_cast<const float4*>(q + (size_t)seq * H * HD);
        const int n4 = H * HD / 4;
        for (int base = tid; base < n4; base += 4 * SLOT_THREADS) {
            float4 v[4];
#pragma unroll
            for (int u = 0; u < 4; u++) {
                const int i = base + u * SLOT_THREADS;
                v[u] = i < n4 ? q4[i] : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
            }
#pragma unroll
            for (int u = 0; u < 4; u++) {
                const int i = (base + u * SLOT_THREADS) * 4;
                if (i < H * HD) {
                    const int h = i / HD, d = i - h * HD;
                    float* dst = sq + (h / G) * L::QROW + ((h % G) * L::NB + d / 32) * 34 + d % 32;
                    *reinterpret_cast<float2*>(dst) = make_float2(v[u].x, v[u].y);
                    *reinterpret_cast<float2*>(dst + 2) = make_float2(v[u].z, v[u].w);
                }
            }
        }
    }
    bool ok = np > 0 && mbar_wait_bounded(&bar[0], 0, err, nullptr);
    __syncthreads();

    // ---- scores: item (position, kv head) split over NBP adjacent lanes, one 32-dim Q8_0
    // block each (block dot times its scale), summed by xor-shuffles inside the lane group.
    // Every thread runs the same number of rounds, so the shuffles see full warps. ----
    {
        constexpr int NBP = L::NB <= 1 ? 1 : L::NB <= 2 ? 2 : L::NB <= 4 ? 4 : 8;
        const int units = np * Hkv * NBP;
        const int rounds = (units + SLOT_THREADS - 1) / SLOT_THREADS;
        for (int rd = 0; rd < rounds; rd++) {
            const int u = rd * SLOT_THREADS + tid;
            const int b = u & (NBP - 1), item = u / NBP;
            const int kvh = item % Hkv, pos = item / Hkv;
            float acc[G];
#pragma unroll
            for (int g = 0; g < G; g++) acc[g] = 0.0f;
            if (ok && u < units && b < L::NB) {
                const uint16_t* blk = reinterpret_cast<const uint16_t*>(
                    raw_k + (size_t)pos * bpp + kvh * L::HB + b * 34);
                const float* qb = sq + kvh * L::QROW + b * 34;
#pragma unroll
                for (int i = 0; i < 16; i++) {
                    float k0, k1;
                    s8x2_to_f32(blk[1 + i], k0, k1);
#pragma unroll
                    for (int g = 0; g < G; g++) {
                        const float2 qv =
                            *reinterpret_cast<const float2*>(qb + g * L::NB * 34 + 2 * i);
                        acc[g] = __fmaf_rn(qv.x, k0, acc[g]);
                        acc[g] = __fmaf_rn(qv.y, k1, acc[g]);
                    }
                }
                const float sc = f16_bits_to_f32(blk[0]);
#pragma unroll
                for (int g = 0; g < G; g++) acc[g] = __fmul_rn(acc[g], sc);
            }
#pragma unroll
            for (int o = 1; o < NBP; o <<= 1)
#pragma unroll
                for (int g = 0; g < G; g++)
                    acc[g] = __fadd_rn(acc[g], __shfl_xor_sync(0xffffffffu, acc[g], o));
            if (ok && u < units && b == 0) {
#pragma unroll
                for (int g = 0; g < G; g++) {
                    float score = __fmul_rn(acc[g], sm_scale);
                    if (softcap > 0.0f) score = tanhf(score / softcap) * softcap;
                    se[(kvh * G + g) * chunk + pos] = score;
                }
            }
        }
    }
    __syncthreads();

    // ---- softmax over the split: one warp per (kv head, query head) row ----
    for (int r = warp; r < rows; r += SLOT_THREADS / 32) {
        float* e = se + r * chunk;
        float m = -INFINITY;
        for (int pos = lane; pos < np; pos += 32) m = fmaxf(m, e[pos]);
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
        float l = 0.0f;
        for (int pos = lane; pos < np; pos += 32) {
            const float x = expf(e[pos] - m);
            e[pos] = x;
            l += x;
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) l += __shfl_xor_sync(0xffffffffu, l, o);
        if (lane == 0) {
            stat[2 * r] = m;
            stat[2 * r + 1] = l;
        }
    }
    // always wait for V when it was requested: the copy must land before the CTA exits
    if (np > 0) ok = mbar_wait_bounded(&bar[1], 0, err, nullptr) && ok;
    __syncthreads();

    // ---- weights times V's block scales: w[kvh][g][pos][b]; a warp per row, a lane per
    // position (no runtime divisions) ----
    if (ok) {
        for (int r = warp; r < rows; r += SLOT_THREADS / 32) {
            const int kvh = r / G;
            for (int pos = lane; pos < np; pos += 32) {
                const float e = se[r * chunk + pos];
                const uint8_t* vrow = raw_v + (size_t)pos * bpp + kvh * L::HB;
#pragma unroll
                for (int b = 0; b < L::NB; b++)
                    sw[(r * chunk + pos) * L::NB + b] = __fmul_rn(
                        e, f16_bits_to_f32(*reinterpret_cast<const uint16_t*>(vrow + b * 34)));
            }
        }
    }
    __syncthreads();

    // ---- V: item (kv head, dim) ----
    const size_t base = (size_t)seq * H;
    for (int item = tid; item < Hkv * HD; item += SLOT_THREADS) {
        const int kvh = item / HD, d = item - kvh * HD;
        const int b = d >> 5;
        float acc[G];
#pragma unroll
        for (int g = 0; g < G; g++) acc[g] = 0.0f;
        if (ok) {
            const int8_t* col =
                reinterpret_cast<const int8_t*>(raw_v + kvh * L::HB + b * 34 + 2 + (d & 31));
            const float* wr = sw + ((size_t)kvh * G * chunk) * L::NB + b;
#pragma unroll 4
            for (int pos = 0; pos < np; pos++) {
                const float v = __fsub_rn(
                    __int_as_float(0x4B400000 + (int)col[(size_t)pos * bpp]), 12582912.0f);
#pragma unroll
                for (int g = 0; g < G; g++)
                    acc[g] = __fmaf_rn(wr[((size_t)g * chunk + pos) * L::NB], v, acc[g]);
            }
        }
#pragma unroll
        for (int g = 0; g < G; g++) {
            const int h = kvh * G + g;
            float* dst = part + ((base + h) * splits + split) * (HD + 2);
            dst[d] = acc[g];
            if (d == 0) {
                dst[HD] = ok ? stat[2 * h] : -INFINITY;
                dst[HD + 1] = ok ? stat[2 * h + 1] : 0.0f;
            }
        }
    }
}

// Shared-memory bytes of the slot form (must equal SlotLayout<HD, G>::bytes; checked at launch).
size_t slot_bytes_generic(int chunk, int Hkv, int G, int HD) {
    const int NB = HD / 32, HB = NB * 34;
    const size_t raw = ((size_t)chunk * Hkv * HB + 127) / 128 * 128;
    size_t off = 2 * raw + (size_t)Hkv * slot_qrow(G, NB) * 4 + (size_t)Hkv * G * chunk * 4 +
                 (size_t)Hkv * G * chunk * NB * 4;
    off = (off + (size_t)Hkv * G * 8 + 15) / 16 * 16;
    return off + 16 + 128;
}

// Whether the slot form can run this launch: no ring wrap, 16-byte slots, aligned rings, and
// the split's tiles fit the shared-memory budget.
bool slot_form_ok(size_t ctx_len, size_t capacity, int Hkv, int G, int HD, int batch,
                  size_t seq_stride, const void* k, const void* v, int chunk) {
    const size_t bpp = (size_t)Hkv * (HD / 32) * 34;
    const size_t stride = batch > 1 ? seq_stride : 0;
    return ctx_len >= 1 && ctx_len <= capacity && bpp % 16 == 0 && stride % 16 == 0 &&
           ((uintptr_t)k % 16) == 0 && ((uintptr_t)v % 16) == 0 && chunk >= 1 &&
           slot_bytes_generic(chunk, Hkv, G, HD) <= SLOT_SMEM_MAX &&
           (size_t)chunk * bpp < (1u << 30) && batch <= 65535 && G >= 1 && G <= 8;
}

// Split count for the slot form, or 0 when the ring does not allow it: one CTA per SM (the
// merge reads every split's partial row, so more splits cost more than they hide), at least 8
// positions per split, and a chunk whose tiles fit two CTAs per SM.
int slot_splits(size_t ctx_len, size_t capacity, int H, int Hkv, int HD, int batch, int num_sms,
                size_t seq_stride, const void* k, const void* v) {
    const int G = H / Hkv;
    if (G < 1 || G > 8) return 0;
    int max_chunk = 256;
    while (max_chunk > 1 && slot_bytes_generic(max_chunk, Hkv, G, HD) > SLOT_SMEM_MAX / 2)
        max_chunk--;
    if (!slot_form_ok(ctx_len, capacity, Hkv, G, HD, batch, seq_stride, k, v, max_chunk))
        return 0;
    const size_t min_splits = (ctx_len + max_chunk - 1) / max_chunk;
    size_t want = ((size_t)num_sms + batch - 1) / batch;
    const size_t cap8 = (ctx_len + 7) / 8;
    if (want > cap8) want = cap8;
    const size_t s = want > min_splits ? want : min_splits;
    return s > 0x7fffffffu ? 0 : (int)(s < 1 ? 1 : s);
}

// Merge of the splits: out = sum_s o_s e^{m_s - M} / sum_s l_s e^{m_s - M}, M = max_s m_s.
// One CTA per (query head, sequence, 32-dimension slice); lane = dimension.  The 8 warps share
// the splits; each warp keeps a running (max, sum, output) and folds in COMBINE_BATCH splits per
// step whose loads are all issued before any is used (the partials are a few MB read once, so
// the merge is bound by load latency, not bandwidth).  The warps' results are merged in a fixed
// order through shared memory.  With q8 set, the merged block is also written as Q8_0
// (quantize_f32_to_q8_0, the o projection's input in forward_token), in the form(s) q8 names.
constexpr int COMBINE_THREADS = 256;
constexpr int COMBINE_BATCH = 20;  // 148 splits / 8 warps: one batch of loads per warp

template <int HD>
__global__ void __launch_bounds__(COMBINE_THREADS)
    attn_decode_combine_kernel(const float* __restrict__ part, int H, int splits,
                               float* __restrict__ out, const Q8Out q8) {
    pdl_launch_dependents();
    pdl_wait_prerequisites();
    constexpr int W = COMBINE_THREADS / 32;
    __shared__ float sm_m[W], sm_l[W], sm_o[W][32];
    const int h = blockIdx.x, seq = blockIdx.y, d = blockIdx.z * 32 + (threadIdx.x & 31);
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const float* p = part + ((size_t)seq * H + h) * splits * (HD + 2);

    float mw = -INFINITY, lw = 0.0f, ow = 0.0f;
    for (int s0 = warp; s0 < splits; s0 += W * COMBINE_BATCH) {
        float m[COMBINE_BATCH], l[COMBINE_BATCH], o[COMBINE_BATCH];
#pragma unroll
        for (int j = 0; j < COMBINE_BATCH; j++) {
            const int s = s0 + j * W;
            const float* ps = p + (size_t)(s < splits ? s : 0) * (HD + 2);
            m[j] = s < splits ? ps[HD] : -INFINITY;
            l[j] = ps[HD + 1];
            o[j] = ps[d];
        }
        float mb = mw;
#pragma unroll
        for (int j = 0; j < COMBINE_BATCH; j++) mb = fmaxf(mb, m[j]);
        if (mb == -INFINITY) continue;                  // nothing seen yet
        const float r = (mw == -INFINITY) ? 0.0f : expf(mw - mb);
        lw *= r;
        ow *= r;
#pragma unroll
        for (int j = 0; j < COMBINE_BATCH; j++) {
            const float f = (m[j] == -INFINITY) ? 0.0f : expf(m[j] - mb);
            lw = __fmaf_rn(l[j], f, lw);
            ow = __fmaf_rn(o[j], f, ow);
        }
        mw = mb;
    }
    if (lane == 0) {
        sm_m[warp] = mw;
        sm_l[warp] = lw;
    }
    sm_o[warp][lane] = ow;
    __syncthreads();
    if (warp == 0 && d < HD) {
        float M = sm_m[0];
#pragma unroll
        for (int w = 1; w < W; w++) M = fmaxf(M, sm_m[w]);
        float L = 0.0f, O = 0.0f;
#pragma unroll
        for (int w = 0; w < W; w++) {
            const float f = (sm_m[w] == -INFINITY) ? 0.0f : expf(sm_m[w] - M);
            L = __fmaf_rn(sm_l[w], f, L);
            O = __fmaf_rn(sm_o[w][lane], f, O);
        }
        const float val = L > 0.0f ? O / L : 0.0f;
        if (out) out[((size_t)seq * H + h) * HD + d] = val;
        // the CTA's 32 dimensions are exactly one Q8_0 block of the [batch][H*HD] output
        if (q8.aos || q8.codes)
            q8_store_block(q8, val, (size_t)seq, h * (HD / 32) + (int)blockIdx.z, lane);
    }
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

template <int HD, int G>
int launch_hdg(sulimo_ctx* ctx, const float* q, const uint8_t* k, const uint8_t* v,
              size_t seq_stride, size_t capacity, size_t ctx_len, int H, int Hkv, int batch,
              float softcap, float* out, float* part, int splits, const Q8Out& q8) {
    using L = AttnLayout<HD>;
    const int chunk = (int)((ctx_len + splits - 1) / splits);
    const float sm_scale = 1.0f / sqrtf((float)HD);
    if (((uintptr_t)q % 16) == 0 &&
        slot_form_ok(ctx_len, capacity, Hkv, G, HD, batch, seq_stride, k, v, chunk)) {
        using SL = SlotLayout<HD, G>;
        const size_t bytes = SL::bytes(chunk, Hkv);
        if (bytes != slot_bytes_generic(chunk, Hkv, G, HD))
            return set_error(SULIMO_ELAUNCH, "slot layout size mismatch");
        static DeviceBits slot_done;  // per device
        if (!slot_done.test(ctx->device)) {
            int st = check_cuda(
                cudaFuncSetAttribute(attn_decode_slots_kernel<HD, G, SLOT_THREADS_WIDE>,
                                     cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     (int)SLOT_SMEM_MAX),
                "attn slot smem attribute");
            if (!st)
                st = check_cuda(
                    cudaFuncSetAttribute(attn_decode_slots_kernel<HD, G, SLOT_THREADS_NARROW>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)SLOT_SMEM_MAX),
                    "attn slot smem attribute");
            if (st) return st;
            slot_done.set(ctx->device);
        }
        dim3 g1(splits, batch);
        if ((size_t)splits * batch <= (size_t)ctx->num_sms)
            (void)launch_pdl(attn_decode_slots_kernel<HD, G, SLOT_THREADS_WIDE>, g1,
                             dim3(SLOT_THREADS_WIDE), bytes, ctx->stream, q, k, v, seq_stride,
                             ctx_len, H, Hkv, chunk, sm_scale, softcap, part, ctx->d_error);
        else
            (void)launch_pdl(attn_decode_slots_kernel<HD, G, SLOT_THREADS_NARROW>, g1,
                             dim3(SLOT_THREADS_NARROW), bytes, ctx->stream, q, k, v, seq_stride,
                             ctx_len, H, Hkv, chunk, sm_scale, softcap, part, ctx->d_error);
        int st = check_cuda(cudaGetLastError(), "attn_decode_slots launch");
        if (st) return st;
        dim3 g2(H, batch, (HD + 31) / 32);
        (void)launch_pdl(attn_decode_combine_kernel<HD>, g2, dim3(COMBINE_THREADS), 0, ctx->stream,
                         (const float*)part, H, splits, out, q8);
        ctx->launches += 2;
        return check_cuda(cudaGetLastError(), "attn_decode_combine launch");
    }
    static DeviceBits attr_done;  // the attribute is per device
    if (!attr_done.test(ctx->device)) {
        const int max_bytes =
            (int)(L::BOXW <= 256 ? L::tma_bytes(ATT_PMAX) : L::bytes) + ATT_SMEM_SLACK;
        int st = check_cuda(cudaFuncSetAttribute(attn_decode_partial_kernel<HD, G, false>,
                                                 cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                 (int)L::bytes + ATT_SMEM_SLACK),
                            "attn smem attribute");
        if (!st)
            st = check_cuda(cudaFuncSetAttribute(attn_decode_partial_kernel<HD, G, true>,
                                                 cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                 max_bytes),
                            "attn smem attribute");
        if (st) return st;
        attr_done.set(ctx->device);
    }
    // TMA staging when the ring geometry allows 16-byte aligned tensor-map copies and the
    // context does not wrap the ring (positions 0..ctx-1 are slots 0..ctx-1)
    const size_t bpp = (size_t)Hkv * L::HB;
    const size_t stride = batch > 1 ? seq_stride : bpp * capacity;
    const bool tma = L::BOXW <= 256 && ctx_len <= capacity && bpp % 16 == 0 &&
                     stride % 16 == 0 && ((uintptr_t)k % 16) == 0 && ((uintptr_t)v % 16) == 0 &&
                     capacity <= 0x7fffffffu && batch <= 65535;
    CUtensorMap tk, tv;
    memset(&tk, 0, sizeof(tk));
    memset(&tv, 0, sizeof(tv));
    if (tma) {
        const uint64_t dims[3] = {(uint64_t)bpp, (uint64_t)capacity, (uint64_t)batch};
        const uint64_t strides[2] = {(uint64_t)bpp, (uint64_t)stride};
        const uint32_t box[3] = {(uint32_t)L::BOXW, (uint32_t)chunk, 1};
        int st = encode_tensor_map(&tk, CU_TENSOR_MAP_DATA_TYPE_UINT8, k, 3, dims, strides, box,
                                   CU_TENSOR_MAP_SWIZZLE_NONE);
        if (!st)
            st = encode_tensor_map(&tv, CU_TENSOR_MAP_DATA_TYPE_UINT8, v, 3, dims, strides, box,
                                   CU_TENSOR_MAP_SWIZZLE_NONE);
        if (st) return st;
    }
    dim3 g1(splits, Hkv, batch);
    if (tma)
        (void)launch_pdl(attn_decode_partial_kernel<HD, G, true>, g1, dim3(ATT_THREADS),
                         L::tma_bytes(chunk) + ATT_SMEM_SLACK, ctx->stream, q, k, v, seq_stride,
                         capacity, ctx_len, H, Hkv, chunk, sm_scale, softcap, part, tk, tv,
                         ctx->d_error);
    else
        (void)launch_pdl(attn_decode_partial_kernel<HD, G, false>, g1, dim3(ATT_THREADS),
                         L::bytes + ATT_SMEM_SLACK, ctx->stream, q, k, v, seq_stride, capacity,
                         ctx_len, H, Hkv, chunk, sm_scale, softcap, part, tk, tv, ctx->d_error);
    int st = check_cuda(cudaGetLastError(), "attn_decode_partial launch");
    if (st) return st;
    dim3 g2(H, batch, (HD + 31) / 32);
    (void)launch_pdl(attn_decode_combine_kernel<HD>, g2, dim3(COMBINE_THREADS), 0, ctx->stream,
                     (const float*)part, H, splits, out, q8);
    ctx->launches += 2;
    return check_cuda(cudaGetLastError(), "attn_decode_combine launch");
}


// The query-group size is a template parameter so that the inner loops carry no predicated
// lanes for the heads a group does not have.
template <int HD>
int launch_hd(sulimo_ctx* ctx, const float* q, const uint8_t* k, const uint8_t* v,
              size_t seq_stride, size_t capacity, size_t ctx_len, int H, int Hkv, int batch,
              float softcap, float* out, float* part, int splits, const Q8Out& q8) {
    switch (H / Hkv) {
#define SULIMO_ATTN_G(g) \
    case g: return launch_hdg<HD, g>(ctx, q, k, v, seq_stride, capacity, ctx_len, H, Hkv, batch, softcap, out, part, splits, q8);
        SULIMO_ATTN_G(1) SULIMO_ATTN_G(2) SULIMO_ATTN_G(3) SULIMO_ATTN_G(4)
        SULIMO_ATTN_G(5) SULIMO_ATTN_G(6) SULIMO_ATTN_G(7) SULIMO_ATTN_G(8)
#undef SULIMO_ATTN_G
        default: return set_error(SULIMO_EINVAL, "at most 8 query heads per KV head");
    }
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
    const Q8Out none = {nullptr, nullptr, nullptr, 0};
    const uint8_t* k = reinterpret_cast<const uint8_t*>(k_ring);
    const uint8_t* v = reinterpret_cast<const uint8_t*>(v_ring);
    switch (head_dim) {
        case 32: return launch_hd<32>(ctx, q, k, v, seq_stride, capacity, context_len, head_count, head_count_kv, batch, softcap, out, partials, splits, none);
        case 64: return launch_hd<64>(ctx, q, k, v, seq_stride, capacity, context_len, head_count, head_count_kv, batch, softcap, out, partials, splits, none);
        case 96: return launch_hd<96>(ctx, q, k, v, seq_stride, capacity, context_len, head_count, head_count_kv, batch, softcap, out, partials, splits, none);
        case 128: return launch_hd<128>(ctx, q, k, v, seq_stride, capacity, context_len, head_count, head_count_kv, batch, softcap, out, partials, splits, none);
        case 256: return launch_hd<256>(ctx, q, k, v, seq_stride, capacity, context_len, head_count, head_count_kv, batch, softcap, out, partials, splits, none);
        default: return set_error(SULIMO_EINVAL, "head_dim must be one of 32, 64, 96, 128, 256");
    }
}

int attn_decode_splits(size_t context_len, size_t capacity, int head_count, int head_count_kv,
                       int head_dim, int batch, int num_sms, size_t seq_stride, const void* k,
                       const void* v) {
    const int s = slot_splits(context_len, capacity, head_count, head_count_kv, head_dim, batch,
                              num_sms, seq_stride, k, v);
    return s > 0 ? s : pick_splits(context_len, head_count_kv, batch, num_sms);
}

size_t attn_decode_partial_bytes(size_t context_len, size_t capacity, int head_count,
                                 int head_count_kv, int head_dim, int batch, int num_sms,
                                 size_t seq_stride, const void* k, const void* v,
                                 int* splits_out) {
    const int splits = attn_decode_splits(context_len, capacity, head_count, head_count_kv,
                                          head_dim, batch, num_sms, seq_stride, k, v);
    if (splits_out) *splits_out = splits;
    const size_t scalar = (size_t)batch * head_count * splits * (head_dim + 2) * sizeof(float);
    const size_t mma = attn_decode_mma_partial_bytes(context_len, capacity, head_count,
                                                     head_count_kv, head_dim, batch, num_sms,
                                                     seq_stride, k, v);
    return scalar > mma ? scalar : mma;
}

int launch_attn_decode(sulimo_ctx* ctx, const float* q, const void* k_ring, const void* v_ring,
                       size_t seq_stride, size_t capacity, size_t context_len, int head_count,
                       int head_count_kv, int head_dim, int batch, float softcap, float* out,
                       float* partials, size_t partial_bytes, const Q8Out* out_q8_form,
                       size_t static_before) {
    const Q8Out none = {nullptr, nullptr, nullptr, 0};
    const Q8Out& out_q8 = out_q8_form ? *out_q8_form : none;
    // the tensor-core kernel where its geometry applies; the scalar kernels otherwise
    bool used = false;
    const int st = launch_attn_decode_mma(ctx, q, k_ring, v_ring, seq_stride, capacity,
                                          context_len, head_count, head_count_kv, head_dim,
                                          batch, softcap, out, partials, partial_bytes,
                                          out_q8, &used, static_before);
    if (st || used) return st;
    const int splits = attn_decode_splits(context_len, capacity, head_count, head_count_kv,
                                          head_dim, batch, ctx->num_sms, seq_stride, k_ring,
                                          v_ring);
    const size_t need = (size_t)batch * head_count * splits * (head_dim + 2) * sizeof(float);
    if (need > partial_bytes) return set_error(SULIMO_EINVAL, "attention workspace too small");
    const uint8_t* k = reinterpret_cast<const uint8_t*>(k_ring);
    const uint8_t* v = reinterpret_cast<const uint8_t*>(v_ring);
    switch (head_dim) {
        case 32: return launch_hd<32>(ctx, q, k, v, seq_stride, capacity, context_len, head_count, head_count_kv, batch, softcap, out, partials, splits, out_q8);
        case 64: return launch_hd<64>(ctx, q, k, v, seq_stride, capacity, context_len, head_count, head_count_kv, batch, softcap, out, partials, splits, out_q8);
        case 96: return launch_hd<96>(ctx, q, k, v, seq_stride, capacity, context_len, head_count, head_count_kv, batch, softcap, out, partials, splits, out_q8);
        case 128: return launch_hd<128>(ctx, q, k, v, seq_stride, capacity, context_len, head_count, head_count_kv, batch, softcap, out, partials, splits, out_q8);
        case 256: return launch_hd<256>(ctx, q, k, v, seq_stride, capacity, context_len, head_count, head_count_kv, batch, softcap, out, partials, splits, out_q8);
        default: return set_error(SULIMO_EINVAL, "head_dim must be one of 32, 64, 96, 128, 256");
    }
}

}  // namespace sulimo
