// attn_decode_mma.cu — decode attention over the Q8_0 KV ring on the tensor cores.
//
// Restates causal_gqa_decode_scalar_ext (crates/sulimo-cpu/src/scalar.rs:287-359) over the ring
// addressing of KvCache::key_ptr / value_ptr (crates/sulimo-core/src/kv_cache.rs:114-128):
//   score[h][p] = (q_h . dequant(K[p % cap][kv(h)])) / sqrt(hd)   [tanh soft-cap if set]
//   out_h = sum_p softmax_p(score[h]) * dequant(V[p % cap][kv(h)])
// in one kernel, split over the context ("flash-decoding") and merged on the device.
//
// Grid: (context splits, kv heads, sequences).  A CTA covers `chunk` consecutive positions of
// one kv head of one sequence:
//   producer (warp 8): per stage of `sp` positions, one TMA tensor copy each of K and V: the box
//     starts at the 16-byte boundary at or below the head's first byte in the slot and is BOXW
//     bytes wide (the head's hd/32 Q8_0 blocks plus that lead-in; BOXW / 4 is 4 (mod 8) words,
//     so eight consecutive rows start in eight different bank quads), `stages`-deep ring,
//     full / empty mbarriers;
//   consumers (warps 0-7): warp w takes 16-position tiles w, w + 8, ... of each stage.  Per
//     tile, with mma.sync.m16n8k16 (f16 in, fp32 accumulate):
//       S^T[head][pos] = Q . K^T: the A operand holds the group's query rows split in two f16
//         parts, hi = f16(q) in rows 0-7 and lo = f16(q - hi) in rows 8-15 (q enters at ~22
//         bits); B = K's int8 codes, exact in f16; each 32-dimension Q8_0 block is two k-steps
//         into a fresh accumulator, then (hi + lo) * d_K[pos] is added in fp32;
//       online softmax per head in fp32 (running max / sum, exp2);
//       O[head][dim] += P' . V: per 32-dimension block b the A operand is P * d_V[pos][b], again
//         hi / lo f16 in rows 0-7 / 8-15, B = V's int8 codes; O accumulates in fp32.
//   merge: the eight warps' (m, l, o) through shared memory into the CTA's partial, written to
//     the workspace; attn_decode_merge_kernel, a programmatic dependent launch, then merges the
//     splits with one warp per (sequence, query head, 32-dimension block) and writes the output
//     (and, for the decode step, its Q8_0 quantization).  With one split the CTA writes the
//     output directly.
// Numerics: products are exact, sums are fp32 in a different order than the reference's
// sequential loop, and q / P' carry ~22 significant bits: the result matches the reference
// within fp32-level rounding (the parity tests bound the relative L2 error at 2e-3).
#include <string.h>

#include <algorithm>

#include "sulimo_common.cuh"
#include "sulimo_internal.h"

namespace sulimo {
namespace {

constexpr int AM_CONSUMERS = 8;                      // consumer warps
constexpr int AM_THREADS = (AM_CONSUMERS + 1) * 32;  // + one producer warp
constexpr int AM_SP = 16 * AM_CONSUMERS;             // positions per stage: one tile per warp
constexpr int AM_MAX_STAGES = 4;
constexpr int AM_MAX_SPLITS = 32;   // splits per (sequence, kv head): the merge kernel reads
                                    // each output dimension's partials in one batch
constexpr size_t AM_SMEM_MAX = 200 * 1024;
constexpr float AM_LOG2E = 1.4426950408889634f;

struct AttnMmaArgs {
    const float* q;         // [batch][H][HD] fp32
    size_t ctx_len;         // positions 0 .. ctx_len-1 (<= capacity: slot = position)
    size_t static_before;   // positions < this are not written by the previous kernel
    int H, Hkv, G;          // query heads, kv heads, H / Hkv
    int chunk;              // positions per CTA
    int stages;
    int boxw;               // bytes per staged row
    float sm_scale;         // 1 / sqrt(hd)
    float softcap;          // <= 0: none
    float* out;             // [batch][H][HD] or null
    Q8Out q8;               // the output as Q8_0 rows [batch][H * HD] (forms it names)
    float* part;            // [batch][Hkv][splits][G][HD + 2]
    int* err;
};

// ---- small PTX helpers ------------------------------------------------------------------
__device__ __forceinline__ uint32_t lds_u16(const uint8_t* p) {
    return *reinterpret_cast<const uint16_t*>(p);
}

__device__ __forceinline__ float lds_f16(const uint8_t* p) {
    return __half2float(*reinterpret_cast<const __half*>(p));
}

// two int8 codes (bytes 0 and 1 of w) -> the f16 pair {byte0, byte1}, exactly: 0x64XX is
// 1024 + XX as f16, XX = code ^ 0x80 is code + 128, so subtracting 1152 leaves the code.
__device__ __forceinline__ uint32_t s8pair_to_h2(uint32_t w) {
    uint32_t t = prmt(w, 0u, 0x7170u) ^ 0x00800080u;  // {b0, 0, b1, 0} with the sign bit flipped
    t |= 0x64006400u;
    __half2 h = __hsub2(*reinterpret_cast<__half2*>(&t), __floats2half2_rn(1152.0f, 1152.0f));
    return *reinterpret_cast<uint32_t*>(&h);
}

// bytes 0 and 2 of w (int8 codes) -> the f16 pair {byte0, byte2}, exactly (as s8pair_to_h2;
// bytes 1 and 3 are ignored): one LOP3 builds 0x64XX with XX = code ^ 0x80.
__device__ __forceinline__ uint32_t s8sel_to_h2(uint32_t w) {
    uint32_t t = (w & 0x00FF00FFu) ^ 0x64806480u;
    __half2 h = __hsub2(*reinterpret_cast<__half2*>(&t), __floats2half2_rn(1152.0f, 1152.0f));
    return *reinterpret_cast<uint32_t*>(&h);
}

__device__ __forceinline__ uint32_t h2_bits(__half2 h) { return *reinterpret_cast<uint32_t*>(&h); }

// D = A * B + C, m16n8k16, f16 inputs, fp32 accumulators
__device__ __forceinline__ void mma_16816(float* c, const uint32_t* a, uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
        "{%8,%9}, {%0,%1,%2,%3};"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// Merge of n partials (m_i, l_i, o_i[d]) held as [HD + 2] float rows:
//   M = max_i m_i, L = sum_i l_i e^(m_i - M), O = sum_i o_i[d] e^(m_i - M).
// Online over steps of 8 partials whose loads are all issued before any is used (the partials
// sit in another CTA's shared memory or in L2: one round trip per step, not per partial).
// rd(i, j) reads element j of partial i; d >= HD computes only M and L.
template <int HD, typename Read>
__device__ __forceinline__ void merge_rows(int n, int d, Read rd, float* o_out, float* l_out,
                                           float* m_out) {
    float M = -INFINITY, L = 0.0f, O = 0.0f;
    for (int i0 = 0; i0 < n; i0 += 8) {
        float mi[8], li[8], oi[8];
#pragma unroll
        for (int j = 0; j < 8; j++) {
            const bool v = i0 + j < n;
            mi[j] = v ? rd(i0 + j, HD) : -INFINITY;
            li[j] = v ? rd(i0 + j, HD + 1) : 0.0f;
            oi[j] = (v && d < HD) ? rd(i0 + j, d) : 0.0f;
        }
        float Mb = M;
#pragma unroll
        for (int j = 0; j < 8; j++) Mb = fmaxf(Mb, mi[j]);
        if (Mb == -INFINITY) continue;
        const float r = (M == -INFINITY) ? 0.0f : exp2f((M - Mb) * AM_LOG2E);
        L *= r;
        O *= r;
#pragma unroll
        for (int j = 0; j < 8; j++) {
            const float f = (mi[j] == -INFINITY) ? 0.0f : exp2f((mi[j] - Mb) * AM_LOG2E);
            L = __fmaf_rn(li[j], f, L);
            O = __fmaf_rn(oi[j], f, O);
        }
        M = Mb;
    }
    *o_out = O;
    *l_out = L;
    *m_out = M;
}

template <int HD>
__global__ void __launch_bounds__(AM_THREADS, 1)
    attn_decode_mma_kernel(const __grid_constant__ AttnMmaArgs a,
                           const __grid_constant__ CUtensorMap tmap_k,
                           const __grid_constant__ CUtensorMap tmap_v) {
    constexpr int NB = HD / 32, HB = NB * 34, KS = HD / 16, NT = HD / 8;
    constexpr int HD2 = HD + 2;
    extern __shared__ __align__(16) uint8_t smem_raw[];
    uint8_t* smem = smem_raw + ((128u - (smem_u32(smem_raw) & 127u)) & 127u);
    const uint32_t rs = (uint32_t)a.boxw;
    const uint32_t stage_bytes = 2u * AM_SP * rs;
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + (size_t)a.stages * stage_bytes);
    uint64_t* empty = full + a.stages;

    const int split = blockIdx.x, kvh = blockIdx.y, seq = blockIdx.z, splits = gridDim.x;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int g = lane >> 2, tig = lane & 3;
    const size_t p0 = (size_t)split * a.chunk;
    const int np = p0 < a.ctx_len ? (int)min((size_t)a.chunk, a.ctx_len - p0) : 0;
    const int nstage = (np + AM_SP - 1) / AM_SP;
    const int x0 = (kvh * HB) & ~15;           // TMA x coordinate: 16-byte aligned
    const int off = kvh * HB - x0;             // the head's first byte inside a staged row

    if (tid == 0) {
        for (int s = 0; s < a.stages; s++) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], AM_CONSUMERS);
        }
        fence_barrier_init();
        prefetch_tensormap(&tmap_k);
        prefetch_tensormap(&tmap_v);
    }
    __syncthreads();
    pdl_launch_dependents();
    // Stages whose positions all lie below static_before (in a decode step: every slot but the
    // newest) are not written by the previous kernel: their copies start before the wait, so
    // the context streams in while the previous kernels of the step still run.
    int early = 0;
    if (warp == AM_CONSUMERS && lane == 0) {
        while (early < nstage && early < a.stages &&
               p0 + (size_t)min(np, (early + 1) * AM_SP) <= a.static_before) {
            uint8_t* dk = smem + (size_t)early * stage_bytes;
            mbar_arrive_expect_tx(&full[early], stage_bytes);
            const int y = (int)(p0 + (size_t)early * AM_SP);
            tma_load_3d(dk, &tmap_k, x0, y, seq, &full[early]);
            tma_load_3d(dk + (size_t)AM_SP * rs, &tmap_v, x0, y, seq, &full[early]);
            early++;
        }
    }
    // q and the ring's newest slot are written by the previous kernel of the step
    pdl_wait_prerequisites();

    if (warp == AM_CONSUMERS) {
        // ------------------------------ producer ------------------------------
        if (lane == 0) {
            for (int st = early; st < nstage; st++) {
                const int s = st % a.stages;
                if (st >= a.stages &&
                    !mbar_wait_bounded(&empty[s], (uint32_t)((st / a.stages) - 1) & 1u, a.err,
                                       nullptr))
                    break;
                uint8_t* dk = smem + (size_t)s * stage_bytes;
                mbar_arrive_expect_tx(&full[s], stage_bytes);
                const int y = (int)(p0 + (size_t)st * AM_SP);
                tma_load_3d(dk, &tmap_k, x0, y, seq, &full[s]);
                tma_load_3d(dk + (size_t)AM_SP * rs, &tmap_v, x0, y, seq, &full[s]);
            }
        }
    }

    // ------------------------------ consumers ------------------------------
    float oc[NT][4];
    float m_run = -INFINITY, l_run = 0.0f;
#pragma unroll
    for (int n = 0; n < NT; n++) oc[n][0] = oc[n][1] = oc[n][2] = oc[n][3] = 0.0f;
    if (warp < AM_CONSUMERS) {
        // query fragments: row g = f16(q) of head g of this kv head's group, row g + 8 = the
        // f16 remainder; columns 2*tig, 2*tig + 1 (+8) of each 16-dimension k-step
        uint32_t qa[KS][4];
        {
            const bool hv = g < a.G;
            const float* qh = a.q + ((size_t)seq * a.H + (size_t)kvh * a.G + (hv ? g : 0)) * HD;
#pragma unroll
            for (int ks = 0; ks < KS; ks++)
#pragma unroll
                for (int hf = 0; hf < 2; hf++) {
                    const int d = ks * 16 + hf * 8 + 2 * tig;
                    const float x0f = hv ? qh[d] : 0.0f, x1f = hv ? qh[d + 1] : 0.0f;
                    const __half2 hi = __floats2half2_rn(x0f, x1f);
                    const float2 hf2 = __half22float2(hi);
                    const __half2 lo = __floats2half2_rn(x0f - hf2.x, x1f - hf2.y);
                    qa[ks][2 * hf] = h2_bits(hi);
                    qa[ks][2 * hf + 1] = h2_bits(lo);
                }
        }
        const bool capped = a.softcap > 0.0f;
        for (int st = 0; st < nstage; st++) {
            const int s = st % a.stages;
            // warp-uniform: the tile loop below runs warp-wide shuffles and MMAs
            const bool landed = __all_sync(
                0xffffffffu,
                mbar_wait_bounded(&full[s], (uint32_t)(st / a.stages) & 1u, a.err, nullptr));
            const int q0 = st * AM_SP;
            const uint8_t* kst = smem + (size_t)s * stage_bytes + off;
            const uint8_t* vst = kst + (size_t)AM_SP * rs;
            for (int t = warp * 16; landed && t < AM_SP && q0 + t < np; t += AM_CONSUMERS * 16) {
                const int valid = np - (q0 + t);  // rows of this tile that hold positions
                const uint8_t* kt = kst + (size_t)t * rs;
                const uint8_t* vt = vst + (size_t)t * rs;
                // ---- scores: two 8-position n-tiles ----
                float x[4];
#pragma unroll
                for (int nt = 0; nt < 2; nt++) {
                    const uint8_t* krow = kt + (size_t)(nt * 8 + g) * rs;
                    const uint8_t* srow = kt + (size_t)(nt * 8 + 2 * tig) * rs;
                    float s0 = 0.0f, s1 = 0.0f;
#pragma unroll
                    for (int b = 0; b < NB; b++) {
                        float c[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll
                        for (int kk = 0; kk < 2; kk++) {
                            const uint8_t* p = krow + b * 34 + 2 + kk * 16 + 2 * tig;
                            mma_16816(c, qa[2 * b + kk], s8pair_to_h2(lds_u16(p)),
                                      s8pair_to_h2(lds_u16(p + 8)));
                        }
                        s0 = __fmaf_rn(c[0] + c[2], lds_f16(srow + b * 34), s0);
                        s1 = __fmaf_rn(c[1] + c[3], lds_f16(srow + rs + b * 34), s1);
                    }
#pragma unroll
                    for (int j = 0; j < 2; j++) {
                        float v = (j ? s1 : s0) * a.sm_scale;
                        if (capped) v = tanhf(v / a.softcap) * a.softcap;
                        x[nt * 2 + j] = (nt * 8 + 2 * tig + j < valid) ? v : -INFINITY;
                    }
                }
                // ---- online softmax (head g's running max is shared by lanes 4g..4g+3) ----
                float tm = fmaxf(fmaxf(x[0], x[1]), fmaxf(x[2], x[3]));
                tm = fmaxf(tm, __shfl_xor_sync(0xffffffffu, tm, 1));
                tm = fmaxf(tm, __shfl_xor_sync(0xffffffffu, tm, 2));
                const float m_new = fmaxf(m_run, tm);
                float p[4];
                float alpha = 1.0f;
                if (m_new == -INFINITY) {
                    p[0] = p[1] = p[2] = p[3] = 0.0f;
                } else {
                    alpha = (m_run == -INFINITY) ? 0.0f : exp2f((m_run - m_new) * AM_LOG2E);
#pragma unroll
                    for (int i = 0; i < 4; i++)
                        p[i] = (x[i] == -INFINITY) ? 0.0f : exp2f((x[i] - m_new) * AM_LOG2E);
                }
                l_run = __fmaf_rn(l_run, alpha, (p[0] + p[1]) + (p[2] + p[3]));
                m_run = m_new;
                if (__any_sync(0xffffffffu, alpha != 1.0f)) {
#pragma unroll
                    for (int n = 0; n < NT; n++) {
                        oc[n][0] *= alpha;
                        oc[n][1] *= alpha;
                        oc[n][2] *= alpha;
                        oc[n][3] *= alpha;
                    }
                }
                // ---- O += P' . V, per 32-dimension block ----
                const uint8_t* v0 = vt + (size_t)(2 * tig) * rs;  // rows 2tig, +1, +8, +9
#pragma unroll
                for (int b = 0; b < NB; b++) {
                    float pp[4];
#pragma unroll
                    for (int i = 0; i < 4; i++) {
                        const int row = (i >> 1) * 8 + (i & 1);
                        pp[i] = p[i] != 0.0f ? p[i] * lds_f16(v0 + (size_t)row * rs + b * 34)
                                             : 0.0f;
                    }
                    uint32_t A[4];
                    {
                        const __half2 h01 = __floats2half2_rn(pp[0], pp[1]);
                        const float2 f01 = __half22float2(h01);
                        const __half2 h89 = __floats2half2_rn(pp[2], pp[3]);
                        const float2 f89 = __half22float2(h89);
                        A[0] = h2_bits(h01);
                        A[1] = h2_bits(__floats2half2_rn(pp[0] - f01.x, pp[1] - f01.y));
                        A[2] = h2_bits(h89);
                        A[3] = h2_bits(__floats2half2_rn(pp[2] - f89.x, pp[3] - f89.y));
                    }
                    // n-tile n4, column c <-> dimension 32b + 4c + n4: lane group g needs dims
                    // 4g .. 4g+3 of the block at each of its four positions, one 4-byte word
                    // per position (two 2-byte loads where the word is 2-byte aligned: the
                    // codes of even blocks start 2 bytes past a 4-byte boundary)
                    uint32_t w[4];
#pragma unroll
                    for (int i = 0; i < 4; i++) {
                        const uint8_t* cp =
                            v0 + (size_t)((i >> 1) * 8 + (i & 1)) * rs + b * 34 + 2 + 4 * g;
                        w[i] = (b & 1) ? *reinterpret_cast<const uint32_t*>(cp)
                                       : prmt(lds_u16(cp), lds_u16(cp + 2), 0x5410u);
                    }
#pragma unroll
                    for (int n4 = 0; n4 < 4; n4++) {
                        const uint32_t sel = (uint32_t)n4 | ((uint32_t)(4 + n4) << 8);
                        const uint32_t b0 = s8sel_to_h2(prmt(w[0], w[1], sel));
                        const uint32_t b1 = s8sel_to_h2(prmt(w[2], w[3], sel));
                        mma_16816(oc[b * 4 + n4], A, b0, b1);
                    }
                }
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[s]);
        }
    }
    __syncthreads();  // every stage consumed: the stage memory becomes the merge area

    // ---- the warps' (m, l, o) per head -> wpart[warp][g][HD + 2] -> the CTA partial ----
    float* wpart = reinterpret_cast<float*>(smem);
    if (warp < AM_CONSUMERS) {
        float l_tot = l_run + __shfl_xor_sync(0xffffffffu, l_run, 1);
        l_tot += __shfl_xor_sync(0xffffffffu, l_tot, 2);
        if (g < a.G) {
            float* row = wpart + ((size_t)warp * a.G + g) * HD2;
#pragma unroll
            for (int n = 0; n < NT; n++) {  // n = 4b + n4: dims 32b + 4c + n4, c = 2tig, +1
                row[(n >> 2) * 32 + 8 * tig + (n & 3)] = oc[n][0] + oc[n][2];
                row[(n >> 2) * 32 + 8 * tig + 4 + (n & 3)] = oc[n][1] + oc[n][3];
            }
            if (tig == 0) {
                row[HD] = m_run;
                row[HD + 1] = l_tot;
            }
        }
    }
    __syncthreads();
    const bool direct = splits == 1;
    float* dst_part = a.part + (((size_t)seq * a.Hkv + kvh) * splits + split) * a.G * HD2;
    // items (g, d), d in [0, HD + 32): dimensions, then m and l; warps align to Q8_0 blocks
    constexpr int HDP = HD + 32;
    for (int it = tid; it < a.G * HDP; it += AM_THREADS) {
        const int gg = it / HDP, d = it % HDP;
        if (d >= HD2) continue;
        auto rd = [&](int i, int dd) { return wpart[((size_t)i * a.G + gg) * HD2 + dd]; };
        float o, l, m;
        merge_rows<HD>(AM_CONSUMERS, d < HD ? d : HD, rd, &o, &l, &m);
        if (direct) {
            if (d < HD) {
                const size_t h = (size_t)kvh * a.G + gg;
                const float val = l > 0.0f ? o / l : 0.0f;
                if (a.out) a.out[((size_t)seq * a.H + h) * HD + d] = val;
                if (a.q8.aos || a.q8.codes)
                    q8_store_block(a.q8, val, (size_t)seq, (int)(h * NB + d / 32), lane);
            }
        } else {
            dst_part[(size_t)gg * HD2 + d] = d < HD ? o : (d == HD ? m : l);
        }
    }
}

// Merge of the splits' partials: one warp per (sequence, query head, 32-dimension block), lane =
// dimension.  Lane s loads split s's (m, l) (splits <= 32) and every lane its dimension of each
// split's o, all issued before any is used; M is a warp max, split s's weight e_s =
// e^(m_s - M) is computed once by lane s and broadcast by shuffle, L = sum_s l_s e_s and
// O = sum_s o_s e_s in split order, out = O / L; the block is also written as one Q8_0 block
// when asked (the decode step's o-projection input).  A programmatic dependent of the split
// kernel: the loads wait in griddepcontrol.wait, the launch overlaps the split kernel's tail.
// The code is kept short (it runs once per launch from a cold instruction cache).
template <int HD>
__global__ void __launch_bounds__(128)
    attn_decode_merge_kernel(const __grid_constant__ AttnMmaArgs a, int splits) {
    constexpr int NB = HD / 32, HD2 = HD + 2;
    pdl_launch_dependents();
    const int lane = threadIdx.x & 31;
    const int item = blockIdx.x * 4 + (threadIdx.x >> 5);  // (head, block)
    const int seq = blockIdx.y;
    if (item >= a.H * NB) return;
    const int h = item / NB, b = item % NB;
    const int kvh = h / a.G, gg = h % a.G;
    const float* base = a.part + ((size_t)seq * a.Hkv + kvh) * splits * a.G * HD2 +
                        (size_t)gg * HD2;
    const size_t sstride = (size_t)a.G * HD2;
    pdl_wait_prerequisites();
    const bool mine = lane < splits;
    const float ms = mine ? __ldcg(base + (size_t)lane * sstride + HD) : -INFINITY;
    const float ls = mine ? __ldcg(base + (size_t)lane * sstride + HD + 1) : 0.0f;
    float oi[AM_MAX_SPLITS];
#pragma unroll
    for (int sp = 0; sp < AM_MAX_SPLITS; sp++)
        oi[sp] = sp < splits ? __ldcg(base + (size_t)sp * sstride + b * 32 + lane) : 0.0f;
    float M = ms;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, o));
    const float es = (ms == -INFINITY) ? 0.0f : exp2f((ms - M) * AM_LOG2E);
    float L = ls * es;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) L += __shfl_xor_sync(0xffffffffu, L, o);
    float O = 0.0f;
#pragma unroll
    for (int sp = 0; sp < AM_MAX_SPLITS; sp++) {
        const float e = __shfl_sync(0xffffffffu, es, sp);
        if (sp < splits) O = __fmaf_rn(oi[sp], e, O);
    }
    const float val = L > 0.0f ? O / L : 0.0f;
    if (a.out) a.out[((size_t)seq * a.H + h) * HD + b * 32 + lane] = val;
    if (a.q8.aos || a.q8.codes) q8_store_block(a.q8, val, (size_t)seq, h * NB + b, lane);
}

struct MmaPlan {
    int splits, chunk, stages, boxw;
    size_t smem;
};

// Geometry of the tensor-core form, or false when it does not apply (the caller falls back to
// the scalar kernels): hd 64 / 128, at most 8 query heads per kv head, 16-byte slots and ring
// bases, a context inside the ring (positions are slots), and at least 8 (kv head, sequence)
// pairs.  With fewer pairs (Qwen2.5-1.5B's 2 kv heads at batch 1) the context splits 16+ ways
// per head and the merge's latency outweighs the tensor cores: the slot form of the scalar
// kernel, one CTA per split over all kv heads, is faster there (config 3 decode: 1.03 against
// 1.28 ms per token).
bool mma_plan(size_t ctx_len, size_t capacity, int H, int Hkv, int HD, int batch, int num_sms,
              size_t seq_stride, const void* k, const void* v, MmaPlan* pl) {
    if (HD != 64 && HD != 128) return false;
    if (Hkv < 1 || H % Hkv != 0 || H / Hkv > 8 || Hkv > 65535) return false;
    if ((size_t)Hkv * batch < 8) return false;
    const size_t HB = (size_t)(HD / 32) * 34, bpp = (size_t)Hkv * HB;
    if (bpp % 16 || ((uintptr_t)k % 16) || ((uintptr_t)v % 16)) return false;
    if (batch > 1 && seq_stride % 16) return false;
    if (ctx_len < 1 || ctx_len > capacity || capacity > 0x7fffffff || batch < 1 ||
        batch > 65535)
        return false;
    int lead = 0;
    for (int h = 0; h < Hkv && h < 16; h++) lead = std::max(lead, (int)((h * HB) % 16));
    int boxw = (int)((lead + HB + 15) / 16 * 16);
    while ((boxw / 4) % 8 != 4) boxw += 16;  // eight rows in eight different bank quads
    if (boxw > 256) return false;
    pl->boxw = boxw;
    const size_t stage = 2u * AM_SP * boxw;
    pl->stages = (int)((AM_SMEM_MAX - 512) / stage);
    if (pl->stages > AM_MAX_STAGES) pl->stages = AM_MAX_STAGES;
    if (pl->stages < 1) return false;
    const size_t G = (size_t)(H / Hkv);
    if ((size_t)AM_CONSUMERS * G * (HD + 2) * 4 > (size_t)pl->stages * stage) return false;
    pl->smem = (size_t)pl->stages * stage + 16 * pl->stages + 16 + 128;
    // about one CTA per SM over all (kv head, sequence) pairs; chunks of whole tiles
    size_t target = (size_t)num_sms / ((size_t)Hkv * batch);
    if (target < 1) target = 1;
    if (target > AM_MAX_SPLITS) target = AM_MAX_SPLITS;
    size_t chunk = (ctx_len + target - 1) / target;
    chunk = (chunk + 15) / 16 * 16;
    const size_t splits = (ctx_len + chunk - 1) / chunk;
    if (splits > AM_MAX_SPLITS) return false;
    pl->chunk = (int)chunk;
    pl->splits = (int)splits;
    return true;
}

template <int HD>
int launch_mma_hd(sulimo_ctx* ctx, const AttnMmaArgs& args, const MmaPlan& pl, int batch,
                  const CUtensorMap& tk, const CUtensorMap& tv) {
    static DeviceBits attr_done;
    if (!attr_done.test(ctx->device)) {
        int st = check_cuda(cudaFuncSetAttribute(attn_decode_mma_kernel<HD>,
                                                 cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                 (int)AM_SMEM_MAX + 1024),
                            "attn mma smem attribute");
        if (st) return st;
        attr_done.set(ctx->device);
    }
    cudaError_t e =
        launch_pdl(attn_decode_mma_kernel<HD>, dim3((unsigned)pl.splits, (unsigned)args.Hkv,
                                                    (unsigned)batch),
                   dim3(AM_THREADS), pl.smem, ctx->stream, args, tk, tv);
    ctx->launches++;
    if (e != cudaSuccess || pl.splits == 1) return check_cuda(e, "attn_decode_mma launch");
    constexpr int NB = HD / 32;
    e = launch_pdl(attn_decode_merge_kernel<HD>,
                   dim3((unsigned)((args.H * NB + 3) / 4), (unsigned)batch), dim3(128), 0,
                   ctx->stream, args, pl.splits);
    ctx->launches++;
    return check_cuda(e, "attn_decode_merge launch");
}

}  // namespace

size_t attn_decode_mma_partial_bytes(size_t ctx_len, size_t capacity, int H, int Hkv, int HD,
                                     int batch, int num_sms, size_t seq_stride, const void* k,
                                     const void* v) {
    MmaPlan pl;
    if (!mma_plan(ctx_len, capacity, H, Hkv, HD, batch, num_sms, seq_stride, k, v, &pl)) return 0;
    return (size_t)batch * H * pl.splits * (HD + 2) * sizeof(float);
}

int launch_attn_decode_mma(sulimo_ctx* ctx, const float* q, const void* k_ring,
                           const void* v_ring, size_t seq_stride, size_t capacity,
                           size_t context_len, int head_count, int head_count_kv, int head_dim,
                           int batch, float softcap, float* out, float* partials,
                           size_t partial_bytes, const Q8Out& out_q8,
                           bool* used, size_t static_before) {
    *used = false;
    MmaPlan pl;
    if (!mma_plan(context_len, capacity, head_count, head_count_kv, head_dim, batch, ctx->num_sms,
                  seq_stride, k_ring, v_ring, &pl))
        return SULIMO_OK;
    const size_t need = (size_t)batch * head_count * pl.splits * (head_dim + 2) * sizeof(float);
    if (pl.splits > 1 && need > partial_bytes) return SULIMO_OK;
    const size_t bpp = (size_t)head_count_kv * (head_dim / 32) * 34;
    const size_t stride = batch > 1 ? seq_stride : bpp * capacity;
    CUtensorMap tk, tv;
    memset(&tk, 0, sizeof(tk));
    memset(&tv, 0, sizeof(tv));
    {
        const uint64_t dims[3] = {(uint64_t)bpp, (uint64_t)capacity, (uint64_t)batch};
        const uint64_t strides[2] = {(uint64_t)bpp, (uint64_t)stride};
        const uint32_t box[3] = {(uint32_t)pl.boxw, (uint32_t)AM_SP, 1};
        int st = encode_tensor_map(&tk, CU_TENSOR_MAP_DATA_TYPE_UINT8, k_ring, 3, dims, strides,
                                   box, CU_TENSOR_MAP_SWIZZLE_NONE);
        if (!st)
            st = encode_tensor_map(&tv, CU_TENSOR_MAP_DATA_TYPE_UINT8, v_ring, 3, dims, strides,
                                   box, CU_TENSOR_MAP_SWIZZLE_NONE);
        if (st) return st;
    }
    AttnMmaArgs args;
    args.q = q;
    args.ctx_len = context_len;
    args.static_before = static_before;
    args.H = head_count;
    args.Hkv = head_count_kv;
    args.G = head_count / head_count_kv;
    args.chunk = pl.chunk;
    args.stages = pl.stages;
    args.boxw = pl.boxw;
    args.sm_scale = 1.0f / sqrtf((float)head_dim);
    args.softcap = softcap;
    args.out = out;
    args.q8 = out_q8;
    args.part = partials;
    args.err = ctx->d_error;
    *used = true;
    return head_dim == 64 ? launch_mma_hd<64>(ctx, args, pl, batch, tk, tv)
                          : launch_mma_hd<128>(ctx, args, pl, batch, tk, tv);
}

}  // namespace sulimo
