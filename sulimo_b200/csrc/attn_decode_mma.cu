// attn_decode_mma.cu — decode attention over the Q8_0 KV ring on the tensor cores.
//
// Restates causal_gqa_decode_scalar_ext (crates/sulimo-cpu/src/scalar.rs:287-359) over the ring
// addressing of KvCache::key_ptr / value_ptr (crates/sulimo-core/src/kv_cache.rs:114-128):
//   score[h][p] = (q_h . dequant(K[p % cap][kv(h)])) / sqrt(hd)   [tanh soft-cap if set]
//   out_h = sum_p softmax_p(score[h]) * dequant(V[p % cap][kv(h)])
// in one kernel, split over the context ("flash-decoding") and merged on the device.
//
// Grid: (splits, sequences) in thread-block clusters of `cl` CTAs along the splits.  A CTA
// covers `chunk` consecutive positions of one sequence for ALL kv heads: every position is one
// ring slot (Hkv * hd/32 Q8_0 blocks), so each slot arrives with one bulk copy per tensor.
//   producer (warp 8): bulk copies of K and V slots into padded shared-memory rows (the row
//     stride is chosen so that eight rows start in eight different bank quads), `stages`-deep
//     ring of stages of `sp` positions, full / empty mbarriers;
//   consumers (warps 0-7): warp w works on kv head w % Hkv and on every (8/Hkv)-th 16-position
//     tile of a stage.  Per tile, with mma.sync.m16n8k16 (f16 in, fp32 accumulate):
//       S^T[head][pos] = Q . K^T: the A operand holds the query rows split in two f16 parts,
//         hi = f16(q) in rows 0-7 and lo = f16(q - hi) in rows 8-15 (so q enters at ~22 bits);
//         B = K's int8 codes, exact in f16; each 32-dimension Q8_0 block is two k-steps into a
//         fresh accumulator, then (hi + lo) * d_K[pos] is added in fp32;
//       online softmax per head in fp32 (running max / sum, exp2);
//       O[head][dim] += P' . V: per 32-dimension block b the A operand is P * d_V[pos][b], again
//         hi / lo f16 in rows 0-7 / 8-15, B = V's int8 codes; O accumulates in fp32.
//   merge: the warps of a kv head through shared memory, the CTAs of a cluster through
//     distributed shared memory (CTA rank r merges heads r, r + cl, ...), then, when a sequence
//     has several clusters, each cluster writes its partial (m, l, o) and the last CTA of each
//     rank (per-sequence counters, zero at rest) merges the clusters' partials and writes the
//     output (and, for the decode step, its Q8_0 quantization).
// Numerics: products are exact, sums are fp32 in a different order than the reference's
// sequential loop, and q / P' carry ~22 significant bits: the result matches the reference
// within fp32-level rounding (the parity tests bound the relative L2 error at 2e-3).
#include "sulimo_common.cuh"
#include "sulimo_internal.h"

namespace sulimo {
namespace {

constexpr int AM_CONSUMERS = 8;                    // consumer warps
constexpr int AM_THREADS = (AM_CONSUMERS + 1) * 32;  // + one producer warp
constexpr size_t AM_SMEM_MAX = 220 * 1024;
constexpr size_t AM_STAGE_TARGET = 72 * 1024;      // K + V bytes per stage
constexpr float AM_LOG2E = 1.4426950408889634f;

struct AttnMmaArgs {
    const float* q;         // [batch][H][HD] fp32
    const uint8_t* kring;   // ring of sequence s at kring + s * seq_stride
    const uint8_t* vring;
    size_t seq_stride;
    size_t capacity;        // ring slots
    size_t ctx_len;         // positions 0 .. ctx_len-1, slot p % capacity
    int H, Hkv, G, wph;     // query heads, kv heads, H / Hkv, consumer warps per kv head
    int chunk;              // positions per CTA
    int sp;                 // positions per stage
    int stages;
    int cl;                 // CTAs per cluster
    uint32_t bpp;           // ring bytes per slot (all kv heads)
    uint32_t rs;            // shared-memory bytes per staged slot
    float sm_scale;         // 1 / sqrt(hd)
    float softcap;          // <= 0: none
    float* out;             // [batch][H][HD] or null
    uint8_t* q8;            // [batch][H * HD / 32] Q8_0 blocks or null
    float* part;            // [batch][clusters][H][HD + 2]
    unsigned* counters;     // [batch][cl]
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

// bytes b0 (of x) and b0 (of y) -> f16 pair {x, y}
__device__ __forceinline__ uint32_t s8two_to_h2(uint32_t x, uint32_t y) {
    return s8pair_to_h2(prmt(x, y, 0x7740u));
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

__device__ __forceinline__ void cluster_sync_all() {
    asm volatile("barrier.cluster.arrive.release.aligned;\n\t"
                 "barrier.cluster.wait.acquire.aligned;" ::: "memory");
}

__device__ __forceinline__ uint32_t cluster_rank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}

// shared-memory address of `p` in CTA `rank` of this cluster
__device__ __forceinline__ uint32_t map_rank(const void* p, uint32_t rank) {
    uint32_t r;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(smem_u32(p)), "r"(rank));
    return r;
}

__device__ __forceinline__ float ld_cluster(uint32_t addr) {
    float v;
    asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(v) : "r"(addr) : "memory");
    return v;
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
    attn_decode_mma_kernel(const __grid_constant__ AttnMmaArgs a) {
    constexpr int NB = HD / 32, HB = NB * 34, KS = HD / 16, NT = HD / 8;
    extern __shared__ __align__(16) uint8_t smem_raw[];
    uint8_t* smem = smem_raw + ((128u - (smem_u32(smem_raw) & 127u)) & 127u);
    const uint32_t stage_bytes = 2u * (uint32_t)a.sp * a.rs;
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + (size_t)a.stages * stage_bytes);
    uint64_t* empty = full + a.stages;
    int* last_flag = reinterpret_cast<int*>(empty + a.stages);

    const int split = blockIdx.x, seq = blockIdx.y;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int g = lane >> 2, tig = lane & 3;
    const size_t p0 = (size_t)split * a.chunk;
    const int np = p0 < a.ctx_len ? (int)min((size_t)a.chunk, a.ctx_len - p0) : 0;
    const int nstage = (np + a.sp - 1) / a.sp;

    if (tid == 0) {
        for (int s = 0; s < a.stages; s++) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], AM_CONSUMERS);
        }
        fence_barrier_init();
    }
    __syncthreads();
    // q and the ring's newest slot are written by the previous kernel of the step
    pdl_launch_dependents();
    pdl_wait_prerequisites();

    if (warp == AM_CONSUMERS) {
        // ------------------------------ producer ------------------------------
        const uint8_t* kseq = a.kring + (size_t)seq * a.seq_stride;
        const uint8_t* vseq = a.vring + (size_t)seq * a.seq_stride;
        for (int st = 0; st < nstage; st++) {
            const int s = st % a.stages;
            if (st >= a.stages &&
                !mbar_wait_bounded(&empty[s], (uint32_t)((st / a.stages) - 1) & 1u, a.err,
                                   nullptr))
                break;
            const int q0 = st * a.sp;
            const int n = min(a.sp, np - q0);
            uint8_t* dk = smem + (size_t)s * stage_bytes;
            uint8_t* dv = dk + (size_t)a.sp * a.rs;
            if (lane == 0) mbar_arrive_expect_tx(&full[s], 2u * (uint32_t)n * a.bpp);
            __syncwarp();
            if (a.rs == a.bpp) {
                // contiguous rows: at most two runs per tensor (the ring may wrap inside)
                if (lane == 0) {
                    const size_t s0 = (p0 + q0) % a.capacity;
                    const int n1 = (int)min((size_t)n, a.capacity - s0);
                    bulk_load(dk, kseq + s0 * a.bpp, (uint32_t)n1 * a.bpp, &full[s]);
                    bulk_load(dv, vseq + s0 * a.bpp, (uint32_t)n1 * a.bpp, &full[s]);
                    if (n1 < n) {
                        bulk_load(dk + (size_t)n1 * a.rs, kseq, (uint32_t)(n - n1) * a.bpp,
                                  &full[s]);
                        bulk_load(dv + (size_t)n1 * a.rs, vseq, (uint32_t)(n - n1) * a.bpp,
                                  &full[s]);
                    }
                }
            } else {
                for (int i = lane; i < n; i += 32) {
                    const size_t slot = (p0 + q0 + i) % a.capacity;
                    bulk_load(dk + (size_t)i * a.rs, kseq + slot * a.bpp, a.bpp, &full[s]);
                    bulk_load(dv + (size_t)i * a.rs, vseq + slot * a.bpp, a.bpp, &full[s]);
                }
            }
        }
    }

    // ------------------------------ consumers ------------------------------
    float oc[NT][4];
    float m_run = -INFINITY, l_run = 0.0f;
#pragma unroll
    for (int n = 0; n < NT; n++) oc[n][0] = oc[n][1] = oc[n][2] = oc[n][3] = 0.0f;
    const int kvh = warp % a.Hkv, wj = warp / a.Hkv;
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
                    const float x0 = hv ? qh[d] : 0.0f, x1 = hv ? qh[d + 1] : 0.0f;
                    const __half2 hi = __floats2half2_rn(x0, x1);
                    const float2 hf2 = __half22float2(hi);
                    const __half2 lo = __floats2half2_rn(x0 - hf2.x, x1 - hf2.y);
                    qa[ks][2 * hf] = h2_bits(hi);
                    qa[ks][2 * hf + 1] = h2_bits(lo);
                }
        }
        const float score_scale = a.sm_scale;
        const bool capped = a.softcap > 0.0f;
        for (int st = 0; st < nstage; st++) {
            const int s = st % a.stages;
            // warp-uniform: the tile loop below runs warp-wide shuffles and MMAs
            const bool landed = __all_sync(
                0xffffffffu,
                mbar_wait_bounded(&full[s], (uint32_t)(st / a.stages) & 1u, a.err, nullptr));
            const int q0 = st * a.sp;
            const uint8_t* kst = smem + (size_t)s * stage_bytes + kvh * HB;
            const uint8_t* vst = kst + (size_t)a.sp * a.rs;
            for (int t = wj * 16; landed && t < a.sp && q0 + t < np; t += a.wph * 16) {
                const int valid = np - (q0 + t);  // rows of this tile that hold positions
                const uint8_t* kt = kst + (size_t)t * a.rs;
                const uint8_t* vt = vst + (size_t)t * a.rs;
                // ---- scores: two 8-position n-tiles ----
                float x[4];
#pragma unroll
                for (int nt = 0; nt < 2; nt++) {
                    const uint8_t* krow = kt + (size_t)(nt * 8 + g) * a.rs;
                    const uint8_t* srow = kt + (size_t)(nt * 8 + 2 * tig) * a.rs;
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
                        s1 = __fmaf_rn(c[1] + c[3], lds_f16(srow + a.rs + b * 34), s1);
                    }
#pragma unroll
                    for (int j = 0; j < 2; j++) {
                        float v = (j ? s1 : s0) * score_scale;
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
                const uint8_t* v0 = vt + (size_t)(2 * tig) * a.rs;  // rows 2tig, +1, +8, +9
#pragma unroll
                for (int b = 0; b < NB; b++) {
                    float pp[4];
#pragma unroll
                    for (int i = 0; i < 4; i++) {
                        const int row = (i >> 1) * 8 + (i & 1);
                        pp[i] = p[i] != 0.0f ? p[i] * lds_f16(v0 + (size_t)row * a.rs + b * 34)
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
#pragma unroll
                    for (int n4 = 0; n4 < 4; n4++) {
                        const uint8_t* col = v0 + b * 34 + 2 + n4 * 8 + g;
                        const uint32_t b0 = s8two_to_h2(col[0], col[a.rs]);
                        const uint32_t b1 = s8two_to_h2(col[(size_t)8 * a.rs], col[(size_t)9 * a.rs]);
                        mma_16816(oc[b * 4 + n4], A, b0, b1);
                    }
                }
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[s]);
        }
    }
    __syncthreads();  // every stage consumed: the stage memory becomes the merge area

    // ---- this warp's (m, l, o) per head -> wpart[warp][g][HD + 2] ----
    const int HD2 = HD + 2;
    float* wpart = reinterpret_cast<float*>(smem);
    float* cpart = wpart + (size_t)AM_CONSUMERS * a.G * HD2;  // [H][HD + 2]
    if (warp < AM_CONSUMERS) {
        float l_tot = l_run + __shfl_xor_sync(0xffffffffu, l_run, 1);
        l_tot += __shfl_xor_sync(0xffffffffu, l_tot, 2);
        if (g < a.G) {
            float* row = wpart + ((size_t)warp * a.G + g) * HD2;
#pragma unroll
            for (int n = 0; n < NT; n++) {
                row[n * 8 + 2 * tig] = oc[n][0] + oc[n][2];
                row[n * 8 + 2 * tig + 1] = oc[n][1] + oc[n][3];
            }
            if (tig == 0) {
                row[HD] = m_run;
                row[HD + 1] = l_tot;
            }
        }
    }
    __syncthreads();
    // ---- the warps of each kv head -> the CTA's partial per query head ----
    for (int it = tid; it < a.H * HD2; it += AM_THREADS) {
        const int h = it / HD2, d = it - h * HD2;
        const int kv = h / a.G, gg = h - kv * a.G;
        auto rd = [&](int i, int dd) {
            return wpart[((size_t)(kv + i * a.Hkv) * a.G + gg) * HD2 + dd];
        };
        float o, l, m;
        merge_rows<HD>(a.wph, d < HD ? d : HD, rd, &o, &l, &m);
        cpart[(size_t)h * HD2 + d] = d < HD ? o : (d == HD ? m : l);
    }
    cluster_sync_all();  // every CTA of the cluster has its partials in shared memory

    // ---- the cluster's CTAs -> heads r, r + cl, ... merged by CTA rank r ----
    const uint32_t rank = cluster_rank();
    const int nclusters = (int)gridDim.x / a.cl, cid = (int)blockIdx.x / a.cl;
    const bool direct = nclusters == 1;  // the cluster holds the whole sequence
    // items (owned head, d), d in [0, HDP): the output dimensions, then m and l; HDP is a
    // multiple of 32 so that every warp's 32 dimensions are one Q8_0 block of one head
    constexpr int HDP = HD + 32;
    const int owned = ((int)a.H - (int)rank + a.cl - 1) / a.cl;
    for (int it = tid; it < owned * HDP; it += AM_THREADS) {
        const int h = (int)rank + (it / HDP) * a.cl, d = it % HDP;
        if (d >= HD2) continue;  // whole warps: HDP - HD2 >= 30 idle lanes sit past HD2
        auto rd = [&](int i, int dd) {
            return ld_cluster(map_rank(cpart + (size_t)h * HD2 + dd, (uint32_t)i));
        };
        float o, l, m;
        merge_rows<HD>(a.cl, d < HD ? d : HD, rd, &o, &l, &m);
        if (direct) {
            if (d < HD) {
                const float val = l > 0.0f ? o / l : 0.0f;
                if (a.out) a.out[((size_t)seq * a.H + h) * HD + d] = val;
                if (a.q8)
                    quantize_block_warp(val, a.q8 + (((size_t)seq * a.H + h) * NB + d / 32) * 34,
                                        lane);
            }
        } else {
            float* dst = a.part + (((size_t)seq * nclusters + cid) * a.H + h) * HD2;
            dst[d] = d < HD ? o : (d == HD ? m : l);
        }
    }
    cluster_sync_all();  // no CTA leaves while a peer still reads its shared memory
    if (direct) return;

    // ---- the last CTA of each rank merges the clusters' partials of its heads ----
    __syncthreads();
    if (tid == 0) {
        __threadfence();
        unsigned* ctr = a.counters + (size_t)seq * a.cl + rank;
        const unsigned old = atomicAdd(ctr, 1u);
        *last_flag = old == (unsigned)(nclusters - 1);
        if (*last_flag) __threadfence();
    }
    __syncthreads();
    if (!*last_flag) return;
    for (int it = tid; it < owned * HDP; it += AM_THREADS) {
        const int h = (int)rank + (it / HDP) * a.cl, d = it % HDP;
        if (d >= HD) continue;
        const float* base = a.part + ((size_t)seq * nclusters * a.H + h) * HD2;
        auto rd = [&](int i, int dd) { return __ldcg(base + (size_t)i * a.H * HD2 + dd); };
        float o, l, m;
        merge_rows<HD>(nclusters, d, rd, &o, &l, &m);
        const float val = l > 0.0f ? o / l : 0.0f;
        if (a.out) a.out[((size_t)seq * a.H + h) * HD + d] = val;
        if (a.q8)
            quantize_block_warp(val, a.q8 + (((size_t)seq * a.H + h) * NB + d / 32) * 34, lane);
    }
    if (tid == 0) a.counters[(size_t)seq * a.cl + rank] = 0u;  // zero at rest for the next call
}

struct MmaPlan {
    int wph, sp, stages, cl, chunk, splits, nclusters;
    uint32_t rs;
    size_t smem;
};

// Geometry of the tensor-core form, or false when it does not apply (the caller falls back to
// the scalar kernels).
bool mma_plan(size_t ctx_len, size_t capacity, int H, int Hkv, int HD, int batch, int num_sms,
              size_t seq_stride, const void* k, const void* v, MmaPlan* pl) {
    if (HD != 64 && HD != 128) return false;
    if (Hkv < 1 || Hkv > AM_CONSUMERS || AM_CONSUMERS % Hkv != 0 || H % Hkv != 0) return false;
    const int G = H / Hkv;
    if (G < 1 || G > 8) return false;
    const size_t bpp = (size_t)Hkv * (HD / 32) * 34;
    if (bpp % 16 || ((uintptr_t)k % 16) || ((uintptr_t)v % 16)) return false;
    if (batch > 1 && seq_stride % 16) return false;
    if (ctx_len < 1 || capacity < 1 || batch < 1 || batch > 65535) return false;
    uint32_t rs = (uint32_t)bpp;
    while (((rs / 4) % 32) % 8 != 4) rs += 16;  // eight rows in eight different bank quads
    pl->rs = rs;
    pl->wph = AM_CONSUMERS / Hkv;
    int tpw = (int)(AM_STAGE_TARGET / (2u * 16u * pl->wph * rs));
    if (tpw < 1) tpw = 1;
    pl->sp = 16 * pl->wph * tpw;
    const size_t stage = 2u * (size_t)pl->sp * rs;
    pl->stages = (int)((AM_SMEM_MAX - 1024) / stage);
    if (pl->stages > 3) pl->stages = 3;
    if (pl->stages < 1) return false;
    // merge area (inside the stage memory): per-warp and per-CTA partials
    const size_t merge = ((size_t)AM_CONSUMERS * G + H) * (HD + 2) * 4;
    if (merge > (size_t)pl->stages * stage) return false;
    pl->smem = (size_t)pl->stages * stage + 2 * 8 * pl->stages + 16 + 128;
    // one CTA per SM over all sequences; chunks of whole 16-position tiles per warp
    const int unit = 16 * pl->wph;
    size_t target = (size_t)num_sms / batch;
    if (target < 1) target = 1;
    size_t chunk = (ctx_len + target - 1) / target;
    chunk = (chunk + unit - 1) / unit * unit;
    if (chunk < (size_t)unit) chunk = unit;
    if (chunk > 0x3fffffff) return false;
    const size_t splits = (ctx_len + chunk - 1) / chunk;
    int best = 1;
    size_t best_waste = (size_t)-1;
    for (int c = 8; c >= 1; c >>= 1) {  // the cluster size wasting the fewest idle CTAs
        const size_t padded = (splits + c - 1) / c * c;
        if (padded - splits < best_waste) {
            best_waste = padded - splits;
            best = c;
        }
    }
    pl->cl = best;
    pl->chunk = (int)chunk;
    const size_t padded = (splits + best - 1) / best * best;
    if (padded > 0x7fffffff) return false;
    pl->splits = (int)padded;
    pl->nclusters = pl->splits / pl->cl;
    return true;
}

template <int HD>
int launch_mma_hd(sulimo_ctx* ctx, const AttnMmaArgs& args, const MmaPlan& pl, int batch) {
    static DeviceBits attr_done;
    if (!attr_done.test(ctx->device)) {
        int st = check_cuda(cudaFuncSetAttribute(attn_decode_mma_kernel<HD>,
                                                 cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                 (int)AM_SMEM_MAX + 1024),
                            "attn mma smem attribute");
        if (st) return st;
        attr_done.set(ctx->device);
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)pl.splits, (unsigned)batch, 1);
    cfg.blockDim = dim3(AM_THREADS);
    cfg.dynamicSmemBytes = pl.smem;
    cfg.stream = ctx->stream;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    attr[1].id = cudaLaunchAttributeClusterDimension;
    attr[1].val.clusterDim.x = (unsigned)pl.cl;
    attr[1].val.clusterDim.y = 1;
    attr[1].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 2;
    const cudaError_t e = cudaLaunchKernelEx(&cfg, attn_decode_mma_kernel<HD>, args);
    ctx->launches++;
    return check_cuda(e, "attn_decode_mma launch");
}

}  // namespace

size_t attn_decode_mma_partial_bytes(size_t ctx_len, size_t capacity, int H, int Hkv, int HD,
                                     int batch, int num_sms, size_t seq_stride, const void* k,
                                     const void* v) {
    MmaPlan pl;
    if (!mma_plan(ctx_len, capacity, H, Hkv, HD, batch, num_sms, seq_stride, k, v, &pl)) return 0;
    return (size_t)batch * pl.nclusters * H * (HD + 2) * sizeof(float);
}

int launch_attn_decode_mma(sulimo_ctx* ctx, const float* q, const void* k_ring,
                           const void* v_ring, size_t seq_stride, size_t capacity,
                           size_t context_len, int head_count, int head_count_kv, int head_dim,
                           int batch, float softcap, float* out, float* partials,
                           size_t partial_bytes, unsigned* counters, uint8_t* out_q8,
                           bool* used) {
    *used = false;
    MmaPlan pl;
    if (!counters ||
        !mma_plan(context_len, capacity, head_count, head_count_kv, head_dim, batch, ctx->num_sms,
                  seq_stride, k_ring, v_ring, &pl))
        return SULIMO_OK;
    const size_t need = (size_t)batch * pl.nclusters * head_count * (head_dim + 2) * sizeof(float);
    if (need > partial_bytes) return SULIMO_OK;
    AttnMmaArgs args;
    args.q = q;
    args.kring = reinterpret_cast<const uint8_t*>(k_ring);
    args.vring = reinterpret_cast<const uint8_t*>(v_ring);
    args.seq_stride = batch > 1 ? seq_stride : 0;
    args.capacity = capacity;
    args.ctx_len = context_len;
    args.H = head_count;
    args.Hkv = head_count_kv;
    args.G = head_count / head_count_kv;
    args.wph = pl.wph;
    args.chunk = pl.chunk;
    args.sp = pl.sp;
    args.stages = pl.stages;
    args.cl = pl.cl;
    args.bpp = (uint32_t)((size_t)head_count_kv * (head_dim / 32) * 34);
    args.rs = pl.rs;
    args.sm_scale = 1.0f / sqrtf((float)head_dim);
    args.softcap = softcap;
    args.out = out;
    args.q8 = out_q8;
    args.part = partials;
    args.counters = counters;
    args.err = ctx->d_error;
    *used = true;
    return head_dim == 64 ? launch_mma_hd<64>(ctx, args, pl, batch)
                          : launch_mma_hd<128>(ctx, args, pl, batch);
}

}  // namespace sulimo
