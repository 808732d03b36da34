// attn_prefill_tc.cu — causal GQA prefill attention over the Q8_0 KV ring on the tcgen05 tensor
// cores: the reference's causal_gqa_attention_prefill (kernels/prefill.cl:120-237), enqueued by
// enqueue_attention_prefill from execute_prefill_ubatch (crates/sulimo-ocl/src/prefill.rs:337-566).
//
// Token t of the ubatch sits at position start_pos + t and attends to positions
// 0 .. start_pos + t (ring slot = position: start_pos + n <= capacity), query head h to kv
// head h / (H / Hkv).
//
// One CTA per (128 query tokens, query head), flash-attention form with the accumulators in TMEM:
//   warp 9, one thread (producer): per chunk of 64 keys, one TMA tensor copy each of the K and
//     V ring rows of the kv head (a box of 64 slots starting at the 16-byte boundary at or below
//     the head's first byte), two chunks in flight;
//   warps 4-7 (converters): the CTA's queries once, as f16, into a 128-byte-swizzled K-major
//     tile; then per chunk the raw Q8_0 rows dequantized to f16(d * q) — K as [key][dim], V
//     transposed as [dim][key], both swizzled K-major B tiles (keys past the CTA's range: 0);
//   warp 8, one thread (MMA): S = Q K^T (tcgen05.mma kind::f16, A and B from shared memory,
//     M = 128, N = 64, fp32 in TMEM, two S buffers so S of the next chunk overlaps the softmax
//     of this one), then O += P V (A = P from TMEM, B = V^T from shared memory, N = hd, O in
//     TMEM for the whole key range);
//   warps 0-3 (softmax, thread = query row = TMEM lane): tcgen05.ld of the row's 64 scores,
//     scale by 1/sqrt(hd), causal mask, online softmax in fp32 with a lazily raised running
//     maximum (O and l are rescaled only when the row maximum grows by more than 8 in log2
//     units, so P <= 256 stays well inside f16), P as f16 into TMEM with tcgen05.st; at the end
//     O / l as f16 to the output row.
// The reference keeps q, the dequantized K/V and the accumulated output in f16 (prefill.cl
// works on half); here K and V enter the tensor cores as f16(d * q) (one rounding), P as f16,
// and every sum is fp32.  Every mbarrier wait is bounded by %globaltimer (device error, abort,
// TMEM freed).  No multicast.
#include <string.h>

#include <algorithm>

#include "sulimo_common.cuh"
#include "sulimo_internal.h"
#include "tc_sm100.cuh"

namespace sulimo {
namespace {

constexpr int AT_TQ = 128;       // query tokens per CTA = MMA M = TMEM lanes
constexpr int AT_CK = 64;        // keys per chunk = S's N
constexpr int AT_THREADS = 320;  // softmax 0-3, converters 4-7, MMA 8, producer 9
constexpr uint32_t AT_TMEM_COLS = 512;
constexpr uint32_t AT_S_COL = 0;     // S buffers: [0, 64), [64, 128)
constexpr uint32_t AT_P_COL = 128;   // P buffers: [128, 160), [160, 192) (f16 pairs)
constexpr uint32_t AT_O_COL = 256;   // O: [256, 256 + hd)
constexpr float AT_LOG2E = 1.4426950408889634f;
constexpr float AT_RESCALE = 8.0f;   // log2 of the largest P before O is rescaled
constexpr uint32_t AT_BOXW_MAX = 160;  // bytes of a staged ring row (hd 128: 136 + lead-in)

template <int HD>
struct AtGeom {
    static constexpr int HB = HD / 32 * 34;                 // ring bytes of one kv head
    static constexpr uint32_t Q_BYTES = AT_TQ * HD * 2;     // Q tile, f16
    static constexpr uint32_t K_BYTES = AT_CK * HD * 2;     // K tile [64 keys][hd]
    static constexpr uint32_t V_BYTES = HD * AT_CK * 2;     // V^T tile [hd][64 keys]
    static constexpr uint32_t RAW_BYTES = AT_CK * AT_BOXW_MAX;  // one tensor's staged rows
    // layout: Q | K0 | K1 | V0 | V1 | raw K0, V0, K1, V1 | barriers
    static constexpr uint32_t OFF_K = Q_BYTES;
    static constexpr uint32_t OFF_V = OFF_K + 2 * K_BYTES;
    static constexpr uint32_t OFF_RAW = OFF_V + 2 * V_BYTES;
    static constexpr uint32_t OFF_BAR = OFF_RAW + 4 * RAW_BYTES;
    static constexpr uint32_t SMEM = OFF_BAR + 256 + 1024;  // + barriers + alignment slack
};
static_assert(AtGeom<128>::SMEM <= 232448, "prefill attention smem (hd 128)");

// Byte offset of 16-byte chunk `kc` (8 f16 along K) of row `row` in a K-major tile of `rows`
// rows with the 128-byte swizzle: atoms of 64 K elements, 8-row groups 1024 bytes apart, the
// chunk index XORed with the row's position in its group (the layout TMA writes and the
// tcgen05 shared-memory descriptor reads).
__device__ __forceinline__ uint32_t sw128_off(int row, int kc, int rows) {
    return (uint32_t)((kc >> 3) * rows * 128 + (row >> 3) * 1024 + (row & 7) * 128 +
                      (((kc & 7) ^ (row & 7)) << 4));
}

__device__ __forceinline__ uint32_t h2(float a, float b) {
    __half2 h = __floats2half2_rn(a, b);
    return *reinterpret_cast<uint32_t*>(&h);
}

// SS-form MMA: A and B from shared-memory descriptors.
__device__ __forceinline__ void mma_ss(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                       uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
}

// TS-form MMA: A from TMEM, B from a shared-memory descriptor.
__device__ __forceinline__ void mma_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc,
                                       uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
        "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
}

__device__ __forceinline__ void commit_to(uint64_t* bar) {
    asm volatile(
        "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
            smem_u32(bar))
        : "memory");
}

struct AtArgs {
    const float* q;        // [n][H][hd] fp32 (after RoPE)
    __half* out;           // [n][H][hd] f16
    size_t start_pos;
    int n, H, Hkv;
    int boxw;              // bytes of a staged ring row (16-byte multiple)
    float scale_log2;      // log2(e) / sqrt(hd)
    int* err;
};

template <int HD>
__global__ void __launch_bounds__(AT_THREADS, 1)
    attn_prefill_tc_kernel(const __grid_constant__ AtArgs a,
                           const __grid_constant__ CUtensorMap tmap_k,
                           const __grid_constant__ CUtensorMap tmap_v) {
    using G = AtGeom<HD>;
    constexpr int NB = HD / 32;
    constexpr unsigned FULL = 0xffffffffu;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
    uint8_t* sQ = smem;
    uint8_t* sK = smem + G::OFF_K;
    uint8_t* sV = smem + G::OFF_V;
    uint8_t* sRaw = smem + G::OFF_RAW;  // stage s: K at 2s, V at 2s + 1 (RAW_BYTES each)
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + G::OFF_BAR);
    uint64_t* q_full = bars;        // converters: the query tile is in place
    uint64_t* raw_full = bars + 1;  // [2] producer: the chunk's ring rows landed
    uint64_t* raw_free = bars + 3;  // [2] converters: done reading the chunk's ring rows
    uint64_t* kv_full = bars + 5;   // [2] converters: the chunk's K and V tiles in place
    uint64_t* kv_free = bars + 7;   // [2] MMA: the chunk's P V done, its tiles may be refilled
    uint64_t* s_full = bars + 9;    // [2] MMA: S of the chunk in TMEM
    uint64_t* p_full = bars + 11;   // [2] softmax: P of the chunk in TMEM, O rescaled
    uint64_t* pv_done = bars + 13;  // MMA: P V of the chunk done (one phase per chunk)
    uint64_t* drained = bars + 14;  // MMA: everything it issued has completed
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 15);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int t0 = blockIdx.x * AT_TQ, h = blockIdx.y;
    const int kvh = h / (a.H / a.Hkv);
    const long last_tok = min((long)a.n - 1, (long)t0 + AT_TQ - 1);
    const long key_end = (long)a.start_pos + last_tok + 1;  // keys [0, key_end) for this CTA
    const int nch = (int)((key_end + AT_CK - 1) / AT_CK);
    const int x0 = (kvh * G::HB) & ~15;  // TMA x coordinate: 16-byte aligned
    const int lead = kvh * G::HB - x0;   // the head's first byte inside a staged row

    if (threadIdx.x == 0) {
        mbar_init(q_full, 4);
        for (int s = 0; s < 2; s++) {
            mbar_init(&raw_full[s], 1);
            mbar_init(&raw_free[s], 4);
            mbar_init(&kv_full[s], 4);
            mbar_init(&kv_free[s], 1);
            mbar_init(&s_full[s], 1);
            mbar_init(&p_full[s], 4);
        }
        mbar_init(pv_done, 1);
        mbar_init(drained, 1);
        *abort_flag = 0;
        fence_barrier_init();
        prefetch_tensormap(&tmap_k);
        prefetch_tensormap(&tmap_v);
    }
    if (warp == 8) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                         smem_u32(tmem_slot)),
                     "r"(AT_TMEM_COLS)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    pdl_launch_dependents();
    pdl_wait_prerequisites();  // q and the ring slots of this ubatch come from the previous kernels
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    if (warp == 9) {
        // ------------------------------ producer ------------------------------
        if (lane == 0) {
            const uint32_t bytes = 2u * AT_CK * (uint32_t)a.boxw;
            for (int c = 0; c < nch; c++) {
                const int s = c & 1;
                if (c >= 2 &&
                    !mbar_wait_bounded(&raw_free[s], ((c >> 1) - 1) & 1, a.err, abort_flag))
                    break;
                mbar_arrive_expect_tx(&raw_full[s], bytes);
                tma_load_2d(sRaw + (2 * s) * G::RAW_BYTES, &tmap_k, x0, c * AT_CK, &raw_full[s]);
                tma_load_2d(sRaw + (2 * s + 1) * G::RAW_BYTES, &tmap_v, x0, c * AT_CK,
                            &raw_full[s]);
            }
        }
    } else if (warp >= 4 && warp < 8) {
        // ------------------------------ converters ------------------------------
        const int ct = threadIdx.x - 128;
        // the queries: batches of QB items per thread, all of a batch's loads issued before any
        // is converted (one L2 round trip per batch, not per item)
        constexpr int QITEMS = AT_TQ * (HD / 8) / 128, QB = 8;
        for (int i0 = 0; i0 < QITEMS; i0 += QB) {
            float4 xv[QB][2];
#pragma unroll
            for (int i = 0; i < QB; i++) {
                const int it = ct + (i0 + i) * 128;
                const int row = it / (HD / 8), kc = it % (HD / 8);
                const int t = t0 + row;
                if (t < a.n) {
                    const float4* src = reinterpret_cast<const float4*>(
                        a.q + ((size_t)t * a.H + h) * HD + kc * 8);
                    xv[i][0] = __ldg(src);
                    xv[i][1] = __ldg(src + 1);
                } else {
                    xv[i][0] = xv[i][1] = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
                }
            }
#pragma unroll
            for (int i = 0; i < QB; i++) {
                const int it = ct + (i0 + i) * 128;
                const int row = it / (HD / 8), kc = it % (HD / 8);
                const float4 x0f = xv[i][0], x1f = xv[i][1];
                *reinterpret_cast<uint4*>(sQ + sw128_off(row, kc, AT_TQ)) =
                    make_uint4(h2(x0f.x, x0f.y), h2(x0f.z, x0f.w), h2(x1f.x, x1f.y),
                               h2(x1f.z, x1f.w));
            }
        }
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) mbar_arrive(q_full);
        for (int c = 0; c < nch; c++) {
            const int s = c & 1;
            if (!__all_sync(FULL, mbar_wait_bounded(&raw_full[s], (c >> 1) & 1, a.err,
                                                    abort_flag)))
                break;
            if (c >= 2 && !__all_sync(FULL, mbar_wait_bounded(&kv_free[s], ((c >> 1) - 1) & 1,
                                                               a.err, abort_flag)))
                break;
            const long k0 = (long)c * AT_CK;
            const uint8_t* rk = sRaw + (2 * s) * G::RAW_BYTES + lead;
            const uint8_t* rv = sRaw + (2 * s + 1) * G::RAW_BYTES + lead;
            // K tile [key][dim]: f16(d * q), one (key, Q8_0 block) per item
            uint8_t* kt = sK + s * G::K_BYTES;
            for (int it = ct; it < AT_CK * NB; it += 128) {
                const int key = it / NB, b = it % NB;
                const bool live = k0 + key < key_end;
                const uint8_t* blk = rk + key * a.boxw + b * 34;
                const float d = live ? __half2float(*reinterpret_cast<const __half*>(blk)) : 0.0f;
#pragma unroll
                for (int c8 = 0; c8 < 4; c8++) {
                    uint32_t w[4];
#pragma unroll
                    for (int e = 0; e < 4; e++) {
                        const uint32_t pr =
                            live ? *reinterpret_cast<const uint16_t*>(blk + 2 + c8 * 8 + 2 * e) : 0u;
                        w[e] = h2(d * (float)(int8_t)(pr & 0xFFu), d * (float)(int8_t)(pr >> 8));
                    }
                    *reinterpret_cast<uint4*>(kt + sw128_off(key, b * 4 + c8, AT_CK)) =
                        make_uint4(w[0], w[1], w[2], w[3]);
                }
            }
            // V^T tile [dim][key]: one (dimension, 8 keys) per item
            uint8_t* vt = sV + s * G::V_BYTES;
            for (int it = ct; it < HD * (AT_CK / 8); it += 128) {
                const int dm = it % HD, o = it / HD;
                const int b = dm >> 5, e = dm & 31;
                uint32_t w[4];
#pragma unroll
                for (int i = 0; i < 4; i++) {
                    const int key = o * 8 + 2 * i;
                    const uint8_t* r0 = rv + key * a.boxw + b * 34;
                    const uint8_t* r1 = r0 + a.boxw;
                    const bool l0 = k0 + key < key_end, l1 = k0 + key + 1 < key_end;
                    const float d0 = l0 ? __half2float(*reinterpret_cast<const __half*>(r0)) : 0.0f;
                    const float d1 = l1 ? __half2float(*reinterpret_cast<const __half*>(r1)) : 0.0f;
                    const int c0 = l0 ? (int)(int8_t)r0[2 + e] : 0;
                    const int c1 = l1 ? (int)(int8_t)r1[2 + e] : 0;
                    w[i] = h2(d0 * (float)c0, d1 * (float)c1);
                }
                *reinterpret_cast<uint4*>(vt + sw128_off(dm, o, HD)) =
                    make_uint4(w[0], w[1], w[2], w[3]);
            }
            fence_proxy_async_smem();
            __syncwarp();
            if (lane == 0) {
                mbar_arrive(&kv_full[s]);
                mbar_arrive(&raw_free[s]);
            }
        }
    } else if (warp == 8) {
        // ------------------------------ MMA issuer ------------------------------
        if (lane == 0) {
            // kind::f16, D f32, A = B = f16 K-major; N >> 3 at bit 17, M >> 4 at bit 24
            const uint32_t idesc_s =
                (1u << 4) | ((uint32_t)(AT_CK >> 3) << 17) | ((uint32_t)(AT_TQ >> 4) << 24);
            const uint32_t idesc_o =
                (1u << 4) | ((uint32_t)(HD >> 3) << 17) | ((uint32_t)(AT_TQ >> 4) << 24);
            auto issue_s = [&](int c) -> bool {
                const int s = c & 1;
                if (!mbar_wait_bounded(&kv_full[s], (c >> 1) & 1, a.err, abort_flag)) return false;
                tc_fence_after();
                const uint32_t qa = smem_u32(sQ), kb = smem_u32(sK + s * G::K_BYTES);
#pragma unroll
                for (int kk = 0; kk < HD / 16; kk++) {
                    const uint64_t ad =
                        sw128_desc(qa + (kk >> 2) * AT_TQ * 128) + (uint64_t)((kk & 3) * 2);
                    const uint64_t bd =
                        sw128_desc(kb + (kk >> 2) * AT_CK * 128) + (uint64_t)((kk & 3) * 2);
                    mma_ss(tmem + AT_S_COL + (uint32_t)s * 64u, ad, bd, idesc_s, kk > 0 ? 1u : 0u);
                }
                commit_to(&s_full[s]);
                return true;
            };
            bool ok = mbar_wait_bounded(q_full, 0, a.err, abort_flag) && issue_s(0);
            for (int c = 0; ok && c < nch; c++) {
                const int s = c & 1;
                // S of the next chunk overlaps this chunk's softmax (its buffer was read by the
                // softmax of chunk c - 1, whose P this loop already waited for)
                if (c + 1 < nch && !issue_s(c + 1)) break;
                if (!mbar_wait_bounded(&p_full[s], (c >> 1) & 1, a.err, abort_flag)) break;
                tc_fence_after();
                const uint32_t vb = smem_u32(sV + s * G::V_BYTES);
#pragma unroll
                for (int kk = 0; kk < AT_CK / 16; kk++)
                    mma_ts(tmem + AT_O_COL, tmem + AT_P_COL + (uint32_t)s * 32u + (uint32_t)kk * 8u,
                           sw128_desc(vb) + (uint64_t)(kk * 2), idesc_o,
                           (c > 0 || kk > 0) ? 1u : 0u);
                commit_to(pv_done);
                commit_to(&kv_free[s]);
            }
            commit_to(drained);
            mbar_wait_bounded(drained, 0, a.err, nullptr);
        }
    } else {
        // ------------------------------ softmax (warps 0-3) ------------------------------
        const int row = warp * 32 + lane;  // TMEM lane
        const int t = t0 + row;
        const long pos = (long)a.start_pos + t;
        const uint32_t lane_base = ((uint32_t)(warp * 32)) << 16;
        float m_used = -INFINITY, l = 0.0f;
        bool ok = true;
        for (int c = 0; c < nch; c++) {
            const int s = c & 1;
            if (!__all_sync(FULL, mbar_wait_bounded(&s_full[s], (c >> 1) & 1, a.err, abort_flag))) {
                ok = false;
                break;
            }
            tc_fence_after();
            uint32_t v[2][32];
            tmem_ld32_issue(tmem + lane_base + AT_S_COL + (uint32_t)s * 64u, v[0]);
            tmem_ld32_issue(tmem + lane_base + AT_S_COL + (uint32_t)s * 64u + 32u, v[1]);
            tmem_ld_wait_carry(v[0]);
            tmem_ld_wait_carry(v[1]);
            const long k0 = (long)c * AT_CK;
            float mx = -INFINITY;
#pragma unroll
            for (int j = 0; j < AT_CK; j++) {
                const float x = (k0 + j <= pos) ? __uint_as_float(v[j >> 5][j & 31]) * a.scale_log2
                                                : -INFINITY;
                v[j >> 5][j & 31] = __float_as_uint(x);
                mx = fmaxf(mx, x);
            }
            // O and this chunk's P buffer are free once P V of chunk c - 1 has completed
            if (c > 0 && !__all_sync(FULL, mbar_wait_bounded(pv_done, (uint32_t)(c - 1) & 1u,
                                                             a.err, abort_flag))) {
                ok = false;
                break;
            }
            tc_fence_after();
            const float m_new = fmaxf(m_used, mx);
            if (c == 0) {
                m_used = m_new;  // key 0 is visible to every row: finite
            } else if (__any_sync(FULL, m_new > m_used + AT_RESCALE)) {
                const bool mine = m_new > m_used + AT_RESCALE;
                const float alpha = mine ? exp2f(m_used - m_new) : 1.0f;
                if (mine) {
                    l *= alpha;
                    m_used = m_new;
                }
#pragma unroll
                for (int c0 = 0; c0 < HD; c0 += 32) {
                    uint32_t o[32];
                    tmem_ld32(tmem + lane_base + AT_O_COL + (uint32_t)c0, o);
#pragma unroll
                    for (int jj = 0; jj < 32; jj++)
                        o[jj] = __float_as_uint(__uint_as_float(o[jj]) * alpha);
                    tmem_st32(tmem + lane_base + AT_O_COL + (uint32_t)c0, o);
                }
            }
            uint32_t pw[32];
            float psum = 0.0f;
#pragma unroll
            for (int j = 0; j < AT_CK; j += 2) {
                const float p0 = exp2f(__uint_as_float(v[j >> 5][j & 31]) - m_used);
                const float p1 = exp2f(__uint_as_float(v[(j + 1) >> 5][(j + 1) & 31]) - m_used);
                psum += p0 + p1;
                pw[j >> 1] = h2(p0, p1);
            }
            l += psum;
            tmem_st32(tmem + lane_base + AT_P_COL + (uint32_t)s * 32u, pw);
            tmem_st_wait();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&p_full[s]);
        }
        if (ok && __all_sync(FULL, mbar_wait_bounded(pv_done, (uint32_t)(nch - 1) & 1u, a.err,
                                                    abort_flag))) {
            tc_fence_after();
            const float inv = l > 0.0f ? 1.0f / l : 0.0f;
#pragma unroll
            for (int c0 = 0; c0 < HD; c0 += 32) {
                uint32_t o[32];
                tmem_ld32(tmem + lane_base + AT_O_COL + (uint32_t)c0, o);
                if (t < a.n) {
                    __half* dst = a.out + ((size_t)t * a.H + h) * HD + c0;
#pragma unroll
                    for (int q4 = 0; q4 < 4; q4++) {
                        const float* f = reinterpret_cast<const float*>(o + q4 * 8);
                        *reinterpret_cast<uint4*>(dst + q4 * 8) =
                            make_uint4(h2(f[0] * inv, f[1] * inv), h2(f[2] * inv, f[3] * inv),
                                       h2(f[4] * inv, f[5] * inv), h2(f[6] * inv, f[7] * inv));
                    }
                }
            }
        }
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 8) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem),
                     "r"(AT_TMEM_COLS)
                     : "memory");
    }
}

template <int HD>
int launch_hd_tc(sulimo_ctx* ctx, const AtArgs& a, const CUtensorMap& tk, const CUtensorMap& tv) {
    static DeviceBits attr;
    if (!attr.test(ctx->device)) {
        int st = check_cuda(cudaFuncSetAttribute(attn_prefill_tc_kernel<HD>,
                                                 cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                 (int)AtGeom<HD>::SMEM),
                            "prefill attention smem attribute");
        if (st) return st;
        attr.set(ctx->device);
    }
    const dim3 grid((unsigned)((a.n + AT_TQ - 1) / AT_TQ), (unsigned)a.H);
    const cudaError_t e = launch_pdl(attn_prefill_tc_kernel<HD>, grid, dim3(AT_THREADS),
                                     (size_t)AtGeom<HD>::SMEM, ctx->stream, a, tk, tv);
    ctx->launches++;
    return check_cuda(e, "attn_prefill_tc launch");
}

}  // namespace

bool attn_prefill_tc_applies(const float* q, const void* k_ring, const void* v_ring,
                             size_t capacity, int Hkv, int hd, const void* out) {
    if (hd != 64 && hd != 128) return false;
    const size_t hb = (size_t)hd / 32 * 34, bpp = (size_t)Hkv * hb;
    size_t lead = 0;
    for (int h = 0; h < Hkv && h < 16; h++) lead = std::max(lead, (h * hb) % 16);
    const size_t boxw = (lead + hb + 15) / 16 * 16;
    const uintptr_t al = reinterpret_cast<uintptr_t>(q) | reinterpret_cast<uintptr_t>(out) |
                         reinterpret_cast<uintptr_t>(k_ring) | reinterpret_cast<uintptr_t>(v_ring);
    return (al & 15) == 0 && bpp % 16 == 0 && bpp >= boxw && boxw <= AT_BOXW_MAX &&
           capacity <= 0x7fffffff;
}

int launch_attn_prefill_tc(sulimo_ctx* ctx, const float* q, const void* k_ring,
                           const void* v_ring, size_t start_pos, size_t capacity, int n_tok,
                           int H, int Hkv, int hd, void* out) {
    const size_t hb = (size_t)hd / 32 * 34, bpp = (size_t)Hkv * hb;
    size_t lead = 0;
    for (int h = 0; h < Hkv && h < 16; h++) lead = std::max(lead, (h * hb) % 16);
    AtArgs a;
    a.q = q;
    a.out = reinterpret_cast<__half*>(out);
    a.start_pos = start_pos;
    a.n = n_tok;
    a.H = H;
    a.Hkv = Hkv;
    a.boxw = (int)((lead + hb + 15) / 16 * 16);
    a.scale_log2 = AT_LOG2E / sqrtf((float)hd);
    a.err = ctx->d_error;
    CUtensorMap tk, tv;
    memset(&tk, 0, sizeof(tk));
    memset(&tv, 0, sizeof(tv));
    int st = encode_2d(&tk, CU_TENSOR_MAP_DATA_TYPE_UINT8, k_ring, (uint64_t)bpp,
                       (uint64_t)capacity, (uint64_t)bpp, (uint32_t)a.boxw, (uint32_t)AT_CK,
                       CU_TENSOR_MAP_SWIZZLE_NONE);
    if (!st)
        st = encode_2d(&tv, CU_TENSOR_MAP_DATA_TYPE_UINT8, v_ring, (uint64_t)bpp,
                       (uint64_t)capacity, (uint64_t)bpp, (uint32_t)a.boxw, (uint32_t)AT_CK,
                       CU_TENSOR_MAP_SWIZZLE_NONE);
    if (st) return st;
    return hd == 64 ? launch_hd_tc<64>(ctx, a, tk, tv) : launch_hd_tc<128>(ctx, a, tk, tv);
}

}  // namespace sulimo
