// attn_prefill_tc.cu — causal GQA prefill attention over the Q8_0 KV ring on the tcgen05 tensor
// cores: the reference's causal_gqa_attention_prefill (kernels/prefill.cl:120-237), enqueued by
// enqueue_attention_prefill from execute_prefill_ubatch (crates/sulimo-ocl/src/prefill.rs:337-566).
//
// Token t of the ubatch sits at position start_pos + t and attends to positions
// 0 .. start_pos + t (ring slot = position: start_pos + n <= capacity), query head h to kv
// head h / (H / Hkv).
//
// One CTA per (128 query tokens, query head, key range), flash-attention form with the
// accumulators in TMEM (when the (tile, head) pairs are fewer than the SMs, a tile's key chunks
// are divided among several CTAs, which write O / l and the row's log2-sum-exp for
// attn_prefill_merge_kernel to combine):
//   warp 13, one thread (producer): per chunk of 64 keys, one TMA tensor copy each of the K and
//     V ring rows of the kv head (a box of 64 slots starting at the 16-byte boundary at or below
//     the head's first byte), two chunks in flight;
//   warps 8-11 (converters): per chunk one thread per (tensor, key): the key's staged ring row
//     read with 16-byte loads, each Q8_0 block dequantized to f16(d * q) by byte permutes and
//     exact half arithmetic, written as [key][dim] into a 128-byte-swizzled tile — K-major B for
//     S = Q K^T, MN-major B for O += P V (keys past the CTA's range: 0), three stages;
//   warp 12, one thread (MMA): S = Q K^T (tcgen05.mma kind::f16, A and B from shared memory,
//     M = 128, N = 64, fp32 in TMEM, two S buffers so S of the next chunk overlaps the softmax
//     of this one), then O += P V (A = P from TMEM, B = V from shared memory read MN-major,
//     N = hd, O in TMEM for the whole key range);
//   warps 0-7 (softmax): the CTA's queries once, as f16, into a 128-byte-swizzled K-major tile;
//     then thread = (query row = TMEM lane, half of the chunk): tcgen05.ld of the row's 32
//     scores, causal mask, the row maximum shared with the other half's warp through shared
//     memory, online softmax in fp32 with a lazily raised running maximum (O and l are rescaled
//     only when the row maximum grows by more than 8 in log2 units, so P <= 256 stays well
//     inside f16), P as f16 into TMEM with tcgen05.st; each half keeps its own row sum and
//     rescales its half of O; at the end O / l (the halves' sums added) staged in the free K/V
//     tiles and stored by TMA.
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
constexpr int AT_THREADS = 448;  // softmax 0-7, converters 8-11, MMA 12, producer 13
constexpr uint32_t AT_TMEM_COLS = 512;
constexpr uint32_t AT_S_COL = 0;     // S buffers: [0, 64), [64, 128)
constexpr uint32_t AT_P_COL = 128;   // P buffers: [128, 160), [160, 192) (f16 pairs)
constexpr uint32_t AT_O_COL = 256;   // O: [256, 256 + hd)
constexpr float AT_LOG2E = 1.4426950408889634f;
constexpr float AT_RESCALE = 8.0f;   // log2 of the largest P before O is rescaled
constexpr uint32_t AT_BOXW_MAX = 160;  // bytes of a staged ring row (hd 128: 136 + lead-in)
constexpr int AT_KV_ST = 3;            // K/V tile stages (the converters run ahead of P V)

template <int HD>
struct AtGeom {
    static constexpr int HB = HD / 32 * 34;                 // ring bytes of one kv head
    static constexpr uint32_t Q_BYTES = AT_TQ * HD * 2;     // Q tile, f16
    static constexpr uint32_t K_BYTES = AT_CK * HD * 2;     // K tile [64 keys][hd]
    static constexpr uint32_t V_BYTES = AT_CK * HD * 2;     // V tile [64 keys][hd]
    static constexpr uint32_t RAW_BYTES = AT_CK * AT_BOXW_MAX;  // one tensor's staged rows
    // layout: Q | K tiles | V tiles | raw K0, V0, K1, V1 | barriers
    static constexpr uint32_t OFF_K = Q_BYTES;
    static constexpr uint32_t OFF_V = OFF_K + AT_KV_ST * K_BYTES;
    static constexpr uint32_t OFF_RAW = OFF_V + AT_KV_ST * V_BYTES;
    static constexpr uint32_t OFF_BAR = OFF_RAW + 4 * RAW_BYTES;
    static constexpr uint32_t OFF_RED = OFF_BAR + 256;  // softmax pairs: row maxima, row sums
    static constexpr uint32_t SMEM = OFF_RED + 3 * 2 * AT_TQ * 4 + 1024;  // + alignment slack
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

// Shared-memory descriptor of an MN-major operand with the 128-byte swizzle: 128-byte rows of
// 64 f16 along MN, 8 rows (K) per 1024-byte atom; `lbo` bytes between the atoms of successive
// 64-element MN blocks, 1024 bytes between successive 8-row K groups.
__device__ __forceinline__ uint64_t sw128_mn_desc(uint32_t saddr, uint32_t lbo) {
    uint64_t d = 0;
    d |= (uint64_t)((saddr >> 4) & 0x3FFFu);
    d |= (uint64_t)((lbo >> 4) & 0x3FFFu) << 16;
    d |= (uint64_t)(1024 >> 4) << 32;
    d |= (uint64_t)1 << 46;
    d |= (uint64_t)2 << 61;
    return d;
}

// One key's staged ring row of one kv head (the head's first byte at LEAD, the row 16-byte
// aligned) dequantized to f16(d * q) into row `key` of a [64 keys][HD] tile with the 128-byte
// swizzle.  A code byte q becomes f16 by a byte permute: (q ^ 0x80) is the low byte of the
// f16 1024 + (q + 128), from which 1152 is subtracted exactly; the product with the block's
// f16 scale is rounded once (mul.rn, no contraction), as f16(float(d) * q) is: the two agree
// bit for bit.  A dead key (past the CTA's range) is written as zeros.
template <int HD, int LEAD>
__device__ __forceinline__ void convert_key_row(const uint8_t* row, uint8_t* tile, int key,
                                                bool live) {
    constexpr int NB = HD / 32;
    constexpr int NW = (LEAD + NB * 34 + 15) / 16 * 4;  // 32-bit words staged for the head
    uint32_t w[NW];
#pragma unroll
    for (int i = 0; i < NW / 4; i++) {
        const uint4 x = reinterpret_cast<const uint4*>(row)[i];
        w[4 * i] = x.x;
        w[4 * i + 1] = x.y;
        w[4 * i + 2] = x.z;
        w[4 * i + 3] = x.w;
    }
    const __half2 bias = __half2half2(__ushort_as_half((unsigned short)0x6480u));  // 1152
#pragma unroll
    for (int b = 0; b < NB; b++) {
        const int so = LEAD + 34 * b;  // the block's scale; its 32 codes follow
        const uint32_t sbits = (so & 2) ? (w[so >> 2] >> 16) : (w[so >> 2] & 0xFFFFu);
        uint32_t d2u = __byte_perm(sbits, 0u, 0x1010);
        if (!live) d2u = 0u;
        const __half2 d2 = *reinterpret_cast<const __half2*>(&d2u);
#pragma unroll
        for (int c8 = 0; c8 < 4; c8++) {
            uint32_t out[4];
#pragma unroll
            for (int jj = 0; jj < 2; jj++) {
                const int o = so + 2 + 8 * c8 + 4 * jj;  // byte offset of 4 codes
                uint32_t x = (o & 3) ? __byte_perm(w[o >> 2], w[(o >> 2) + 1], 0x5432) : w[o >> 2];
                x ^= 0x80808080u;
                uint32_t lo = __byte_perm(x, 0x64646464u, 0x5140);
                uint32_t hi = __byte_perm(x, 0x64646464u, 0x7362);
                __half2 hl = __hmul2_rn(__hsub2(*reinterpret_cast<__half2*>(&lo), bias), d2);
                __half2 hh = __hmul2_rn(__hsub2(*reinterpret_cast<__half2*>(&hi), bias), d2);
                out[2 * jj] = *reinterpret_cast<uint32_t*>(&hl);
                out[2 * jj + 1] = *reinterpret_cast<uint32_t*>(&hh);
            }
            *reinterpret_cast<uint4*>(tile + sw128_off(key, b * 4 + c8, AT_CK)) =
                make_uint4(out[0], out[1], out[2], out[3]);
        }
    }
}

template <int HD>
__device__ __forceinline__ void convert_key_row_any(int lead, const uint8_t* row, uint8_t* tile,
                                                    int key, bool live) {
    if (lead == 0) {
        convert_key_row<HD, 0>(row, tile, key, live);
    } else if (lead == 8) {
        convert_key_row<HD, 8>(row, tile, key, live);
    } else if constexpr (HD == 64) {
        if (lead == 4)
            convert_key_row<HD, 4>(row, tile, key, live);
        else
            convert_key_row<HD, 12>(row, tile, key, live);
    }
}

__device__ __forceinline__ float fmax3(float x, float y, float z) {
    float r;
    asm("max.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(x), "f"(y), "f"(z));
    return r;
}

// 2^x by the special-function unit's approximation (ex2.approx; -inf -> +0)
__device__ __forceinline__ float ex2_approx(float x) {
    float r;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(x));
    return r;
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
    float* part;           // split tiles: [work][H][128 rows][hd] fp32 O / l
    float* part_lse;       // split tiles: [work][H][128 rows] m + log2(l), log2 units
    size_t start_pos;
    int n, H, Hkv;
    int boxw;              // bytes of a staged ring row (16-byte multiple)
    int per_cta;           // key-chunk budget of a CTA: c chunks run as ceil(c / per_cta) CTAs
    float scale_log2;      // log2(e) / sqrt(hd)
    int* err;
};

// Key chunks of the 128-token tile x: positions 0 .. start_pos + the tile's last token.
__host__ __device__ __forceinline__ int at_tile_chunks(size_t start_pos, int n, int x) {
    const long last = (long)(x + 1) * AT_TQ < (long)n ? (long)(x + 1) * AT_TQ : (long)n;
    return (int)(((long)start_pos + last + AT_CK - 1) / AT_CK);
}

// The CTA `w` of a launch: tile, its chunk range (the tile's chunks divided evenly among its
// splits), the tile's split count and the work index of its first split.
struct AtWork {
    int tile, c_begin, c_end, splits, first;
};

__device__ __forceinline__ AtWork at_work(const AtArgs& a, int w) {
    const int tiles = (a.n + AT_TQ - 1) / AT_TQ;
    if (a.per_cta >= at_tile_chunks(a.start_pos, a.n, tiles - 1))  // no tile is split
        return {w, 0, at_tile_chunks(a.start_pos, a.n, w), 1, w};
    int first = 0;
    for (int x = 0; x < tiles; x++) {
        const int nch = at_tile_chunks(a.start_pos, a.n, x);
        const int gx = (nch + a.per_cta - 1) / a.per_cta;
        if (w < first + gx) {
            const int g = w - first;
            return {x, g * nch / gx, (g + 1) * nch / gx, gx, first};
        }
        first += gx;
    }
    return {tiles, 0, 0, 0, first};
}

template <int HD>
__global__ void __launch_bounds__(AT_THREADS, 1)
    attn_prefill_tc_kernel(const __grid_constant__ AtArgs a,
                           const __grid_constant__ CUtensorMap tmap_k,
                           const __grid_constant__ CUtensorMap tmap_v,
                           const __grid_constant__ CUtensorMap tmap_o,
                           const __grid_constant__ CUtensorMap tmap_p) {
    using G = AtGeom<HD>;
    constexpr unsigned FULL = 0xffffffffu;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
    uint8_t* sQ = smem;
    uint8_t* sK = smem + G::OFF_K;
    uint8_t* sV = smem + G::OFF_V;
    uint8_t* sRaw = smem + G::OFF_RAW;  // stage s: K at 2s, V at 2s + 1 (RAW_BYTES each)
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + G::OFF_BAR);
    uint64_t* q_full = bars;        // softmax warps: the query tile is in place
    uint64_t* raw_full = bars + 1;  // [2] producer: the chunk's ring rows landed
    uint64_t* raw_free = bars + 3;  // [2] converters: done reading the chunk's ring rows
    uint64_t* kv_full = bars + 5;   // [3] converters: the chunk's K and V tiles in place
    uint64_t* kv_free = bars + 8;   // [3] MMA: the chunk's P V done, its tiles may be refilled
    uint64_t* s_full = bars + 11;   // [2] MMA: S of the chunk in TMEM
    uint64_t* p_full = bars + 13;   // [2] softmax: P of the chunk in TMEM, O rescaled
    uint64_t* pv_done = bars + 15;  // [2] MMA: P V of the chunk done (per P buffer)
    uint64_t* drained = bars + 17;  // MMA: everything it issued has completed
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 18);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
    float* red = reinterpret_cast<float*>(smem + G::OFF_RED);  // [3][2][128]: max (2 slots), l

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const AtWork wk = at_work(a, blockIdx.x);
    const int t0 = wk.tile * AT_TQ, h = blockIdx.y;
    const int kvh = h / (a.H / a.Hkv);
    const long last_tok = min((long)a.n - 1, (long)t0 + AT_TQ - 1);
    const long key_end = (long)a.start_pos + last_tok + 1;  // keys [0, key_end) for the tile
    const int cb = wk.c_begin, nloc = wk.c_end - wk.c_begin;  // this CTA's chunks
    if (wk.tile >= (a.n + AT_TQ - 1) / AT_TQ || nloc <= 0) return;  // (not for a planned grid)
    const int x0 = (kvh * G::HB) & ~15;  // TMA x coordinate: 16-byte aligned
    const int lead = kvh * G::HB - x0;   // the head's first byte inside a staged row

    if (threadIdx.x == 0) {
        mbar_init(q_full, 8);
        for (int s = 0; s < 2; s++) {
            mbar_init(&raw_full[s], 1);
            mbar_init(&raw_free[s], 4);
            mbar_init(&s_full[s], 1);
            mbar_init(&p_full[s], 8);
            mbar_init(&pv_done[s], 1);
        }
        for (int s = 0; s < AT_KV_ST; s++) {
            mbar_init(&kv_full[s], 4);
            mbar_init(&kv_free[s], 1);
        }
        mbar_init(drained, 1);
        *abort_flag = 0;
        fence_barrier_init();
        prefetch_tensormap(&tmap_k);
        prefetch_tensormap(&tmap_v);
        prefetch_tensormap(wk.splits > 1 ? &tmap_p : &tmap_o);
    }
    if (warp == 12) {
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

    if (warp < 8) {
        // the queries (softmax warps, while the converters start on the first chunk), f16 into
        // the swizzled K-major tile: batches of QB items per thread, all of a batch's loads
        // issued before any is converted
        constexpr int QITEMS = AT_TQ * (HD / 8) / 256, QB = QITEMS < 8 ? QITEMS : 8;
#pragma unroll
        for (int i0 = 0; i0 < QITEMS; i0 += QB) {
            float4 xv[QB][2];
#pragma unroll
            for (int i = 0; i < QB; i++) {
                const int it = threadIdx.x + (i0 + i) * 256;
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
                const int it = threadIdx.x + (i0 + i) * 256;
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
    }

    if (warp == 13) {
        // ------------------------------ producer ------------------------------
        if (lane == 0) {
            const uint32_t bytes = 2u * AT_CK * (uint32_t)a.boxw;
            for (int i = 0; i < nloc; i++) {
                const int s = i & 1, c = cb + i;
                if (i >= 2 &&
                    !mbar_wait_bounded(&raw_free[s], ((i >> 1) - 1) & 1, a.err, abort_flag))
                    break;
                mbar_arrive_expect_tx(&raw_full[s], bytes);
                tma_load_2d(sRaw + (2 * s) * G::RAW_BYTES, &tmap_k, x0, c * AT_CK, &raw_full[s]);
                tma_load_2d(sRaw + (2 * s + 1) * G::RAW_BYTES, &tmap_v, x0, c * AT_CK,
                            &raw_full[s]);
            }
        }
    } else if (warp >= 8 && warp < 12) {
        // ------------------------------ converters ------------------------------
        const int ct = threadIdx.x - 256;
        for (int i = 0; i < nloc; i++) {
            const int s = i & 1, c = cb + i;
            if (!__all_sync(FULL, mbar_wait_bounded(&raw_full[s], (i >> 1) & 1, a.err,
                                                    abort_flag)))
                break;
            const int ks = i % AT_KV_ST;
            if (i >= AT_KV_ST &&
                !__all_sync(FULL, mbar_wait_bounded(&kv_free[ks], (i / AT_KV_ST - 1) & 1, a.err,
                                                    abort_flag)))
                break;
            // thread ct: tensor ct / 64 (K, V), key ct % 64 of the chunk
            const int tsel = ct >> 6, key = ct & 63;
            const bool live = (long)c * AT_CK + key < key_end;
            convert_key_row_any<HD>(lead, sRaw + (2 * s + tsel) * G::RAW_BYTES + key * a.boxw,
                                    (tsel ? sV + ks * G::V_BYTES : sK + ks * G::K_BYTES), key,
                                    live);
            fence_proxy_async_smem();
            __syncwarp();
            if (lane == 0) {
                mbar_arrive(&kv_full[ks]);
                mbar_arrive(&raw_free[s]);
            }
        }
    } else if (warp == 12) {
        // ------------------------------ MMA issuer ------------------------------
        if (lane == 0) {
            // kind::f16, D f32, A = B = f16; N >> 3 at bit 17, M >> 4 at bit 24
            const uint32_t idesc_s =
                (1u << 4) | ((uint32_t)(AT_CK >> 3) << 17) | ((uint32_t)(AT_TQ >> 4) << 24);
            // O += P V: B = V read MN-major (bit 16)
            const uint32_t idesc_o = (1u << 4) | (1u << 16) | ((uint32_t)(HD >> 3) << 17) |
                                     ((uint32_t)(AT_TQ >> 4) << 24);
            auto issue_s = [&](int i) -> bool {
                const int s = i & 1, ks = i % AT_KV_ST;
                if (!mbar_wait_bounded(&kv_full[ks], (i / AT_KV_ST) & 1, a.err, abort_flag))
                    return false;
                tc_fence_after();
                const uint32_t qa = smem_u32(sQ), kb = smem_u32(sK + ks * G::K_BYTES);
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
            for (int i = 0; ok && i < nloc; i++) {
                const int s = i & 1;
                // S of the next chunk overlaps this chunk's softmax (its buffer was read by the
                // softmax of chunk i - 1, whose P this loop already waited for)
                if (i + 1 < nloc && !issue_s(i + 1)) break;
                if (!mbar_wait_bounded(&p_full[s], (i >> 1) & 1, a.err, abort_flag)) break;
                tc_fence_after();
                const uint32_t vb = smem_u32(sV + (i % AT_KV_ST) * G::V_BYTES);
#pragma unroll
                for (int kk = 0; kk < AT_CK / 16; kk++)
                    mma_ts(tmem + AT_O_COL, tmem + AT_P_COL + (uint32_t)s * 32u + (uint32_t)kk * 8u,
                           sw128_mn_desc(vb + (uint32_t)kk * 2048u, 64u * 128u), idesc_o,
                           (i > 0 || kk > 0) ? 1u : 0u);
                commit_to(&pv_done[s]);
                commit_to(&kv_free[i % AT_KV_ST]);
            }
            commit_to(drained);
            mbar_wait_bounded(drained, 0, a.err, nullptr);
        }
    } else {
        // ------------------------------ softmax (warps 0-7) ------------------------------
        // warp w: TMEM lanes 32 (w % 4) .. (rows), half w / 4 of every chunk's 64 keys and of O's
        // columns; the two warps of a row quarter share each chunk's row maximum through `red`
        // behind a 64-thread named barrier.  Neither leaves the loop early (a missing partner
        // would hold the other at the barrier): after a failed wait a warp only keeps meeting
        // the barriers.
        const int rq = warp & 3, hf = warp >> 2;
        const int row = rq * 32 + lane;  // TMEM lane
        const int t = t0 + row;
        const long pos = (long)a.start_pos + t;
        const uint32_t lane_base = ((uint32_t)(rq * 32)) << 16;
        const long pos_first = (long)a.start_pos + t0;  // the tile's first query position
        const float sc = a.scale_log2;
        float* red_max = red;              // [2 chunk slots][2 halves][128 rows]
        float* red_l = red + 4 * AT_TQ;    // [2 halves][128 rows]
        // running maximum in log2 units (-inf while no key of the CTA's range is visible to
        // the row: possible in a split other than the tile's first), this half's row sum
        float m_used = -INFINITY, l = 0.0f;
        bool ok = true;
        for (int i = 0; i < nloc; i++) {
            const int s = i & 1;
            ok = ok && __all_sync(FULL, mbar_wait_bounded(&s_full[s], (i >> 1) & 1, a.err,
                                                          abort_flag));
            uint32_t v[32];
            float mxh = -INFINITY;
            if (ok) {
                tc_fence_after();
                tmem_ld32(tmem + lane_base + AT_S_COL + (uint32_t)s * 64u + (uint32_t)hf * 32u, v);
                const long k0 = (long)(cb + i) * AT_CK + hf * 32;
                if (k0 + 31 > pos_first) {  // the half reaches past some row's position
#pragma unroll
                    for (int j = 0; j < 32; j++)
                        if (k0 + j > pos) v[j] = __float_as_uint(-INFINITY);
                }
                // the half's maximum of the raw scores (the scale is positive)
                float mx4[4];
#pragma unroll
                for (int q8 = 0; q8 < 4; q8++) {
                    const uint32_t* u = &v[q8 * 8];
                    mx4[q8] = fmax3(fmax3(__uint_as_float(u[0]), __uint_as_float(u[1]),
                                          __uint_as_float(u[2])),
                                    fmax3(__uint_as_float(u[3]), __uint_as_float(u[4]),
                                          __uint_as_float(u[5])),
                                    fmaxf(__uint_as_float(u[6]), __uint_as_float(u[7])));
                }
                mxh = fmax3(mx4[0], mx4[1], fmaxf(mx4[2], mx4[3]));
            }
            // slot i % 2: the partner read slot i % 2 of chunk i - 2 before the barrier of i - 1
            red_max[((i & 1) * 2 + hf) * AT_TQ + row] = mxh;
            named_barrier_sync(2 + rq, 64);
            const float mx = fmaxf(mxh, red_max[((i & 1) * 2 + (hf ^ 1)) * AT_TQ + row]);
            if (!ok) continue;
            const float m_new = fmaxf(m_used, mx * sc);
            if (i == 0) {
                m_used = m_new;
            } else if (__any_sync(FULL, m_new > m_used + AT_RESCALE)) {
                // O holds P V up to the previous chunk: wait for it before scaling this half
                if (!__all_sync(FULL, mbar_wait_bounded(&pv_done[(i - 1) & 1],
                                                        (uint32_t)((i - 1) >> 1) & 1u, a.err,
                                                        abort_flag))) {
                    ok = false;
                    continue;
                }
                tc_fence_after();
                const bool mine = m_new > m_used + AT_RESCALE;
                const float alpha = mine ? ex2_approx(m_used - m_new) : 1.0f;
                if (mine) {
                    l *= alpha;
                    m_used = m_new;
                }
#pragma unroll
                for (int c0 = hf * (HD / 2); c0 < (hf + 1) * (HD / 2); c0 += 32) {
                    uint32_t o[32];
                    tmem_ld32(tmem + lane_base + AT_O_COL + (uint32_t)c0, o);
#pragma unroll
                    for (int jj = 0; jj < 32; jj++)
                        o[jj] = __float_as_uint(__uint_as_float(o[jj]) * alpha);
                    tmem_st32(tmem + lane_base + AT_O_COL + (uint32_t)c0, o);
                }
            }
            // this P buffer was last read by P V two chunks back
            if (i >= 2 && !__all_sync(FULL, mbar_wait_bounded(&pv_done[s],
                                                              (uint32_t)((i >> 1) - 1) & 1u,
                                                              a.err, abort_flag))) {
                ok = false;
                continue;
            }
            tc_fence_after();
            uint32_t pw[16];
            float ps[4] = {0.0f, 0.0f, 0.0f, 0.0f};
            const float nm = m_used == -INFINITY ? 0.0f : -m_used;
#pragma unroll
            for (int j = 0; j < 32; j += 2) {
                const float p0 = ex2_approx(fmaf(__uint_as_float(v[j]), sc, nm));
                const float p1 = ex2_approx(fmaf(__uint_as_float(v[j + 1]), sc, nm));
                ps[(j >> 1) & 3] += p0 + p1;
                pw[j >> 1] = h2(p0, p1);
            }
            l += (ps[0] + ps[1]) + (ps[2] + ps[3]);
            tmem_st16(tmem + lane_base + AT_P_COL + (uint32_t)s * 32u + (uint32_t)hf * 16u, pw);
            tmem_st_wait();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&p_full[s]);
        }
        // epilogue: the row sum of both halves; O / l staged in the (now unused) K/V tiles as
        // 128-byte-swizzled boxes of 128 rows, each half its columns, then stored by TMA — f16
        // into out for a tile of one CTA, fp32 partials (+ the row's lse) for a split tile
        const bool fin = ok && __all_sync(FULL, mbar_wait_bounded(&pv_done[(nloc - 1) & 1],
                                                                  (uint32_t)((nloc - 1) >> 1) & 1u,
                                                                  a.err, abort_flag));
        red_l[hf * AT_TQ + row] = l;
        named_barrier_sync(2 + rq, 64);
        const float lt = red_l[row] + red_l[AT_TQ + row];
        const bool split = wk.splits > 1;
        uint8_t* stg = sK;
        if (fin) {
            tc_fence_after();
            const float inv = lt > 0.0f ? 1.0f / lt : 0.0f;
#pragma unroll
            for (int c0 = hf * (HD / 2); c0 < (hf + 1) * (HD / 2); c0 += 32) {
                uint32_t o[32];
                tmem_ld32(tmem + lane_base + AT_O_COL + (uint32_t)c0, o);
                const float* f = reinterpret_cast<const float*>(o);
                if (split) {
                    uint8_t* bx = stg + (c0 / 32) * (AT_TQ * 128) + row * 128;
#pragma unroll
                    for (int k = 0; k < 8; k++)
                        *reinterpret_cast<float4*>(bx + ((k ^ (row & 7)) << 4)) =
                            make_float4(f[4 * k] * inv, f[4 * k + 1] * inv, f[4 * k + 2] * inv,
                                        f[4 * k + 3] * inv);
                } else {
                    uint8_t* bx = stg + (c0 / 64) * (AT_TQ * 128) + row * 128;
#pragma unroll
                    for (int k = 0; k < 4; k++) {
                        const int kc = (c0 % 64) / 8 + k;
                        *reinterpret_cast<uint4*>(bx + ((kc ^ (row & 7)) << 4)) =
                            make_uint4(h2(f[8 * k] * inv, f[8 * k + 1] * inv),
                                       h2(f[8 * k + 2] * inv, f[8 * k + 3] * inv),
                                       h2(f[8 * k + 4] * inv, f[8 * k + 5] * inv),
                                       h2(f[8 * k + 6] * inv, f[8 * k + 7] * inv));
                    }
                }
            }
            if (split && hf == 0 && t < a.n)
                a.part_lse[((size_t)blockIdx.x * a.H + h) * AT_TQ + row] =
                    lt > 0.0f ? m_used + __log2f(lt) : -INFINITY;
        }
        fence_proxy_async_smem();
        named_barrier_sync(1, 256);
        if (threadIdx.x == 0 && *abort_flag == 0) {
            if (split) {
                for (int j = 0; j < HD / 32; j++)
                    tma_store_2d(&tmap_p, j * 32, (blockIdx.x * a.H + h) * AT_TQ,
                                 stg + j * (AT_TQ * 128));
            } else {
                for (int j = 0; j < HD / 64; j++)
                    tma_store_3d(&tmap_o, j * 64, h, t0, stg + j * (AT_TQ * 128));
            }
            bulk_commit();
            bulk_wait_read_all();
        }
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 12) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem),
                     "r"(AT_TMEM_COLS)
                     : "memory");
    }
}

// Merges the splits of each split tile: out = sum_g 2^(lse_g - m) (O/l)_g / sum_g 2^(lse_g - m)
// as f16, combined online over the splits (split 0 holds key 0, so its lse is finite).
// Grid (tiles x 128 / RPB, H): a block is RPB rows of one tile, a thread 4 dimensions of a row;
// blocks of tiles with one split return at once.
template <int HD>
__global__ void __launch_bounds__(256) attn_prefill_merge_kernel(const __grid_constant__ AtArgs a) {
    pdl_launch_dependents();
    constexpr int TPR = HD / 4;     // threads per row
    constexpr int RPB = 256 / TPR;  // rows per block
    const int x = blockIdx.x / (AT_TQ / RPB), h = blockIdx.y;
    const int row = (blockIdx.x % (AT_TQ / RPB)) * RPB + threadIdx.x / TPR;
    const int sub = threadIdx.x % TPR;
    int first = 0, gx = 0;
    for (int xx = 0; xx <= x; xx++) {
        const int g = (at_tile_chunks(a.start_pos, a.n, xx) + a.per_cta - 1) / a.per_cta;
        if (xx == x)
            gx = g;
        else
            first += g;
    }
    const int t = x * AT_TQ + row;
    if (gx <= 1 || t >= a.n) return;
    pdl_wait_prerequisites();
    size_t u = ((size_t)first * a.H + h) * AT_TQ + row;
    const size_t ustep = (size_t)a.H * AT_TQ;
    float m = a.part_lse[u], wsum = 1.0f;
    float4 acc = *reinterpret_cast<const float4*>(a.part + u * HD + sub * 4);
#pragma unroll 4
    for (int g = 1; g < gx; g++) {
        u += ustep;
        const float lg = a.part_lse[u];
        const float4 p = *reinterpret_cast<const float4*>(a.part + u * HD + sub * 4);
        const float mn = fmaxf(m, lg);
        const float so = ex2_approx(m - mn), w = ex2_approx(lg - mn);
        acc = make_float4(fmaf(w, p.x, acc.x * so), fmaf(w, p.y, acc.y * so),
                          fmaf(w, p.z, acc.z * so), fmaf(w, p.w, acc.w * so));
        wsum = fmaf(wsum, so, w);
        m = mn;
    }
    const float inv = 1.0f / wsum;
    *reinterpret_cast<uint2*>(a.out + ((size_t)t * a.H + h) * HD + sub * 4) =
        make_uint2(h2(acc.x * inv, acc.y * inv), h2(acc.z * inv, acc.w * inv));
}

template <int HD>
int launch_hd_tc(sulimo_ctx* ctx, const AtArgs& a, int nwork, const CUtensorMap& tk,
                 const CUtensorMap& tv, const CUtensorMap& to, const CUtensorMap& tp) {
    static DeviceBits attr;
    if (!attr.test(ctx->device)) {
        int st = check_cuda(cudaFuncSetAttribute(attn_prefill_tc_kernel<HD>,
                                                 cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                 (int)AtGeom<HD>::SMEM),
                            "prefill attention smem attribute");
        if (st) return st;
        attr.set(ctx->device);
    }
    const int tiles = (a.n + AT_TQ - 1) / AT_TQ;
    cudaError_t e = launch_pdl(attn_prefill_tc_kernel<HD>, dim3((unsigned)nwork, (unsigned)a.H),
                               dim3(AT_THREADS), (size_t)AtGeom<HD>::SMEM, ctx->stream, a, tk,
                               tv, to, tp);
    ctx->launches++;
    int st = check_cuda(e, "attn_prefill_tc launch");
    if (st || nwork == tiles) return st;
    constexpr int rpb = 256 / (HD / 4);
    e = launch_pdl(attn_prefill_merge_kernel<HD>,
                   dim3((unsigned)(tiles * (AT_TQ / rpb)), (unsigned)a.H), dim3(256), 0,
                   ctx->stream, a);
    ctx->launches++;
    return check_cuda(e, "attn_prefill_merge launch");
}

// The chunk budget of a CTA: the smallest (at least two chunks) whose CTAs, over all tiles
// and heads, fit in one wave of one CTA per SM.  Returns the number of CTAs per head.
int plan_splits(size_t start_pos, int n, int H, int num_sms, int* per_cta) {
    const int tiles = (n + AT_TQ - 1) / AT_TQ;
    const int per_head = std::max(1, (num_sms > 0 ? num_sms : 148) / H);
    int total = 0, most = 1;
    for (int x = 0; x < tiles; x++) {
        const int c = at_tile_chunks(start_pos, n, x);
        total += c;
        most = std::max(most, c);
    }
    auto ctas = [&](int per) {
        int w = 0;
        for (int x = 0; x < tiles; x++) w += (at_tile_chunks(start_pos, n, x) + per - 1) / per;
        return w;
    };
    int per = tiles >= per_head ? most : std::max(2, (total + per_head - 1) / per_head);
    while (per < most && ctas(per) > per_head) per++;
    per = std::min(per, most);
    *per_cta = per;
    return ctas(per);
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
    a.part = nullptr;
    a.part_lse = nullptr;
    const int nwork = plan_splits(start_pos, n_tok, H, ctx->num_sms, &a.per_cta);
    if (nwork > (n_tok + AT_TQ - 1) / AT_TQ) {
        // split partials: O / l then lse, per (CTA, head, row)
        const size_t rows = (size_t)nwork * H * AT_TQ;
        int st = ensure_workspace(ctx, rows * ((size_t)hd + 1) * sizeof(float));
        if (st) return st;
        a.part = reinterpret_cast<float*>(ctx->workspace);
        a.part_lse = a.part + rows * hd;
    }
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
    // the output as [n][H][hd] f16 and the split partials as [rows][hd] fp32, both stored in
    // boxes of 128 rows x 128 bytes with the 128-byte swizzle
    CUtensorMap to, tp;
    memset(&to, 0, sizeof(to));
    memset(&tp, 0, sizeof(tp));
    const uint64_t odims[3] = {(uint64_t)hd, (uint64_t)H, (uint64_t)n_tok};
    const uint64_t ostr[2] = {(uint64_t)hd * 2, (uint64_t)H * hd * 2};
    const uint32_t obox[3] = {64, 1, (uint32_t)AT_TQ};
    if ((st = encode_tensor_map(&to, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, out, 3, odims, ostr, obox,
                                CU_TENSOR_MAP_SWIZZLE_128B)))
        return st;
    if (a.part &&
        (st = encode_2d(&tp, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, a.part, (uint64_t)hd,
                        (uint64_t)nwork * H * AT_TQ, (uint64_t)hd * 4, 32, (uint32_t)AT_TQ,
                        CU_TENSOR_MAP_SWIZZLE_128B)))
        return st;
    return hd == 64 ? launch_hd_tc<64>(ctx, a, nwork, tk, tv, to, tp)
                    : launch_hd_tc<128>(ctx, a, nwork, tk, tv, to, tp);
}

}  // namespace sulimo
