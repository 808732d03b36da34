// gemm_q4_0_tc.cu — Q4_0-weight prefill GEMM on sm_100a tensor cores (tcgen05 + TMEM + TMA).
//
// Computes the reference's gemm_q4_0_f16 (kernels/gemm_q4_0.cl:13-130, host crates/sulimo-ocl/
// src/gemm.rs:28-102, CPU form gemm.rs:106-147):
//     out[t][r] = sum_b d[r][b] * sum_i x[t][32b+i] * (q[r][b][i] - 8)
// for m weight rows ("features") r, k input channels and n tokens t, f16 activations, fp32
// accumulation, f16 (or f32) results.
//
// Data flow per CTA (128 features x up to 256 tokens, K streamed in 64-wide stages):
//   warp 0   TMA: activations x[n0.., k0..k0+63] -> smem (128B-swizzled, K-major) and the raw
//            Q4_0 nibbles of the 128 feature rows (32 bytes per row) -> smem.
//   warps 2-17 dequant, in four groups of four warps (one warp per TMEM lane quarter); group g
//            takes the stages j = g (mod 4).  Each thread owns one feature row (= one TMEM
//            lane), turns the stage's two Q4_0 blocks of its row into 64 f16 weights
//            f16(d*(q-8)) (exact (q-8) via the 0x6400 magic, one RNE multiply by d; the rounding
//            of the reference's f16 embedding path, crates/sulimo-engine/src/scheduler.rs:
//            345-357) and writes them to the stage's TMEM columns with tcgen05.st.  The weights
//            never touch shared memory.
//   warp 1   one thread issues tcgen05.mma kind::f16, A = weights from TMEM (M = 128 features),
//            B = activations from smem (N = tokens), D = fp32 accumulators in TMEM; each stage
//            is released with tcgen05.commit.
//   warps 2-17 epilogue: per group, 32-token chunks: tcgen05.ld of the accumulators (lane =
//            feature), convert, stage [32 tokens][128 features] in shared memory, one TMA
//            tensor store per chunk.
// Outputs with few tiles (the down projection: 1536 features) split K across CTAs; the fp32
// partials are added in split order by splitk_reduce_kernel (deterministic).  Launches use
// programmatic dependent launch (a kernel's prologue overlaps the previous kernel's tail).
// Every mbarrier wait is bounded (%globaltimer); on expiry the kernel records a device error,
// drains its in-flight copies / MMAs (again bounded), frees TMEM and returns.
// No TMA multicast: each CTA loads its own tiles.
#include <string.h>

#include "sulimo_common.cuh"
#include "sulimo_internal.h"
#include "tc_sm100.cuh"

namespace sulimo {
namespace {

constexpr int BM = 128;           // features per CTA = MMA M = TMEM lanes
constexpr int BK = 64;            // k per stage: 2 Q4_0 blocks, one 128-byte swizzle row of f16
constexpr int BN_MAX = 256;       // tokens per CTA = MMA N (max)
// The ring depth is chosen per launch: as many stages as shared memory (bn*128 + 4096 bytes
// each) and TMEM (32 weight columns each, next to bn accumulator columns) allow, at most
// MAX_STAGES.  A slot turns over in ~1.5 us (MMA, commit, TMA issue, L2/DRAM latency,
// dequant), so 256-token tiles (6 stages) keep ~4 stages of MMA work queued and narrow tiles get
// deeper rings.
constexpr int MAX_STAGES = 16;
constexpr uint32_t SMEM_LIMIT = 232448;  // dynamic shared memory per CTA on sm_100
// Dequant warps form DEQ_GROUPS groups of four (one warp per TMEM lane quarter); group g turns
// the stages j = g (mod DEQ_GROUPS) into TMEM weights, so four stages' tcgen05.st round trips
// are in flight at once (one group alone needs ~0.25 us per stage, the MMA ~0.27 us).
constexpr int DEQ_GROUPS = 4;
constexpr int DEQ_WARPS = 4 * DEQ_GROUPS;
constexpr int THREADS = 64 + 32 * DEQ_WARPS;
constexpr int EPI_TOKENS = 32;    // tokens per epilogue chunk (one TMA store each)
constexpr uint32_t TMEM_COLS = 512;
constexpr uint32_t A_COL = 0;               // A stages: columns [32*s, 32*s+32)
constexpr uint32_t Q_STAGE = BM * 32;       // bytes of raw Q4_0 nibbles per stage
constexpr uint32_t BAR_BYTES = 512;         // mbarriers + TMEM slot + flags
static_assert((3 * MAX_STAGES + 1) * 8 + 8 <= BAR_BYTES, "barrier block");
static_assert(THREADS * 112 <= 65536, "register budget of one CTA per SM");

// Shared memory of a launch: the X and Q rings, the barrier block, 1024 bytes of alignment.
__host__ __device__ constexpr uint32_t ring_bytes(int bn, int stages) {
    return (uint32_t)stages * ((uint32_t)bn * 128u + Q_STAGE);
}
__host__ __device__ constexpr uint32_t smem_bytes(int bn, int stages) {
    return ring_bytes(bn, stages) + BAR_BYTES + 1024;
}
// TMEM columns of one stage's weights: 32 f16x2 columns, or 64 in the exact-weight form
// (f16 high parts, then f16 low parts).
__host__ __device__ constexpr uint32_t stage_cols(bool exact) { return exact ? 64u : 32u; }
// Deepest ring for a token-tile width (>= 2 stages for every bn <= 256).
__host__ __device__ constexpr int ring_stages(int bn, bool exact = false) {
    int s = MAX_STAGES;
    const int by_tmem = (int)((TMEM_COLS - (uint32_t)bn) / stage_cols(exact));
    if (by_tmem < s) s = by_tmem;
    while (s > 2 && smem_bytes(bn, s) > SMEM_LIMIT) s--;
    return s;
}
static_assert(ring_stages(BN_MAX) == 6 && smem_bytes(BN_MAX, 6) <= SMEM_LIMIT, "256-token ring");
static_assert(ring_bytes(BN_MAX, 6) >= BN_MAX * BM * 4, "epilogue staging tile fits the ring");

// One stage = four K=16 MMAs into the accumulators (the first one overwrites them when
// `accumulate` is 0), issued in one instruction stream together with a non-blocking test of the
// next stage's barrier.  An mbarrier test costs ~250 cycles even on a completed phase; reading
// its result only after the MMAs are queued hides that latency behind the MMA issue.
__device__ __forceinline__ uint32_t mma_stage_and_peek(uint32_t d_tmem, uint32_t a_tmem,
                                                       uint64_t b_desc, uint32_t idesc,
                                                       uint32_t accumulate, uint64_t* peek_bar,
                                                       uint32_t peek_parity) {
    uint32_t ready;
    asm volatile(
        "{\n\t.reg .pred pa, pt, q;\n\t"
        "mbarrier.test_wait.parity.shared::cta.b64 q, [%1], %2;\n\t"
        "setp.ne.b32 pa, %7, 0;\n\t"
        "setp.eq.u32 pt, 0, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%3], [%4], %5, %6, pa;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%3], [%8], %9, %6, pt;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%3], [%10], %11, %6, pt;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%3], [%12], %13, %6, pt;\n\t"
        "selp.u32 %0, 1, 0, q;\n\t}"
        : "=r"(ready)
        : "r"(smem_u32(peek_bar)), "r"(peek_parity), "r"(d_tmem), "r"(a_tmem), "l"(b_desc),
          "r"(idesc), "r"(accumulate), "r"(a_tmem + 8u), "l"(b_desc + 2), "r"(a_tmem + 16u),
          "l"(b_desc + 4), "r"(a_tmem + 24u), "l"(b_desc + 6)
        : "memory");
    return ready;
}

// Four K=16 MMAs accumulating into D (the low-part weights of an exact-form stage).
__device__ __forceinline__ void mma_stage_acc(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc,
                                              uint32_t idesc) {
    asm volatile(
        "{\n\t.reg .pred pt;\n\t"
        "setp.eq.u32 pt, 0, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, pt;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], [%4], %5, %3, pt;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], [%6], %7, %3, pt;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], [%8], %9, %3, pt;\n\t}"
        :
        : "r"(d_tmem), "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(a_tmem + 8u), "l"(b_desc + 2),
          "r"(a_tmem + 16u), "l"(b_desc + 4), "r"(a_tmem + 24u), "l"(b_desc + 6)
        : "memory");
}

__device__ __forceinline__ void mma_commit(uint64_t* bar) {
    asm volatile(
        "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
            smem_u32(bar))
        : "memory");
}

// Row-sharded projection with the all-gather fused into the epilogue: every output chunk is
// stored (TMA tensor store, no multicast) into each rank's row-major result Y[n][F] over
// NVLink peer mappings, at this rank's column offset; when a CTA's stores are complete it adds
// 1 to every rank's arrival counter (system-scope atomics).  A rank's result is complete when
// its counter has received every rank's CTAs (wait_counter_kernel).
// Release handshake (no write-after-read on Y across calls): call `epoch` of rank r first
// publishes epoch in r's release word, from every CTA right after griddepcontrol.wait, i.e.
// once everything r enqueued on its stream before this call (its readers of the previous Y)
// has completed; a CTA stores into peer r's Y only after it has seen r's release word reach
// this call's epoch (bounded wait).
constexpr int MAX_PEERS = 8;
struct PeerOut {
    CUtensorMap map[MAX_PEERS];    // [m_local cols][n rows] of rank r's Y, 32-token boxes
    CUtensorMap map16[MAX_PEERS];  // the same, 16-token boxes (a tile's 16-token remainder)
    unsigned* flags[MAX_PEERS];    // rank r's arrival counter
    unsigned* release[MAX_PEERS];  // rank r's release word
    unsigned epoch;                // this call's number (modulo 2^32, never 0)
    int world, rank;
};

// Bounded wait until a release word reaches `epoch` (modulo 2^32); false after
// SULIMO_WAIT_LIMIT_NS, with the device error recorded.
__device__ __forceinline__ bool wait_release(const unsigned* word, unsigned epoch, int* err) {
    const uint64_t t0 = globaltimer_ns();
    while (true) {
        unsigned v;
        asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(word) : "memory");
        if ((int)(v - epoch) >= 0) return true;
        if (globaltimer_ns() - t0 > SULIMO_WAIT_LIMIT_NS) {
            record_device_error(err, SULIMO_DEVERR_WAIT_TIMEOUT);
            return false;
        }
        __nanosleep(128);
    }
}

// OUT_MODE: 0 = f16 out, 1 = f32 out, 2 = fp32 split-K partial to the workspace
// [split][n][m], 3 / 4 = f16 / f32 to every rank's Y (all by TMA tensor stores).
// EXACT: every weight d*(q-8) enters the tensor cores as two f16 parts, hi = f16(d*(q-8)) and
// lo = f16(d*(q-8) - hi), each multiplied by the same activations (twice the MMAs per stage);
// hi + lo equals d*(q-8) exactly, so every product is the reference's exact product and only
// the fp32 accumulation order differs from the reference's scalar sum.
template <int OUT_MODE, bool EXACT = false>
__device__ __forceinline__ void gemm_body(const CUtensorMap& tmap_x, const CUtensorMap& tmap_q,
                                          const CUtensorMap& tmap_out,
                                          const CUtensorMap& tmap_out16,
                                          const uint16_t* __restrict__ scales, int m, int k,
                                          int n, int bn, int nb, int iters_per_split, int stages,
                                          const PeerOut* peers, int* __restrict__ err) {
    extern __shared__ uint8_t smem_raw[];
    const uint32_t raw = smem_u32(smem_raw);
    uint8_t* smem = smem_raw + ((1024u - (raw & 1023u)) & 1023u);
    const uint32_t x_stage = (uint32_t)bn * 128u;  // a multiple of 1024: SW128 atoms stay aligned
    constexpr uint32_t SC = stage_cols(EXACT);
    const uint32_t acc_col = (uint32_t)stages * SC;  // accumulators: [acc_col, acc_col + bn)
    uint8_t* sx = smem;
    uint8_t* sq = smem + stages * x_stage;
    uint64_t* full = reinterpret_cast<uint64_t*>(sq + stages * Q_STAGE);
    uint64_t* empty = full + MAX_STAGES;
    uint64_t* afull = empty + MAX_STAGES;
    uint64_t* done = afull + MAX_STAGES;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done + 1);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int m0 = blockIdx.x * BM, n0 = blockIdx.y * bn;
    const int num_k_total = (k + BK - 1) / BK;
    const int i_begin = blockIdx.z * iters_per_split;
    const int i_end = min(num_k_total, i_begin + iters_per_split);
    const int num_k = max(0, i_end - i_begin);

    if (threadIdx.x == 0) {
        for (int s = 0; s < stages; s++) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
            mbar_init(&afull[s], 4);  // one arrival per dequant warp of the stage's group
        }
        mbar_init(done, 1);
        *abort_flag = 0;
        fence_barrier_init();
        asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmap_x)) : "memory");
        asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmap_q)) : "memory");
        asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmap_out)) : "memory");
        // Launched as a programmatic dependent: let the next kernel's CTAs start their own
        // prologue as SMs free up, then wait until the previous kernel's writes are visible
        // before the first global read (the __syncthreads below orders the other threads).
        pdl_launch_dependents();
        pdl_wait_prerequisites();
        if (OUT_MODE >= 3)  // this rank's earlier stream work is done: its Y may be rewritten
            asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(peers->release[peers->rank]),
                         "r"(peers->epoch)
                         : "memory");
        // The first ring pass needs no empty-slot waits: issue it before the TMEM allocation.
        for (int j = 0; j < num_k && j < stages; j++) {
            mbar_arrive_expect_tx(&full[j], x_stage + Q_STAGE);
            tma_load_2d(sx + j * x_stage, &tmap_x, (i_begin + j) * BK, n0, &full[j]);
            tma_load_2d(sq + j * Q_STAGE, &tmap_q, (i_begin + j) * 32, m0, &full[j]);
        }
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                         smem_u32(tmem_slot)),
                     "r"(TMEM_COLS)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    if (warp == 0) {
        // ------------------------------ TMA producer ------------------------------
        if (lane == 0) {
            int issued = num_k < stages ? num_k : stages;
            for (int j = stages; j < num_k; j++) {
                const int s = j % stages;
                const uint32_t ph = (uint32_t)(j / stages) & 1u;
                if (!mbar_wait_bounded(&empty[s], ph ^ 1u, err, abort_flag)) break;
                mbar_arrive_expect_tx(&full[s], x_stage + Q_STAGE);
                tma_load_2d(sx + s * x_stage, &tmap_x, (i_begin + j) * BK, n0, &full[s]);
                tma_load_2d(sq + s * Q_STAGE, &tmap_q, (i_begin + j) * 32, m0, &full[s]);
                issued = j + 1;
            }
            if (*abort_flag) {
                // drain: the copies already issued must land before the CTA's smem is released
                for (int j = (issued > stages ? issued - stages : 0); j < issued; j++)
                    mbar_wait_bounded(&full[j % stages], (uint32_t)(j / stages) & 1u, err,
                                      nullptr);
            }
        }
    } else if (warp == 1) {
        // ------------------------------ MMA issuer ------------------------------
        if (lane == 0) {
            // kind::f16: D f32 (bits 4-5 = 1), A = B = f16, both K-major, N>>3 at 17, M>>4 at 24
            const uint32_t idesc =
                (1u << 4) | ((uint32_t)(bn >> 3) << 17) | ((uint32_t)(BM >> 4) << 24);
            int s = 0;
            uint32_t ph = 0;
            bool ready = false;  // afull[s] already seen complete by the previous peek
            for (int j = 0; j < num_k; j++) {
                if (!ready && !mbar_wait_bounded(&afull[s], ph, err, abort_flag)) break;
                tc_fence_after();
                const int s1 = s + 1 == stages ? 0 : s + 1;
                const uint32_t ph1 = s + 1 == stages ? ph ^ 1u : ph;
                // K steps advance 32 bytes inside the swizzled 128-byte rows (descriptor +2) and
                // 8 TMEM columns of the stage's weights
                const uint64_t bdesc = sw128_desc(smem_u32(sx + s * x_stage));
                ready = mma_stage_and_peek(tmem + acc_col, tmem + A_COL + (uint32_t)s * SC, bdesc,
                                           idesc, j > 0 ? 1u : 0u, &afull[s1], ph1) != 0 &&
                        j + 1 < num_k;
                if (EXACT)
                    mma_stage_acc(tmem + acc_col, tmem + A_COL + (uint32_t)s * SC + 32u, bdesc,
                                  idesc);
                mma_commit(&empty[s]);
                if (++s == stages) {
                    s = 0;
                    ph ^= 1u;
                }
            }
            mma_commit(done);
            if (*abort_flag) mbar_wait_bounded(done, 0, err, nullptr);  // MMAs drained
        }
    } else {
        // --------------------------- dequant, then epilogue ---------------------------
        // warp w in 2..17: TMEM lane quarter w % 4, group (w - 2) / 4
        const uint32_t quarter = (uint32_t)(warp & 3);
        const int group = (warp - 2) >> 2;
        const int r = (int)quarter * 32 + lane;  // feature row within the tile == TMEM lane
        const int grow = m0 + r;
        const bool row_ok = grow < m;
        const uint16_t* srow = scales + (size_t)(row_ok ? grow : 0) * nb;
        const uint32_t lane_base = (quarter * 32u) << 16;
        // block scales of the group's next stage (two Q4_0 blocks per stage)
        auto load_scales = [&](int j, uint32_t& a, uint32_t& b) {
            const int kb = 2 * (i_begin + j);
            a = (row_ok && j < num_k && kb < nb) ? __ldg(srow + kb) : 0u;
            b = (row_ok && j < num_k && kb + 1 < nb) ? __ldg(srow + kb + 1) : 0u;
        };
        uint32_t sa_next, sb_next;
        load_scales(group, sa_next, sb_next);
        bool ok = true;
        for (int j = group; j < num_k; j += DEQ_GROUPS) {
            const int s = j % stages;
            const uint32_t ph = (uint32_t)(j / stages) & 1u;
            const uint32_t sa = sa_next, sb = sb_next;
            load_scales(j + DEQ_GROUPS, sa_next, sb_next);
            // warp-uniform, so the warp reaches its __syncwarp below together
            if (!__all_sync(0xffffffffu, mbar_wait_bounded(&full[s], ph, err, abort_flag))) {
                ok = false;
                break;
            }
            const uint4* qp = reinterpret_cast<const uint4*>(sq + s * Q_STAGE + r * 32);
            const uint4 q0 = qp[0], q1 = qp[1];
            uint32_t cols[32];
            if (EXACT) {
                uint32_t lo[32];
                dequant_block_exact(q0, sa, cols, lo);
                dequant_block_exact(q1, sb, cols + 16, lo + 16);
                tmem_st32(tmem + lane_base + A_COL + (uint32_t)s * SC, cols);
                tmem_st32(tmem + lane_base + A_COL + (uint32_t)s * SC + 32u, lo);
            } else {
                dequant_block(q0, sa, cols);
                dequant_block(q1, sb, cols + 16);
                tmem_st32(tmem + lane_base + A_COL + (uint32_t)s * SC, cols);
            }
            tmem_st_wait();
            tc_fence_before();
            __syncwarp();  // every lane's stores are complete before the warp's single arrival
            if (lane == 0) mbar_arrive(&afull[s]);
        }
        // Epilogue: each group takes 32-token chunks of the accumulators (chunk c = group,
        // group + DEQ_GROUPS, ...), stages chunk c as a [32 tokens][128 features] tile in the
        // X ring (free once `done` fired) and stores it with one TMA tensor store; the tensor
        // map clips ragged edges.  The group barriers run whether or not the accumulators are
        // valid, so a warp that gave up on a wait cannot strand the others.
        const bool have = ok && (num_k == 0 || mbar_wait_bounded(done, 0, err, abort_flag));
        if (have) tc_fence_after();
        constexpr int ES = (OUT_MODE == 0 || OUT_MODE == 3) ? 2 : 4;
        {
            const bool issuer = (warp - 2) % 4 == 0 && lane == 0;
            bool released = false;  // every peer's release word seen at this epoch
            for (int c0 = group * EPI_TOKENS; c0 < bn; c0 += DEQ_GROUPS * EPI_TOKENS) {
                uint8_t* tile = sx + (size_t)c0 * BM * ES;
                if (have) {
                    uint32_t v[32];
                    if (num_k > 0) {
                        tmem_ld32(tmem + lane_base + acc_col + (uint32_t)c0, v);
                    } else {
#pragma unroll
                        for (int jj = 0; jj < 32; jj++) v[jj] = 0u;
                    }
                    uint8_t* col = tile + (size_t)r * ES;
#pragma unroll
                    for (int jj = 0; jj < 32; jj++) {
                        const float f = __uint_as_float(v[jj]);
                        if (ES == 2)
                            *reinterpret_cast<__half*>(col + (size_t)jj * BM * ES) =
                                __float2half_rn(f);
                        else
                            *reinterpret_cast<float*>(col + (size_t)jj * BM * ES) = f;
                    }
                    fence_proxy_async_smem();
                }
                named_barrier_sync(1 + group, 128);
                if (issuer && have && !*abort_flag && n0 + c0 < n) {
                    // a 16-token remainder (bn % 32 == 16) must not spill into the next tile
                    const bool whole = c0 + EPI_TOKENS <= bn;
                    if (OUT_MODE >= 3) {
                        if (!released) {
                            for (int rk = 0; rk < peers->world; rk++)
                                if (rk != peers->rank &&
                                    !wait_release(peers->release[rk], peers->epoch, err)) {
                                    *abort_flag = 1;
                                    break;
                                }
                            asm volatile("fence.proxy.async.global;" ::: "memory");
                            released = true;
                        }
                        if (!*abort_flag)
                            for (int rk = 0; rk < peers->world; rk++)
                                tma_store_2d(whole ? &peers->map[rk] : &peers->map16[rk], m0,
                                             n0 + c0, tile);
                    } else {
                        const CUtensorMap* map = whole ? &tmap_out : &tmap_out16;
                        if (OUT_MODE == 2)
                            tma_store_3d(map, m0, n0 + c0, (int)blockIdx.z, tile);
                        else
                            tma_store_2d(map, m0, n0 + c0, tile);
                    }
                    bulk_commit();
                }
            }
            if (issuer) {
                if (OUT_MODE >= 3)
                    bulk_wait_all();  // the peers read these rows once the counters say so
                else
                    bulk_wait_read_all();
            }
        }
        if (OUT_MODE >= 3) {
            named_barrier_sync(5, 32 * DEQ_WARPS);
            if (warp == 2 && lane == 0 && have && !*abort_flag) {
                __threadfence_system();
                for (int rk = 0; rk < peers->world; rk++) atomicAdd_system(peers->flags[rk], 1u);
            }
        }
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem),
                     "r"(TMEM_COLS)
                     : "memory");
    }
}

template <int OUT_MODE, bool EXACT>
__global__ void __launch_bounds__(THREADS, 1)
    gemm_q4_0_tc_kernel(const __grid_constant__ CUtensorMap tmap_x,
                        const __grid_constant__ CUtensorMap tmap_q,
                        const __grid_constant__ CUtensorMap tmap_out,
                        const __grid_constant__ CUtensorMap tmap_out16,
                        const uint16_t* __restrict__ scales, int m, int k, int n, int bn, int nb,
                        int iters_per_split, int stages, int* __restrict__ err) {
    gemm_body<OUT_MODE, EXACT>(tmap_x, tmap_q, tmap_out, tmap_out16, scales, m, k, n, bn, nb,
                               iters_per_split, stages, nullptr, err);
}

template <int OUT_MODE>
__global__ void __launch_bounds__(THREADS, 1)
    gemm_q4_0_tc_allgather_kernel(const __grid_constant__ CUtensorMap tmap_x,
                                  const __grid_constant__ CUtensorMap tmap_q,
                                  const uint16_t* __restrict__ scales, int m, int k, int n, int bn,
                                  int nb, int stages, const __grid_constant__ PeerOut peers,
                                  int* __restrict__ err) {
    gemm_body<OUT_MODE>(tmap_x, tmap_q, tmap_x, tmap_x, scales, m, k, n, bn, nb, (k + BK - 1) / BK,
                        stages, &peers, err);
}

// Bounded wait (one thread) until *flag reaches target; records a device error after
// SULIMO_WAIT_LIMIT_NS instead of hanging.  Waits only on other GPUs' kernels (and this GPU's
// earlier, already finished, launch).
__global__ void wait_counter_kernel(const unsigned* __restrict__ flag, unsigned target,
                                    int* __restrict__ err) {
    if (threadIdx.x != 0) return;
    const uint64_t t0 = globaltimer_ns();
    while (true) {
        unsigned v;
        asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(flag) : "memory");
        if ((int)(v - target) >= 0) break;
        if (globaltimer_ns() - t0 > SULIMO_WAIT_LIMIT_NS) {
            record_device_error(err, SULIMO_DEVERR_WAIT_TIMEOUT);
            break;
        }
        __nanosleep(256);
    }
}

// Encodes a tiled tensor map of rank 2 or 3; dims/box innermost first, strides in bytes for
// dims 1.. (rank-1 entries).
int encode_map(CUtensorMap* map, CUtensorMapDataType dt, const void* base, int rank,
               const uint64_t* dims, const uint64_t* strides, const uint32_t* box,
               CUtensorMapSwizzle swz) {
    return encode_tensor_map(map, dt, base, rank, dims, strides, box, swz);
}


template <int MODE, bool EXACT = false>
int set_smem_attr(int device) {
    static DeviceBits done;  // the attribute is per device
    if (done.test(device)) return SULIMO_OK;
    int st;
    if constexpr (MODE >= 3)
        st = check_cuda(cudaFuncSetAttribute(gemm_q4_0_tc_allgather_kernel<MODE>,
                                             cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             (int)SMEM_LIMIT),
                        "gemm smem attribute");
    else
        st = check_cuda(cudaFuncSetAttribute(gemm_q4_0_tc_kernel<MODE, EXACT>,
                                             cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             (int)SMEM_LIMIT),
                        "gemm smem attribute");
    if (!st) done.set(device);
    return st;
}

}  // namespace

// Token-tile width: all tokens up to 256 (rounded up to 16), else 256.  Narrower tiles do not
// pay: every stage costs the MMA issuer a fixed ~0.15 us (barrier test, fence, commit, issue)
// whatever N is, and each weight is dequantized once per token tile.
int gemm_token_tile(int n) { return n <= BN_MAX ? ((n + 15) / 16) * 16 : BN_MAX; }

// Split count: enough CTAs to fill the SMs when the output has few tiles (the down projection
// 512 x 8960 -> 1536 has 24 tiles of 128 x 256), each split keeping >= 8 k-stages.
int gemm_splits(int tiles, int num_k, int num_sms) {
    if (tiles * 2 > num_sms) return 1;
    int s = num_sms / tiles;
    const int by_k = num_k / 8;
    if (s > by_k) s = by_k;
    return s < 1 ? 1 : s;
}

// Form of the GEMM for a shape: the CTA-pair kernel (gemm_q4_0_pair.cu) when the output has
// more than one 128-feature tile, at least 32 tokens and k >= 128, else this one-CTA kernel
// (narrow token counts such as the last-token logits, single-tile outputs).  SULIMO_GEMM_FORM=1 selects the
// one-CTA kernel for every shape (a measurement switch).
bool gemm_uses_pair(int m, int k, int n) {
    static const int forced = [] {
        const char* e = getenv("SULIMO_GEMM_FORM");
        return e ? atoi(e) : 0;
    }();
    return forced != 1 && m > BM && n >= 32 && k >= 128;
}

namespace {

// The one-CTA kernel of a launch: output mode x weight form.
template <int MODE>
auto one_cta_kernel(bool exact) {
    return exact ? gemm_q4_0_tc_kernel<MODE, true> : gemm_q4_0_tc_kernel<MODE, false>;
}

}  // namespace

int launch_gemm_q4_0_f16(sulimo_ctx* ctx, const void* scales, const void* quants, const void* x,
                         void* out, int m, int k, int n, int out_dtype, int x_row_stride,
                         int x_row_offset, bool exact) {
    if (!exact && gemm_uses_pair(m, k, n))
        return launch_gemm_pair(ctx, scales, quants, x, out, m, k, n, out_dtype, x_row_stride,
                                x_row_offset);
    const int nb = k / 32;
    const int bn = gemm_token_tile(n);
    const int stages = ring_stages(bn, exact);
    const uint32_t smem = smem_bytes(bn, stages);
    const uint8_t* xb = reinterpret_cast<const uint8_t*>(x) + (size_t)x_row_offset * x_row_stride * 2;
    CUtensorMap tx, tq;
    int st = encode_2d(&tx, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, xb, (uint64_t)k, (uint64_t)n,
                       (uint64_t)x_row_stride * 2, BK, (uint32_t)bn, CU_TENSOR_MAP_SWIZZLE_128B);
    if (st) return st;
    st = encode_2d(&tq, CU_TENSOR_MAP_DATA_TYPE_UINT8, quants, (uint64_t)nb * 16, (uint64_t)m,
                   (uint64_t)nb * 16, 32, BM, CU_TENSOR_MAP_SWIZZLE_NONE);
    if (st) return st;
    if (exact ? ((st = set_smem_attr<0, true>(ctx->device)) ||
                 (st = set_smem_attr<1, true>(ctx->device)) ||
                 (st = set_smem_attr<2, true>(ctx->device)))
              : ((st = set_smem_attr<0>(ctx->device)) || (st = set_smem_attr<1>(ctx->device)) ||
                 (st = set_smem_attr<2>(ctx->device))))
        return st;

    const int mt = (m + BM - 1) / BM, nt = (n + bn - 1) / bn;
    const int num_k = (k + BK - 1) / BK;
    const int splits = gemm_splits(mt * nt, num_k, ctx->num_sms);
    const int ips = (num_k + splits - 1) / splits;
    if (nt > 65535) return set_error(SULIMO_EINVAL, "too many token tiles");
    const uint16_t* sc = reinterpret_cast<const uint16_t*>(scales);
    CUtensorMap to, to16;
    if (splits == 1) {
        const bool f32 = out_dtype == SULIMO_OUT_F32;
        const CUtensorMapDataType dt =
            f32 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
        const uint64_t rowb = (uint64_t)m * (f32 ? 4 : 2);
        st = encode_2d(&to, dt, out, (uint64_t)m, (uint64_t)n, rowb, BM, (uint32_t)EPI_TOKENS,
                       CU_TENSOR_MAP_SWIZZLE_NONE);
        if (st) return st;
        st = encode_2d(&to16, dt, out, (uint64_t)m, (uint64_t)n, rowb, BM, 16u,
                       CU_TENSOR_MAP_SWIZZLE_NONE);
        if (st) return st;
        dim3 grid(mt, nt, 1);
        const cudaError_t e =
            f32 ? launch_pdl(one_cta_kernel<1>(exact), grid, dim3(THREADS), smem, ctx->stream, tx,
                             tq, to, to16, sc, m, k, n, bn, nb, ips, stages, ctx->d_error)
                : launch_pdl(one_cta_kernel<0>(exact), grid, dim3(THREADS), smem, ctx->stream, tx,
                             tq, to, to16, sc, m, k, n, bn, nb, ips, stages, ctx->d_error);
        ctx->launches++;
        return check_cuda(e, "gemm_q4_0_tc launch");
    }
    // split-K: fp32 partials [split][n][m] (rank 3, so a ragged token tile cannot spill into the
    // next split), then the ordered reduction
    const size_t nm = (size_t)n * m;
    if ((st = ensure_workspace(ctx, nm * splits * sizeof(float)))) return st;
    float* ws = reinterpret_cast<float*>(ctx->workspace);
    {
        const uint64_t dims[3] = {(uint64_t)m, (uint64_t)n, (uint64_t)splits};
        const uint64_t strides[2] = {(uint64_t)m * 4, (uint64_t)nm * 4};
        const uint32_t box[3] = {BM, (uint32_t)EPI_TOKENS, 1};
        const uint32_t box16[3] = {BM, 16u, 1};
        st = encode_map(&to, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, ws, 3, dims, strides, box,
                        CU_TENSOR_MAP_SWIZZLE_NONE);
        if (st) return st;
        st = encode_map(&to16, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, ws, 3, dims, strides, box16,
                        CU_TENSOR_MAP_SWIZZLE_NONE);
        if (st) return st;
    }
    dim3 grid(mt, nt, splits);
    st = check_cuda(launch_pdl(one_cta_kernel<2>(exact), grid, dim3(THREADS), smem, ctx->stream,
                               tx, tq, to, to16, sc, m, k, n, bn, nb, ips, stages, ctx->d_error),
                    "gemm_q4_0_tc split-K launch");
    if (st) return st;
    ctx->launches++;
    return launch_splitk_reduce(ctx, ws, out, nm, splits, out_dtype == SULIMO_OUT_F32);
}

int launch_splitk_reduce(sulimo_ctx* ctx, const float* ws, void* out, size_t nm, int splits,
                         bool out_f32) {
    const unsigned rb = (unsigned)((nm / 4 + 255) / 256);  // m % 8 == 0, so nm % 4 == 0
    const cudaError_t e =
        out_f32 ? launch_pdl(splitk_reduce_kernel<true>, dim3(rb), dim3(256), 0, ctx->stream, ws,
                             out, nm, splits)
                : launch_pdl(splitk_reduce_kernel<false>, dim3(rb), dim3(256), 0, ctx->stream, ws,
                             out, nm, splits);
    ctx->launches++;
    return check_cuda(e, "splitk_reduce launch");
}

}  // namespace sulimo

namespace sulimo {

int launch_gemm_allgather(sulimo_ctx* ctx, const void* scales, const void* quants, const void* x,
                          int m_local, int m_valid, int k, int n, int out_dtype,
                          void* const* out_bases, size_t f_total, size_t col0,
                          unsigned* const* flags, unsigned* const* release, int world, int rank,
                          unsigned epoch, unsigned* tiles_out) {
    const int nb = k / 32;
    const int bn = gemm_token_tile(n);
    const int stages = ring_stages(bn);
    const uint32_t smem = smem_bytes(bn, stages);
    const bool f32 = out_dtype == SULIMO_OUT_F32;
    const int es = f32 ? 4 : 2;
    CUtensorMap tx, tq;
    int st = encode_2d(&tx, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, x, (uint64_t)k, (uint64_t)n,
                       (uint64_t)k * 2, BK, (uint32_t)bn, CU_TENSOR_MAP_SWIZZLE_128B);
    if (st) return st;
    st = encode_2d(&tq, CU_TENSOR_MAP_DATA_TYPE_UINT8, quants, (uint64_t)nb * 16, (uint64_t)m_local,
                   (uint64_t)nb * 16, 32, BM, CU_TENSOR_MAP_SWIZZLE_NONE);
    if (st) return st;
    PeerOut peers;
    memset(&peers, 0, sizeof(peers));
    peers.world = world;
    peers.rank = rank;
    peers.epoch = epoch;
    const CUtensorMapDataType dt = f32 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
    for (int r = 0; r < world; r++) {
        const uint8_t* base = reinterpret_cast<const uint8_t*>(out_bases[r]) + col0 * es;
        // the map spans only this shard's valid columns: zero-scale padding rows are clipped
        if ((st = encode_2d(&peers.map[r], dt, base, (uint64_t)m_valid, (uint64_t)n,
                            (uint64_t)f_total * es, BM, (uint32_t)EPI_TOKENS,
                            CU_TENSOR_MAP_SWIZZLE_NONE)) ||
            (st = encode_2d(&peers.map16[r], dt, base, (uint64_t)m_valid, (uint64_t)n,
                            (uint64_t)f_total * es, BM, 16u, CU_TENSOR_MAP_SWIZZLE_NONE)))
            return st;
        peers.flags[r] = flags[r];
        peers.release[r] = release[r];
    }
    if ((st = f32 ? set_smem_attr<4>(ctx->device) : set_smem_attr<3>(ctx->device))) return st;
    const int mt = (m_local + BM - 1) / BM, nt = (n + bn - 1) / bn;
    if (nt > 65535) return set_error(SULIMO_EINVAL, "too many token tiles");
    *tiles_out = (unsigned)(mt * nt);
    const uint16_t* sc = reinterpret_cast<const uint16_t*>(scales);
    dim3 grid(mt, nt, 1);
    const cudaError_t e =
        f32 ? launch_pdl(gemm_q4_0_tc_allgather_kernel<4>, grid, dim3(THREADS), smem, ctx->stream,
                         tx, tq, sc, m_local, k, n, bn, nb, stages, peers, ctx->d_error)
            : launch_pdl(gemm_q4_0_tc_allgather_kernel<3>, grid, dim3(THREADS), smem, ctx->stream,
                         tx, tq, sc, m_local, k, n, bn, nb, stages, peers, ctx->d_error);
    ctx->launches++;
    return check_cuda(e, "gemm_q4_0_tc all-gather launch");
}

int launch_wait_counter(sulimo_ctx* ctx, const unsigned* flag, unsigned target) {
    wait_counter_kernel<<<1, 32, 0, ctx->stream>>>(flag, target, ctx->d_error);
    ctx->launches++;
    return check_cuda(cudaGetLastError(), "wait_counter launch");
}

}  // namespace sulimo
