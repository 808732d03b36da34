// gemm_q4_0_pair.cu — the Q4_0-weight prefill GEMM on CTA pairs (tcgen05 cta_group::2).
//
// Same contraction and numerics as gemm_q4_0_tc.cu (the reference's gemm_q4_0_f16,
// kernels/gemm_q4_0.cl:13-130, host crates/sulimo-ocl/src/gemm.rs:28-102):
//     out[t][r] = sum_b d[r][b] * sum_i x[t][32b+i] * (q[r][b][i] - 8)
// with the weights dequantized once to f16(d*(q-8)), f16 activations, fp32 accumulation.
//
// A thread-block cluster of two CTAs (one per SM) computes a 256-feature x bn-token tile with
// one tcgen05.mma.cta_group::2 stream issued by a single thread of CTA 0:
//   - A (weights, 256 x K) comes from TMEM: CTA r dequantizes its own 128 feature rows
//     m0 = 256 * pair + 128 * r into the same TMEM columns of its own SM;
//   - B (activations, bn tokens x K) comes from shared memory: CTA r holds tokens
//     n0 + r * bn/2 .. n0 + (r + 1) * bn/2 - 1 at the same offsets in its own SM;
//   - D (fp32, 128 rows x bn tokens per CTA) lands in each CTA's TMEM.
// Against the one-CTA kernel this halves the instructions the issuing thread spends per unit
// of tensor work (each MMA covers two SMs) and halves each SM's activation traffic (it loads
// bn/2 tokens, not bn).  K advances 128 values (four Q4_0 blocks, eight K=16 MMAs) per ring
// stage, so the per-stage barrier test, fence and commit are paid once per 128 k.
//
// Roles per CTA (576 threads):
//   warp 0    one thread: TMA loads of this CTA's activation half (two 64-k boxes, 128-byte
//             swizzle, K-major) and its 128 rows' raw nibbles (64 bytes per row) into the
//             stage; no multicast.  Waits on its own `empty` barrier before refilling a stage.
//   warps 2-17 dequant in four groups of four warps (one warp per TMEM lane quarter; group g
//             takes Q4_0 block g of every stage): 16 f16x2 TMEM columns per stage per row; then
//             each warp arrives on CTA 0's `afull` barrier of the stage (32 arrivals: both CTAs).
//   warp 1    CTA 0, one thread: waits `afull`, issues the eight MMAs of the stage and commits
//             to the `empty` barriers of both CTAs (multicast commit); a final commit to both
//             CTAs' `done` barriers releases the epilogues.
//   warps 2-17 epilogue (each CTA, its own 128 rows): tcgen05.ld -> f16 / f32 -> smem -> one
//             TMA tensor store per 32-token chunk; fp32 split-K partials as in the one-CTA form.
// TMEM is allocated with cta_group::2 (512 columns on each SM: the stages' weights, then the
// accumulators).  Every wait is bounded by %globaltimer; a CTA that gives up records a device
// error, drains what it issued and still reaches the closing cluster barrier, so neither CTA
// leaves while the other may still signal its shared memory.
#include <string.h>

#include "sulimo_common.cuh"
#include "sulimo_internal.h"
#include "tc_sm100.cuh"

namespace sulimo {
namespace {

constexpr int PM = 128;            // feature rows per CTA = TMEM lanes (a pair covers 256)
constexpr int PK = 128;            // k per stage: four Q4_0 blocks
constexpr int P_BN_MAX = 256;      // tokens per pair tile = MMA N (each CTA holds half)
constexpr int P_MAX_STAGES = 8;
constexpr uint32_t P_SMEM_LIMIT = 232448;
constexpr int P_DEQ_GROUPS = 4;
constexpr int P_DEQ_WARPS = 4 * P_DEQ_GROUPS;
constexpr int P_THREADS = 64 + 32 * P_DEQ_WARPS;
constexpr int P_EPI_TOKENS = 32;
constexpr uint32_t P_TMEM_COLS = 512;
constexpr uint32_t P_STAGE_COLS = PK / 2;   // f16x2 TMEM columns of a stage's weights
constexpr uint32_t P_Q_STAGE = PM * 64;     // raw nibbles per stage: 128 rows x 4 blocks x 16 B
constexpr uint32_t P_BAR_BYTES = 512;
static_assert((4 * P_MAX_STAGES + 1) * 8 + 8 <= P_BAR_BYTES, "barrier block");

// Shared memory per CTA: stages x (activation half: bn/2 rows x 256 bytes, nibbles), barriers,
// 1024 bytes of alignment slack.
__host__ __device__ constexpr uint32_t p_x_stage(int bn) { return (uint32_t)bn * 128u; }
__host__ __device__ constexpr uint32_t p_smem_bytes(int bn, int stages) {
    return (uint32_t)stages * (p_x_stage(bn) + P_Q_STAGE) + P_BAR_BYTES + 1024;
}
__host__ __device__ constexpr int p_ring_stages(int bn) {
    int s = P_MAX_STAGES;
    const int by_tmem = (int)((P_TMEM_COLS - (uint32_t)bn) / P_STAGE_COLS);
    if (by_tmem < s) s = by_tmem;
    while (s > 2 && p_smem_bytes(bn, s) > P_SMEM_LIMIT) s--;
    return s;
}
static_assert(p_ring_stages(P_BN_MAX) == 4, "256-token pair ring");
// the epilogue stages a CTA's whole fp32 tile (128 rows x bn) in the ring
static_assert(4u * (p_x_stage(256) + P_Q_STAGE) >= 256u * PM * 4u, "epilogue tile fits (256)");
static_assert(6u * (p_x_stage(128) + P_Q_STAGE) >= 128u * PM * 4u, "epilogue tile fits (128)");

__device__ __forceinline__ uint32_t cluster_ctarank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}

// Cluster barrier with a relaxed arrival: it orders no memory by itself (the mbarrier
// initializations are published by fence.mbarrier_init, the TMEM address by __syncthreads), so
// it does not wait for the arriving thread's memory operations in flight.
__device__ __forceinline__ void cluster_sync_relaxed() {
    asm volatile(
        "barrier.cluster.arrive.relaxed.aligned;\n\t"
        "barrier.cluster.wait.aligned;" ::: "memory");
}

// Gated epilogue (OUT_MODE 3): a CTA's TMEM lanes 0-63 hold 64 rows of the gate matrix, lanes
// 64-127 the same 64 rows of the up matrix; per 32-token chunk the up lanes hand their
// accumulators to the gate lanes through an exchange area ([token][64] fp32) placed after the
// f16 staging tiles ([token][64]) of the whole token tile.
__host__ __device__ constexpr uint32_t p_gate_xch_off(int bn) { return (uint32_t)bn * 64u * 2u; }
__host__ __device__ constexpr uint32_t p_gate_xch_bytes(int bn) { return (uint32_t)bn * 64u * 4u; }
static_assert(p_gate_xch_off(256) + p_gate_xch_bytes(256) <=
                  4u * (p_x_stage(256) + P_Q_STAGE), "gated exchange fits (256)");

// silu(g) * u = g * u / (1 + e^-g) with the special-function unit's exponential and reciprocal
// (relative error ~1e-6, far inside the f16 rounding of the result; e^-g = inf -> 0)
__device__ __forceinline__ float silu_times(float g, float u) {
    float r;
    asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(__fadd_rn(1.0f, __expf(-g))));
    return __fmul_rn(__fmul_rn(g, r), u);
}

// Shared-memory address of the same variable in CTA `rank` of the cluster.
__device__ __forceinline__ uint32_t mapa_shared(uint32_t addr, uint32_t rank) {
    uint32_t out;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(out) : "r"(addr), "r"(rank));
    return out;
}

// Arrival on an mbarrier in either CTA of the cluster (shared::cluster address).  The TMEM
// stores it publishes are ordered by tcgen05.wait::st + tcgen05.fence::before_thread_sync on
// this side and tcgen05.fence::after_thread_sync after the leader's wait, so the arrival keeps
// the default CTA-scope release: a cluster-scope release would also wait for this thread's
// unrelated loads in flight (the next stage's block scales).
// TMA tensor load into this CTA's shared memory whose completion is signalled on an mbarrier
// of CTA 0 of the pair (shared::cluster address): both CTAs' activation halves complete on the
// leader's barrier, the one its MMA issuer waits on.  No multicast.
__device__ __forceinline__ void tma_load_2d_to_leader(void* dst, const CUtensorMap* map, int c0,
                                                      int c1, uint32_t leader_bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%2, %3}], [%4];" ::"r"(smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(leader_bar)
        : "memory");
}

__device__ __forceinline__ void mbar_arrive_remote(uint32_t cluster_addr) {
    asm volatile("mbarrier.arrive.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr) : "memory");
}

// The eight K=16 MMAs of one 128-k stage (two 64-k activation halves of the stage, four MMAs
// each), A from TMEM, B from shared memory, into the pair's accumulators.  The first MMA
// overwrites the accumulators when `accumulate` is 0.
__device__ __forceinline__ void mma_pair_stage(uint32_t d_tmem, uint32_t a_tmem, uint64_t b0,
                                               uint64_t b1, uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred pa, pt;\n\t"
        "setp.ne.b32 pa, %4, 0;\n\t"
        "setp.eq.u32 pt, 0, 0;\n\t"
        "tcgen05.mma.cta_group::2.kind::f16 [%0], [%1], %2, %3, pa;\n\t"
        "tcgen05.mma.cta_group::2.kind::f16 [%0], [%5], %6, %3, pt;\n\t"
        "tcgen05.mma.cta_group::2.kind::f16 [%0], [%7], %8, %3, pt;\n\t"
        "tcgen05.mma.cta_group::2.kind::f16 [%0], [%9], %10, %3, pt;\n\t"
        "tcgen05.mma.cta_group::2.kind::f16 [%0], [%11], %12, %3, pt;\n\t"
        "tcgen05.mma.cta_group::2.kind::f16 [%0], [%13], %14, %3, pt;\n\t"
        "tcgen05.mma.cta_group::2.kind::f16 [%0], [%15], %16, %3, pt;\n\t"
        "tcgen05.mma.cta_group::2.kind::f16 [%0], [%17], %18, %3, pt;\n\t}"
        :
        : "r"(d_tmem), "r"(a_tmem), "l"(b0), "r"(idesc), "r"(accumulate), "r"(a_tmem + 8u),
          "l"(b0 + 2), "r"(a_tmem + 16u), "l"(b0 + 4), "r"(a_tmem + 24u), "l"(b0 + 6),
          "r"(a_tmem + 32u), "l"(b1), "r"(a_tmem + 40u), "l"(b1 + 2), "r"(a_tmem + 48u),
          "l"(b1 + 4), "r"(a_tmem + 56u), "l"(b1 + 6)
        : "memory");
}

// Arrives on the barrier at this shared-memory offset in both CTAs of the pair once every MMA
// issued before it has completed.
__device__ __forceinline__ void mma_commit_pair(uint64_t* bar) {
    asm volatile(
        "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 "
        "[%0], %1;" ::"r"(smem_u32(bar)),
        "h"((uint16_t)3)
        : "memory");
}

// OUT_MODE: 0 = f16 out, 1 = f32 out, 2 = fp32 split-K partial to the workspace [split][n][m],
// 3 = gated: CTA r of pair p computes rows p*128 + 64r .. + 63 of matrix 0 (gate) in its TMEM
// lanes 0-63 and the same rows of matrix 1 (up) in lanes 64-127, and writes silu(gate) * up for
// those 64 features as f16 [n][m] (m = rows per matrix; nibble maps of 64-row boxes).
// Otherwise the m weight rows may be up to three matrices stacked (segment g from row start[g], a
// multiple of 128, so that every CTA's 128 rows lie in one matrix): nibbles through
// tmap_q / tmap_q1 / tmap_q2, block scales from scales[g], rows[g] rows each.
template <int OUT_MODE>
__global__ void __launch_bounds__(P_THREADS, 1)
    gemm_q4_0_pair_kernel(const __grid_constant__ CUtensorMap tmap_x,
                          const __grid_constant__ CUtensorMap tmap_q,
                          const __grid_constant__ CUtensorMap tmap_q1,
                          const __grid_constant__ CUtensorMap tmap_q2,
                          const __grid_constant__ CUtensorMap tmap_out,
                          const __grid_constant__ CUtensorMap tmap_out16,
                          const __grid_constant__ PairSegs sg, int m, int k, int n, int bn, int nb,
                          int iters_per_split, int stages, int* __restrict__ err) {
    extern __shared__ uint8_t smem_raw[];
    // the same offset in both CTAs: the leader's B descriptors address both SMs' stages
    uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
    const uint32_t x_stage = p_x_stage(bn);       // two 64-k halves of bn/2 rows x 128 bytes
    const uint32_t x_half = x_stage / 2;
    const uint32_t acc_col = (uint32_t)stages * P_STAGE_COLS;  // accumulators: bn columns
    uint8_t* sx = smem;
    uint8_t* sq = smem + stages * x_stage;
    uint64_t* qfull = reinterpret_cast<uint64_t*>(sq + stages * P_Q_STAGE);  // own nibbles
    uint64_t* xfull = qfull + P_MAX_STAGES;  // CTA 0: both CTAs' activation halves
    uint64_t* empty = xfull + P_MAX_STAGES;
    uint64_t* afull = empty + P_MAX_STAGES;
    uint64_t* done = afull + P_MAX_STAGES;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done + 1);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t crank = cluster_ctarank();
    // gated: m0 = the CTA's first output feature (64 per CTA); otherwise its first row (128)
    const int m0 = OUT_MODE == 3 ? (blockIdx.x >> 1) * PM + (int)crank * (PM / 2)
                                 : (blockIdx.x >> 1) * (2 * PM) + (int)crank * PM;
    const int seg = OUT_MODE == 3 ? 0 : (m0 >= sg.start[2] ? 2 : (m0 >= sg.start[1] ? 1 : 0));
    const CUtensorMap* qmap = seg == 0 ? &tmap_q : (seg == 1 ? &tmap_q1 : &tmap_q2);
    const int lm0 = OUT_MODE == 3 ? m0 : m0 - sg.start[seg];  // first row within its matrix
    // one stage's nibbles: the CTA's 128 rows, or (gated) 64 gate rows then the same 64 up rows
    auto load_q = [&](uint8_t* dst, int kx, uint64_t* bar) {
        if (OUT_MODE == 3) {
            tma_load_2d(dst, &tmap_q, kx, m0, bar);
            tma_load_2d(dst + P_Q_STAGE / 2, &tmap_q1, kx, m0, bar);
        } else {
            tma_load_2d(dst, qmap, kx, lm0, bar);
        }
    };
    const int n0 = blockIdx.y * bn;
    const int nx0 = n0 + (int)crank * (bn / 2);  // this CTA's activation rows
    const int num_k_total = (k + PK - 1) / PK;
    const int i_begin = blockIdx.z * iters_per_split;
    const int i_end = min(num_k_total, i_begin + iters_per_split);
    const int num_k = max(0, i_end - i_begin);

    if (threadIdx.x == 0) {
        for (int s = 0; s < stages; s++) {
            mbar_init(&qfull[s], 1);
            mbar_init(&xfull[s], 1);  // CTA 0's producer arrives with both halves' bytes
            mbar_init(&empty[s], 1);
            mbar_init(&afull[s], 2 * P_DEQ_WARPS);  // every dequant warp of both CTAs
        }
        mbar_init(done, 1);
        *abort_flag = 0;
        fence_barrier_init();
        prefetch_tensormap(&tmap_x);
        prefetch_tensormap(qmap);
        if (OUT_MODE == 3) prefetch_tensormap(&tmap_q1);
        prefetch_tensormap(&tmap_out);
        pdl_launch_dependents();
        // The weights are static (no kernel that writes them lets its dependents start early):
        // the first ring pass of nibbles streams, and is dequantized, while this grid still
        // waits for the previous kernel; the activations follow the programmatic wait below.
        for (int j = 0; j < num_k && j < stages; j++) {
            mbar_arrive_expect_tx(&qfull[j], P_Q_STAGE);
            load_q(sq + j * P_Q_STAGE, (i_begin + j) * PK / 2, &qfull[j]);
        }
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                         smem_u32(tmem_slot)),
                     "r"(P_TMEM_COLS)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
    }
    // both CTAs' barriers are initialized and both TMEM allocations done before any remote
    // arrival or MMA
    tc_fence_before();
    __syncthreads();  // the barrier inits and the TMEM address

    // dequant role (warps 2-17): TMEM lane quarter warp % 4, group (warp - 2) / 4
    const uint32_t quarter = (uint32_t)(warp & 3);
    const int group = (warp - 2) >> 2;
    const int r = (int)quarter * 32 + lane;  // feature row within the CTA == TMEM lane
    // (gated: lanes 0-63 gate rows, 64-127 the same up rows)
    const int lrow = OUT_MODE == 3 ? m0 + (r & 63) : lm0 + r;
    const int rseg = OUT_MODE == 3 ? (r >> 6) : seg;
    const bool row_ok = OUT_MODE == 3 ? lrow < m : (lrow < sg.rows[seg] && m0 + r < m);
    const uint16_t* srow = sg.scales[rseg] + (size_t)(row_ok ? lrow : 0) * nb;
    const uint32_t lane_base = (quarter * 32u) << 16;
    const uint32_t afull_leader0 = mapa_shared(smem_u32(&afull[0]), 0);
    // block `group` of every stage: its scale for stage j (zero past the matrix or past k)
    auto load_scale = [&](int j) -> uint32_t {
        const int kb = 4 * (i_begin + j) + group;
        return (row_ok && j < num_k && kb < nb) ? (uint32_t)__ldg(srow + kb) : 0u;
    };
    // scales of stages 0 and 1 in flight during the cluster barrier
    uint32_t sc0 = 0u, sc1 = 0u;
    if (warp >= 2) {
        sc0 = load_scale(0);
        sc1 = load_scale(1);
    }

    cluster_sync_relaxed();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    if (warp == 0) {
        // ------------------------------ TMA producer ------------------------------
        if (lane == 0) {
            // the activations are the previous kernel's output
            pdl_wait_prerequisites();
            const uint32_t xbar0 = mapa_shared(smem_u32(&xfull[0]), 0);
            // stage j's activation halves; CTA 0 arrives with both CTAs' bytes (the peer's may
            // complete first: the phase still waits for this arrival)
            auto load_x = [&](int j, int s) {
                const int kk = (i_begin + j) * PK;
                if (crank == 0) mbar_arrive_expect_tx(&xfull[s], 2u * x_stage);
                tma_load_2d_to_leader(sx + s * x_stage, &tmap_x, kk, nx0, xbar0 + 8u * s);
                tma_load_2d_to_leader(sx + s * x_stage + x_half, &tmap_x, kk + 64, nx0,
                                      xbar0 + 8u * s);
            };
            for (int j = 0; j < num_k && j < stages; j++) load_x(j, j);
            int issued = num_k < stages ? num_k : stages;
            for (int j = stages; j < num_k; j++) {
                const int s = j % stages;
                const uint32_t ph = (uint32_t)(j / stages) & 1u;
                if (!mbar_wait_bounded(&empty[s], ph ^ 1u, err, abort_flag)) break;
                mbar_arrive_expect_tx(&qfull[s], P_Q_STAGE);
                load_q(sq + s * P_Q_STAGE, (i_begin + j) * PK / 2, &qfull[s]);
                load_x(j, s);
                issued = j + 1;
            }
            // Tail: every issued stage has landed and has been released by the leader's MMA
            // commits (multicast into this CTA; a release implies both activation halves had
            // landed), so no copy or commit still targets this CTA's shared memory when it
            // leaves.
            for (int j = (issued > stages ? issued - stages : 0); j < issued; j++) {
                const int s = j % stages;
                const uint32_t ph = (uint32_t)(j / stages) & 1u;
                mbar_wait_bounded(&qfull[s], ph, err, nullptr);
                if (!*abort_flag) mbar_wait_bounded(&empty[s], ph, err, abort_flag);
            }
        }
    } else if (warp == 1) {
        // ------------------------------ MMA issuer (CTA 0) ------------------------------
        if (lane == 0 && crank == 0) {
            // kind::f16: D f32 (bits 4-5 = 1), A = B = f16, K-major, N >> 3 at 17, M >> 4 at 24
            const uint32_t idesc =
                (1u << 4) | ((uint32_t)(bn >> 3) << 17) | ((uint32_t)((2 * PM) >> 4) << 24);
            int s = 0;
            uint32_t ph = 0;
            for (int j = 0; j < num_k; j++) {
                if (!mbar_wait_bounded(&xfull[s], ph, err, abort_flag) ||
                    !mbar_wait_bounded(&afull[s], ph, err, abort_flag))
                    break;
                tc_fence_after();
                const uint32_t xs = smem_u32(sx + s * x_stage);
                mma_pair_stage(tmem + acc_col, tmem + (uint32_t)s * P_STAGE_COLS, sw128_desc(xs),
                               sw128_desc(xs + x_half), idesc, j > 0 ? 1u : 0u);
                mma_commit_pair(&empty[s]);
                if (++s == stages) {
                    s = 0;
                    ph ^= 1u;
                }
            }
            mma_commit_pair(done);
        }
    } else {
        // --------------------------- dequant, then epilogue ---------------------------
        // Every warp dequantizes block `group` of every stage for its 32 rows (16 TMEM columns),
        // so a stage's four blocks are done by the four groups side by side and the first
        // stage is ready after one block's work.
        bool ok = true;
        for (int j = 0; j < num_k; j++) {
            const int s = j % stages;
            const uint32_t ph = (uint32_t)(j / stages) & 1u;
            const uint32_t sc = sc0;
            sc0 = sc1;
            sc1 = load_scale(j + 2);
            if (!__all_sync(0xffffffffu, mbar_wait_bounded(&qfull[s], ph, err, abort_flag))) {
                ok = false;
                break;
            }
            const uint4 qb = *reinterpret_cast<const uint4*>(sq + s * P_Q_STAGE + r * 64 +
                                                             group * 16);
            uint32_t cols[16];
            dequant_block(qb, sc, cols);
            tmem_st16(tmem + lane_base + (uint32_t)s * P_STAGE_COLS + 16u * (uint32_t)group,
                      cols);
            tmem_st_wait();
            tc_fence_before();
            __syncwarp();  // every lane's stores are complete before the warp's single arrival
            if (lane == 0) mbar_arrive_remote(afull_leader0 + (uint32_t)s * 8u);
        }
        // Epilogue: as in the one-CTA kernel, over this CTA's 128 rows and all bn tokens.
        // `done` is committed even when this split has no k stages, and is always waited for:
        // no commit may still be in flight towards this CTA when it leaves
        const bool have = ok && mbar_wait_bounded(done, 0, err, abort_flag);
        if (have) tc_fence_after();
        constexpr int ES = OUT_MODE == 0 ? 2 : 4;
        const bool issuer = (warp - 2) % 4 == 0 && lane == 0;
        // the group's chunks are c0 = 32 * (group + 4 * ci); all their TMEM loads are in flight
        // before the first wait (warp-uniform: TMEM loads are warp-collective)
        constexpr int CH = P_BN_MAX / (P_DEQ_GROUPS * P_EPI_TOKENS);
        uint32_t v[CH][32];
        const bool ld = __all_sync(0xffffffffu, have) && num_k > 0;
#pragma unroll
        for (int ci = 0; ci < CH; ci++) {
            const int c0 = (group + ci * P_DEQ_GROUPS) * P_EPI_TOKENS;
            if (ld && c0 < bn) {
                tmem_ld32_issue(tmem + lane_base + acc_col + (uint32_t)c0, v[ci]);
            } else {
#pragma unroll
                for (int jj = 0; jj < 32; jj++) v[ci][jj] = 0u;
            }
        }
#pragma unroll
        for (int ci = 0; ci < CH; ci++) tmem_ld_wait_carry(v[ci]);
        if (OUT_MODE == 3) {
            // per chunk: the up lanes (quarters 2, 3) leave their accumulators in the exchange
            // area, the gate lanes (quarters 0, 1) write silu(gate) * up as f16, and one thread
            // of the group stores the 64-feature x 32-token box
            float* xch = reinterpret_cast<float*>(sx + p_gate_xch_off(bn));
            const bool up_lane = quarter >= 2;
            const int f = r & 63;
#pragma unroll
            for (int ci = 0; ci < CH; ci++) {
                const int c0 = (group + ci * P_DEQ_GROUPS) * P_EPI_TOKENS;
                if (c0 >= bn) break;
                float* xc = xch + (size_t)c0 * 64;
                uint8_t* tile = sx + (size_t)c0 * 64 * 2;
                if (up_lane && have) {
#pragma unroll
                    for (int jj = 0; jj < 32; jj++) xc[jj * 64 + f] = __uint_as_float(v[ci][jj]);
                }
                named_barrier_sync(1 + group, 128);
                if (!up_lane && have) {
#pragma unroll
                    for (int jj = 0; jj < 32; jj++) {
                        const float y = silu_times(__uint_as_float(v[ci][jj]), xc[jj * 64 + f]);
                        *reinterpret_cast<__half*>(tile + (size_t)(jj * 64 + f) * 2) =
                            __float2half_rn(y);
                    }
                    fence_proxy_async_smem();
                }
                named_barrier_sync(1 + group, 128);
                if (issuer && have && !*abort_flag && n0 + c0 < n && m0 < m) {
                    const bool whole = c0 + P_EPI_TOKENS <= bn;
                    tma_store_2d(whole ? &tmap_out : &tmap_out16, m0, n0 + c0, tile);
                    bulk_commit();
                }
            }
        }
#pragma unroll
        for (int ci = 0; ci < CH; ci++) {
            const int c0 = (group + ci * P_DEQ_GROUPS) * P_EPI_TOKENS;
            if (OUT_MODE == 3 || c0 >= bn) break;
            uint8_t* tile = sx + (size_t)c0 * PM * ES;
            if (have) {
                uint8_t* col = tile + (size_t)r * ES;
#pragma unroll
                for (int jj = 0; jj < 32; jj++) {
                    const float f = __uint_as_float(v[ci][jj]);
                    if (ES == 2)
                        *reinterpret_cast<__half*>(col + (size_t)jj * PM * ES) = __float2half_rn(f);
                    else
                        *reinterpret_cast<float*>(col + (size_t)jj * PM * ES) = f;
                }
                fence_proxy_async_smem();
            }
            named_barrier_sync(1 + group, 128);
            if (issuer && have && !*abort_flag && n0 + c0 < n && m0 < m) {
                const bool whole = c0 + P_EPI_TOKENS <= bn;
                const CUtensorMap* map = whole ? &tmap_out : &tmap_out16;
                if (OUT_MODE == 2)
                    tma_store_3d(map, m0, n0 + c0, (int)blockIdx.z, tile);
                else
                    tma_store_2d(map, m0, n0 + c0, tile);
                bulk_commit();
            }
        }
        if (issuer) bulk_wait_read_all();
    }

    // Neither CTA frees its TMEM or leaves before both are done with the pair's MMAs, TMEM and
    // barriers.
    tc_fence_before();
    __syncthreads();
    cluster_sync_relaxed();
    if (warp == 1) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem),
                     "r"(P_TMEM_COLS)
                     : "memory");
    }
}

template <int MODE>
int pair_setup(int device) {
    static DeviceBits done;
    if (done.test(device)) return SULIMO_OK;
    int st = check_cuda(cudaFuncSetAttribute(gemm_q4_0_pair_kernel<MODE>,
                                             cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             (int)P_SMEM_LIMIT),
                        "pair gemm smem attribute");
    if (!st) done.set(device);
    return st;
}

// Launch with a cluster of two CTAs along x and programmatic stream serialization.
template <typename... Params, typename... Args>
cudaError_t launch_pair(void (*kernel)(Params...), dim3 grid, size_t smem, cudaStream_t stream,
                        Args&&... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = dim3(P_THREADS);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 2;
    return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

// Pairs that can be resident at once (clusters are placed inside a GPC, so this can be below
// half the SM count); cached per device.
int max_active_pairs(int device, int num_sms) {
    static std::atomic<int> cache[64];
    int v = cache[device & 63].load(std::memory_order_relaxed);
    if (v > 0) return v;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(2 * num_sms);
    cfg.blockDim = dim3(P_THREADS);
    cfg.dynamicSmemBytes = p_smem_bytes(P_BN_MAX, p_ring_stages(P_BN_MAX));
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    int n = 0;
    if (cudaOccupancyMaxActiveClusters(&n, gemm_q4_0_pair_kernel<0>, &cfg) != cudaSuccess ||
        n <= 0) {
        cudaGetLastError();
        n = num_sms / 2;
    }
    cache[device & 63].store(n, std::memory_order_relaxed);
    return n;
}

}  // namespace

// Tile plan of the pair kernel: token-tile width (a multiple of 32, at most 256) and K splits.
// The output tiles (256 features x bn tokens) fill the resident pairs by themselves when there
// are enough; otherwise K is split over more pairs (each split keeping >= 4 stages of 128),
// with 128-token tiles when K is at most 16 stages.
// SULIMO_PAIR_SPLIT_BN=<w> (a measurement switch) uses w-token tiles for the outputs that
// split K: narrower tiles need fewer splits for the same fill, so fewer fp32 partials.
PairPlan gemm_pair_plan(int m, int k, int n, int max_pairs) {
    PairPlan p;
    const int pm = (m + 2 * PM - 1) / (2 * PM);
    const int num_k = (k + PK - 1) / PK;
    int bn = n >= P_BN_MAX ? P_BN_MAX : ((n + 31) / 32) * 32;
    int tiles = pm * ((n + bn - 1) / bn);
    int splits = 1;
    if (tiles * 2 <= max_pairs) {
        static const int split_bn = [] {
            const char* e = getenv("SULIMO_PAIR_SPLIT_BN");
            const int v = e ? atoi(e) : 0;
            return (v >= 32 && v <= P_BN_MAX && v % 32 == 0) ? v : 0;
        }();
        if (split_bn && split_bn < bn) {
            bn = split_bn;
            tiles = pm * ((n + bn - 1) / bn);
        } else if (num_k <= 16 && bn > 128) {
            // short K: the split CTAs' fixed costs (prologue, fp32 partial epilogue) outweigh
            // their few stages; 128-token tiles need fewer splits and halve each CTA's partials
            bn = 128;
            tiles = pm * ((n + bn - 1) / bn);
        }
        splits = max_pairs / tiles;
        if (splits > num_k / 4) splits = num_k / 4;
        if (splits < 1) splits = 1;
    }
    p.bn = bn;
    p.splits = splits;
    p.iters_per_split = (num_k + splits - 1) / splits;
    p.stages = p_ring_stages(bn);
    p.smem = p_smem_bytes(bn, p.stages);
    p.grid_x = 2 * pm;
    p.grid_y = (n + bn - 1) / bn;
    return p;
}

namespace {

// Encodes the nibble map of one matrix (rows x nb*16 bytes, boxes of box_rows rows x 64 bytes).
int encode_nibbles(CUtensorMap* map, const void* quants, int rows, int nb, int box_rows = PM) {
    return encode_2d(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, quants, (uint64_t)nb * 16,
                     (uint64_t)(rows > 0 ? rows : 1), (uint64_t)nb * 16, 64, (uint32_t)box_rows,
                     CU_TENSOR_MAP_SWIZZLE_NONE);
}

// The pair GEMM over `nseg` stacked matrices.  partials != null: fp32 split-K partials into the
// workspace whatever the split count, left for the caller; otherwise `out` (f16 / f32), a
// split plan reduced by splitk_reduce.
int launch_pair_impl(sulimo_ctx* ctx, const GemmSeg* segs, int nseg, const void* x, void* out,
                     int k, int n, int out_dtype, int x_row_stride, int x_row_offset,
                     const float** partials, int* splits_out) {
    const int nb = k / 32;
    int st;
    if ((st = pair_setup<0>(ctx->device)) || (st = pair_setup<1>(ctx->device)) ||
        (st = pair_setup<2>(ctx->device)))
        return st;
    PairSegs sg;
    int m = 0;
    for (int g = 0; g < 3; g++) {
        const bool have = g < nseg;
        sg.scales[g] = reinterpret_cast<const uint16_t*>(have ? segs[g].scales : segs[0].scales);
        sg.start[g] = m;
        sg.rows[g] = have ? segs[g].rows : 0;
        m += sg.rows[g];
    }
    for (int g = nseg; g < 3; g++) sg.start[g] = m;
    const PairPlan p = gemm_pair_plan(m, k, n, max_active_pairs(ctx->device, ctx->num_sms));
    if (p.grid_y > 65535) return set_error(SULIMO_EINVAL, "too many token tiles");
    const uint8_t* xb =
        reinterpret_cast<const uint8_t*>(x) + (size_t)x_row_offset * x_row_stride * 2;
    CUtensorMap tx, tq[3], to, to16;
    st = encode_2d(&tx, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, xb, (uint64_t)k, (uint64_t)n,
                   (uint64_t)x_row_stride * 2, 64, (uint32_t)(p.bn / 2),
                   CU_TENSOR_MAP_SWIZZLE_128B);
    if (st) return st;
    for (int g = 0; g < 3; g++) {
        if (g < nseg) {
            if ((st = encode_nibbles(&tq[g], segs[g].quants, segs[g].rows, nb))) return st;
        } else {
            tq[g] = tq[0];
        }
    }
    if (p.splits == 1 && !partials) {
        const bool f32 = out_dtype == SULIMO_OUT_F32;
        const CUtensorMapDataType dt =
            f32 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
        const uint64_t rowb = (uint64_t)m * (f32 ? 4 : 2);
        if ((st = encode_2d(&to, dt, out, (uint64_t)m, (uint64_t)n, rowb, PM,
                            (uint32_t)P_EPI_TOKENS, CU_TENSOR_MAP_SWIZZLE_NONE)) ||
            (st = encode_2d(&to16, dt, out, (uint64_t)m, (uint64_t)n, rowb, PM, 16u,
                            CU_TENSOR_MAP_SWIZZLE_NONE)))
            return st;
        const dim3 grid(p.grid_x, p.grid_y, 1);
        const cudaError_t e =
            f32 ? launch_pair(gemm_q4_0_pair_kernel<1>, grid, p.smem, ctx->stream, tx, tq[0],
                              tq[1], tq[2], to, to16, sg, m, k, n, p.bn, nb, p.iters_per_split,
                              p.stages, ctx->d_error)
                : launch_pair(gemm_q4_0_pair_kernel<0>, grid, p.smem, ctx->stream, tx, tq[0],
                              tq[1], tq[2], to, to16, sg, m, k, n, p.bn, nb, p.iters_per_split,
                              p.stages, ctx->d_error);
        ctx->launches++;
        return check_cuda(e, "gemm_q4_0_pair launch");
    }
    const size_t nm = (size_t)n * m;
    if ((st = ensure_workspace(ctx, nm * p.splits * sizeof(float)))) return st;
    float* ws = reinterpret_cast<float*>(ctx->workspace);
    {
        const uint64_t dims[3] = {(uint64_t)m, (uint64_t)n, (uint64_t)p.splits};
        const uint64_t strides[2] = {(uint64_t)m * 4, (uint64_t)nm * 4};
        const uint32_t box[3] = {PM, (uint32_t)P_EPI_TOKENS, 1};
        const uint32_t box16[3] = {PM, 16u, 1};
        if ((st = encode_tensor_map(&to, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, ws, 3, dims, strides,
                                    box, CU_TENSOR_MAP_SWIZZLE_NONE)) ||
            (st = encode_tensor_map(&to16, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, ws, 3, dims, strides,
                                    box16, CU_TENSOR_MAP_SWIZZLE_NONE)))
            return st;
    }
    const dim3 grid(p.grid_x, p.grid_y, p.splits);
    st = check_cuda(launch_pair(gemm_q4_0_pair_kernel<2>, grid, p.smem, ctx->stream, tx, tq[0],
                                tq[1], tq[2], to, to16, sg, m, k, n, p.bn, nb, p.iters_per_split,
                                p.stages, ctx->d_error),
                    "gemm_q4_0_pair split-K launch");
    if (st) return st;
    ctx->launches++;
    if (partials) {
        *partials = ws;
        *splits_out = p.splits;
        return SULIMO_OK;
    }
    return launch_splitk_reduce(ctx, ws, out, nm, p.splits, out_dtype == SULIMO_OUT_F32);
}

}  // namespace

int launch_gemm_pair(sulimo_ctx* ctx, const void* scales, const void* quants, const void* x,
                     void* out, int m, int k, int n, int out_dtype, int x_row_stride,
                     int x_row_offset) {
    const GemmSeg seg{scales, quants, m};
    return launch_pair_impl(ctx, &seg, 1, x, out, k, n, out_dtype, x_row_stride, x_row_offset,
                            nullptr, nullptr);
}

bool gemm_gated_applies(int rows, int k, int n) {
    if (!gemm_uses_pair(2 * rows, k, n) || k % 32) return false;
    const PairPlan p = gemm_pair_plan(2 * rows, k, n, 74);
    return p_gate_xch_off(p.bn) + p_gate_xch_bytes(p.bn) <=
           (uint32_t)p.stages * (p_x_stage(p.bn) + P_Q_STAGE);
}

int launch_gemm_pair_gated(sulimo_ctx* ctx, const GemmSeg& gate, const GemmSeg& up,
                           const void* x, int k, int n, void* out) {
    const int rows = gate.rows, nb = k / 32;
    int st = pair_setup<3>(ctx->device);
    if (st) return st;
    PairPlan p = gemm_pair_plan(2 * rows, k, n, max_active_pairs(ctx->device, ctx->num_sms));
    if (p.grid_y > 65535) return set_error(SULIMO_EINVAL, "too many token tiles");
    p.splits = 1;  // silu is not linear: no split-K
    p.iters_per_split = (k + PK - 1) / PK;
    PairSegs sg;
    sg.scales[0] = reinterpret_cast<const uint16_t*>(gate.scales);
    sg.scales[1] = reinterpret_cast<const uint16_t*>(up.scales);
    sg.scales[2] = sg.scales[0];
    for (int g = 0; g < 3; g++) {
        sg.start[g] = 0;
        sg.rows[g] = rows;
    }
    CUtensorMap tx, tg, tu, to, to16;
    if ((st = encode_2d(&tx, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, x, (uint64_t)k, (uint64_t)n,
                        (uint64_t)k * 2, 64, (uint32_t)(p.bn / 2), CU_TENSOR_MAP_SWIZZLE_128B)) ||
        (st = encode_nibbles(&tg, gate.quants, rows, nb, PM / 2)) ||
        (st = encode_nibbles(&tu, up.quants, rows, nb, PM / 2)) ||
        (st = encode_2d(&to, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, out, (uint64_t)rows, (uint64_t)n,
                        (uint64_t)rows * 2, PM / 2, (uint32_t)P_EPI_TOKENS,
                        CU_TENSOR_MAP_SWIZZLE_NONE)) ||
        (st = encode_2d(&to16, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, out, (uint64_t)rows, (uint64_t)n,
                        (uint64_t)rows * 2, PM / 2, 16u, CU_TENSOR_MAP_SWIZZLE_NONE)))
        return st;
    const dim3 grid(2 * ((rows + PM - 1) / PM), p.grid_y, 1);
    const cudaError_t e = launch_pair(gemm_q4_0_pair_kernel<3>, grid, p.smem, ctx->stream, tx, tg,
                                      tu, tg, to, to16, sg, rows, k, n, p.bn, nb,
                                      p.iters_per_split, p.stages, ctx->d_error);
    ctx->launches++;
    return check_cuda(e, "gemm_q4_0_pair gated launch");
}

bool gemm_stacked_applies(const GemmSeg* segs, int nseg, int k, int n) {
    if (nseg < 1 || nseg > 3) return false;
    int m = 0;
    for (int g = 0; g < nseg; g++) {
        if (segs[g].rows <= 0 || (g + 1 < nseg && segs[g].rows % PM)) return false;
        m += segs[g].rows;
    }
    return gemm_uses_pair(m, k, n) && k % 32 == 0;
}

int launch_gemm_pair_stacked(sulimo_ctx* ctx, const GemmSeg* segs, int nseg, const void* x, int k,
                             int n, const float** partials, int* splits) {
    return launch_pair_impl(ctx, segs, nseg, x, nullptr, k, n, SULIMO_OUT_F32, k, 0, partials,
                            splits);
}

}  // namespace sulimo
