// gemv_mma_q4_0_q8_0.cu — the decode matvec Q4_0 (SoA) x Q8_0 for several sequences at once, on
// the tensor cores ("fast mode" numerics, like gemv_fast_q4_0_q8_0.cu).
//
// The reference runs its matvec once per sequence (matvec_q4_0_q8_0, avx2.rs:113-164 /
// scalar.rs:173-205):
//   y[t][r] = sum_b  d_w[r][b] * d_x[t][b] * s(r, t, b),   s = sum_i (q_i - 8) * x_i  (exact int)
// Here the sequences share every weight byte.  Per 32-value block, the integer sums of 16 rows
// x 8 sequences are one mma.sync.m16n8k32 (u8 nibbles x s8 codes, int32 accumulate).  The
// accumulator is seeded with 0x4B400000 - 8 * sum(x) per sequence, so the result is s plus the
// bits of 1.5 * 2^23: as a float it is exactly 1.5 * 2^23 + s (no int -> float conversion
// instruction).  Then, per (row, sequence), in block order:
//   v   = fma(D as float, d_x, -1.5 * 2^23 * d_x)     = s * d_x, rounded once
//   acc = fma(v, d_w, acc)
// The integer block sums are the reference's; only the fp32 grouping and rounding steps differ
// from the AVX2 kernel (relative L2 error ~1e-7, like the lane-tree fast form).
//
// Operands.  A (16 rows x 32 values): lane (g, t) needs row g and g + 8, values 4t..4t+3 and
// 16+4t..16+4t+3.  A Q4_0 block's byte j holds value j (low nibble) and value j + 16 (high
// nibble), so word t of the 16-byte block gives both: low nibbles -> a0 / a1, high nibbles ->
// a2 / a3 (unsigned 0..15; the -8 is in the seed).  B (32 values x 8 sequences): words t and
// t + 4 of the sequence's codes for the block.
//
// Activations arrive in the staged form (Q8Out in sulimo_common.cuh) that the decode step's
// producers write: codes [Bp][K] i8 and aux [Bp/8][K/32][8] {d_x, seed}; the C-ABI's Q8_0
// block arrays are restaged by q8_stage_kernel first.
//
// Grid (CTAs, sequence groups of 8 * NT).  A CTA walks row bands blockIdx.x, + gridDim.x, ...
// (bands of BH = 16 * rw rows, numbered matrix by matrix so that none straddles two):
//   warp 8 (producer) copies the group's activations (all of K; rows padded by 16 bytes so the
//     eight sequences of a fragment load sit in eight bank quads) into shared memory once, and
//     streams each band's weights in stages of kc blocks through a `stages`-deep ring of full /
//     empty mbarriers: per stage, kc / 8 TMA tensor copies of the quants (boxes of BH rows x
//     128 bytes = 8 blocks) and kc / 64 of the scales (BH x 64 blocks), both with the 128-byte
//     swizzle, so a fragment load's eight rows again hit eight different bank quads.  Rows past
//     a matrix's end read as zeros.  Static weights (a decode step's model) start streaming
//     before the programmatic-launch wait.
//   warps 0-7 (consumers) = rw row tiles (16 rows) x kw = 8 / rw block groups: warp (rt, kg)
//     takes blocks kg, kg + kw, ... of each stage for row tile rt; at a band's end the kw
//     partial sums of a row tile are added in a fixed order through shared memory and stored.
// The band height is chosen so that the bands cover the SMs.
#include <string.h>

#include "sulimo_common.cuh"
#include "sulimo_internal.h"

namespace sulimo {
namespace {

constexpr int GM_CONSUMERS = 8;
constexpr int GM_THREADS = (GM_CONSUMERS + 1) * 32;
constexpr int GM_MAX_MATS = 3;
constexpr int GM_MAX_STAGES = 4;
constexpr size_t GM_SMEM_MAX = 225 * 1024;
constexpr float GM_MAGIC = 12582912.0f;  // 1.5 * 2^23 (bits 0x4B400000)

struct GmArgs {
    float* out[GM_MAX_MATS];
    int rows[GM_MAX_MATS];
    int first_band[GM_MAX_MATS];  // index of the matrix's first band
    int count;
    const int8_t* codes;  // [tiles * 8][K]
    const int2* aux;      // [tiles][nb][8]
    int K, nb, batch, tiles;
    int rw, kc, stages, bands;
    int static_weights;
    int* err;
};

// Per matrix: quants as bytes [rows][nb * 16], box 128 x BH; scales as u16 [rows][nb], box
// 64 x BH; both 128-byte swizzled.
struct GmMaps {
    CUtensorMap q[GM_MAX_MATS];
    CUtensorMap s[GM_MAX_MATS];
};

__device__ __forceinline__ uint32_t lds32(const uint8_t* p) {
    return *reinterpret_cast<const uint32_t*>(p);
}

// D = A * B + D, m16n8k32, A unsigned bytes, B signed bytes, int32 accumulators
__device__ __forceinline__ void mma_u8s8(int* d, const uint32_t* a, uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k32.row.col.s32.u8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
        "{%8,%9}, {%0,%1,%2,%3};"
        : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

__device__ __forceinline__ void consumers_sync() {
    asm volatile("bar.sync 1, %0;" ::"n"(GM_CONSUMERS * 32) : "memory");
}

__device__ __forceinline__ int matrix_of_band(const GmArgs& a, int band) {
    int m = 0;
#pragma unroll
    for (int i = 1; i < GM_MAX_MATS; i++)
        if (i < a.count && band >= a.first_band[i]) m = i;
    return m;
}

// Shared-memory geometry shared by the host plan and the kernel.  Stages come first (each a
// multiple of 1024 bytes: the swizzled boxes need 1024-byte alignment), then the activations,
// the kw-merge area and the barriers.
struct GmGeom {
    int BH;             // band rows
    int nqb, nsb;       // quants / scales boxes per stage
    size_t box;         // bytes per box (BH x 128)
    size_t stage;       // bytes per stage
    size_t act_codes;   // bytes of the codes area (8 * NT rows of K + 16)
    size_t act_aux;     // bytes of the aux area
    size_t red;         // bytes of the kw-merge area
};

__host__ __device__ inline GmGeom gm_geom(int nt, int K, int rw, int kc) {
    GmGeom g;
    g.BH = 16 * rw;
    g.nqb = kc / 8;
    g.nsb = (kc + 63) / 64;
    g.box = (size_t)g.BH * 128;
    g.stage = (size_t)(g.nqb + g.nsb) * g.box;
    g.act_codes = (size_t)8 * nt * (K + 16);
    g.act_aux = (size_t)nt * (K / 32) * 64;
    g.red = rw < GM_CONSUMERS ? (size_t)GM_CONSUMERS * 32 * nt * 4 * sizeof(float) : 0;
    return g;
}

// NT: 8-sequence tiles per CTA group; KW: block groups (8 / KW row tiles per band).
template <int NT, int KW>
__global__ void __launch_bounds__(GM_THREADS, 1)
    gemv_mma_kernel(const __grid_constant__ GmArgs a, const __grid_constant__ GmMaps maps) {
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
    const GmGeom G = gm_geom(NT, a.K, a.rw, a.kc);
    uint8_t* stages_base = smem;
    uint8_t* act_codes = stages_base + (size_t)a.stages * G.stage;
    uint8_t* act_aux = act_codes + G.act_codes;
    float* red = reinterpret_cast<float*>(act_aux + G.act_aux);
    uint64_t* full = reinterpret_cast<uint64_t*>(reinterpret_cast<uint8_t*>(red) + G.red);
    uint64_t* empty = full + a.stages;
    uint64_t* act_bar = empty + a.stages;
    volatile int* abort_flag = reinterpret_cast<volatile int*>(act_bar + 1);

    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    constexpr int kw = KW;
    const int nb = a.nb, kc = a.kc;
    const int nks = (nb + kc - 1) / kc;
    const int my_bands =
        (int)blockIdx.x < a.bands ? (a.bands - (int)blockIdx.x + (int)gridDim.x - 1) / (int)gridDim.x
                                  : 0;
    const int total = my_bands * nks;                       // stages this CTA consumes
    const int tile0 = blockIdx.y * NT;                      // first sequence tile of the group
    const int nt = min(NT, a.tiles - tile0);                // tiles of this group

    if (tid == 0) {
        for (int s = 0; s < a.stages; s++) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], GM_CONSUMERS);
        }
        mbar_init(act_bar, 1);
        *abort_flag = 0;
        fence_barrier_init();
        for (int m = 0; m < a.count; m++) {
            prefetch_tensormap(&maps.q[m]);
            prefetch_tensormap(&maps.s[m]);
        }
    }
    __syncthreads();
    pdl_launch_dependents();

    // stage seq -> (band, k-stage): lane j < nqb copies quants box j, the next lanes the scales
    auto issue = [&](int seq) {
        const int band = (int)blockIdx.x + (seq / nks) * (int)gridDim.x;
        const int ks = seq % nks;
        const int s = seq % a.stages;
        const int k0 = ks * kc, kcs = min(kc, nb - k0);
        const int m = matrix_of_band(a, band);
        const int lr0 = (band - a.first_band[m]) * G.BH;
        const int nq = kcs / 8, ns = (kcs + 63) / 64;
        uint8_t* dst = stages_base + (size_t)s * G.stage;
        if (lane == 0) mbar_arrive_expect_tx(&full[s], (uint32_t)((nq + ns) * G.box));
        __syncwarp();
        if (lane < nq)
            tma_load_2d(dst + (size_t)lane * G.box, &maps.q[m], (k0 + lane * 8) * 16, lr0, &full[s]);
        else if (lane - nq < ns)
            tma_load_2d(dst + (size_t)(G.nqb + lane - nq) * G.box, &maps.s[m],
                        k0 + (lane - nq) * 64, lr0, &full[s]);
    };

    // Static weights: the first stage streams in while the previous kernel drains; the rest
    // queue behind the activations, which the consumers need first.
    int issued = 0;
    if (warp == GM_CONSUMERS && a.static_weights && total > 0) issue(issued++);
    // the activations (and non-static weights) are written by the previous kernel
    pdl_wait_prerequisites();

    if (warp == GM_CONSUMERS) {
        // ------------------------------ producer ------------------------------
        if (total > 0) {
            const uint32_t code_bytes = (uint32_t)a.K;
            const uint32_t aux_bytes = (uint32_t)(nt * nb * 64);
            if (lane == 0) mbar_arrive_expect_tx(act_bar, (uint32_t)nt * 8 * code_bytes + aux_bytes);
            __syncwarp();
            for (int i = lane; i < nt * 8; i += 32)
                bulk_load(act_codes + (size_t)i * (a.K + 16),
                          a.codes + (size_t)(tile0 * 8 + i) * a.K, code_bytes, act_bar);
            if (lane == 0)
                bulk_load(act_aux, a.aux + (size_t)tile0 * nb * 8, aux_bytes, act_bar);
        }
        for (int seq = issued; seq < total; seq++) {
            const int s = seq % a.stages;
            if (seq >= a.stages) {
                bool ok = true;
                if (lane == 0)
                    ok = mbar_wait_bounded(&empty[s], (uint32_t)((seq / a.stages) - 1) & 1u,
                                           a.err, abort_flag);
                if (!__shfl_sync(0xffffffffu, (int)ok, 0)) break;
            }
            issue(seq);
            issued = seq + 1;
        }
    } else {
        // ------------------------------ consumers ------------------------------
        const int g = lane >> 2, t = lane & 3;
        const int rt = warp / kw, kg = warp % kw;
        const int CS = a.K + 16;
        bool ok = total == 0 ||
                  __all_sync(0xffffffffu, mbar_wait_bounded(act_bar, 0u, a.err, abort_flag));
        float acc[NT][4];
#pragma unroll
        for (int n = 0; n < NT; n++) acc[n][0] = acc[n][1] = acc[n][2] = acc[n][3] = 0.0f;
        for (int seq = 0; seq < total; seq++) {
            const int s = seq % a.stages, ks = seq % nks;
            ok = ok && __all_sync(0xffffffffu, mbar_wait_bounded(&full[s],
                                                                 (uint32_t)(seq / a.stages) & 1u,
                                                                 a.err, abort_flag));
            if (ok) {
                const int k0 = ks * kc, kcs = min(kc, nb - k0);
                const uint8_t* st = stages_base + (size_t)s * G.stage;
                // row rt*16 + g of every box; the 128-byte swizzle puts 16-byte chunk c of row
                // r at chunk c ^ (r & 7), and r & 7 = g
                const uint8_t* qg = st + (size_t)(rt * 16 + g) * 128 + 4 * t;
                const uint8_t* sg = st + (size_t)G.nqb * G.box + (size_t)(rt * 16 + g) * 128;
                // U blocks per step: their fragment loads are issued before their MMAs
                constexpr int U = NT == 1 ? 4 : (NT == 2 ? 2 : 1);
                for (int b0 = kg; b0 < kcs; b0 += KW * U) {
                    uint32_t A[U][4];
                    float dw0[U], dw1[U];
#pragma unroll
                    for (int u = 0; u < U; u++) {
                        const int bl = b0 + u * KW;
                        if (bl < kcs) {
                            const uint8_t* qb =
                                qg + (size_t)(bl >> 3) * G.box + (((bl & 7) ^ g) << 4);
                            const uint32_t wa = lds32(qb), wb = lds32(qb + 8 * 128);
                            A[u][0] = wa & 0x0F0F0F0Fu;
                            A[u][1] = wb & 0x0F0F0F0Fu;
                            A[u][2] = (wa >> 4) & 0x0F0F0F0Fu;
                            A[u][3] = (wb >> 4) & 0x0F0F0F0Fu;
                            const uint8_t* sb = sg + (size_t)(bl >> 6) * G.box +
                                                ((((bl >> 3) & 7) ^ g) << 4) + (bl & 7) * 2;
                            dw0[u] = f16_bits_to_f32(*reinterpret_cast<const uint16_t*>(sb));
                            dw1[u] = f16_bits_to_f32(
                                *reinterpret_cast<const uint16_t*>(sb + 8 * 128));
                        }
                    }
#pragma unroll
                    for (int n = 0; n < NT; n++) {
                        if (n >= nt) continue;
                        const uint8_t* crow = act_codes + (size_t)(n * 8 + g) * CS + 4 * t;
                        const uint8_t* arow = act_aux + ((size_t)n * nb * 8 + 2 * t) * 8;
#pragma unroll
                        for (int u = 0; u < U; u++) {
                            const int kb = k0 + b0 + u * KW;
                            if (b0 + u * KW >= kcs) continue;
                            const uint8_t* cr = crow + (size_t)kb * 32;
                            const int4 ax =
                                *reinterpret_cast<const int4*>(arow + (size_t)kb * 64);
                            int d[4] = {ax.y, ax.w, ax.y, ax.w};
                            mma_u8s8(d, A[u], lds32(cr), lds32(cr + 16));
                            const float dx0 = __int_as_float(ax.x), dx1 = __int_as_float(ax.z);
                            const float p0 = dx0 * -GM_MAGIC, p1 = dx1 * -GM_MAGIC;
                            acc[n][0] = __fmaf_rn(__fmaf_rn(__int_as_float(d[0]), dx0, p0), dw0[u],
                                                  acc[n][0]);
                            acc[n][1] = __fmaf_rn(__fmaf_rn(__int_as_float(d[1]), dx1, p1), dw0[u],
                                                  acc[n][1]);
                            acc[n][2] = __fmaf_rn(__fmaf_rn(__int_as_float(d[2]), dx0, p0), dw1[u],
                                                  acc[n][2]);
                            acc[n][3] = __fmaf_rn(__fmaf_rn(__int_as_float(d[3]), dx1, p1), dw1[u],
                                                  acc[n][3]);
                        }
                    }
                }
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[s]);
            if (ks != nks - 1) continue;

            // ---- end of a band: add the kw block groups, store ----
            const int band = (int)blockIdx.x + (seq / nks) * (int)gridDim.x;
            if (kw > 1) {
#pragma unroll
                for (int n = 0; n < NT; n++)
#pragma unroll
                    for (int i = 0; i < 4; i++)
                        red[((size_t)(warp * NT + n) * 4 + i) * 32 + lane] = acc[n][i];
                consumers_sync();
            }
            if (kg == 0) {
#pragma unroll
                for (int n = 0; n < NT; n++) {
#pragma unroll
                    for (int i = 0; i < 4; i++) {
                        float v = acc[n][i];
                        for (int k = 1; k < kw; k++)
                            v = __fadd_rn(v, red[((size_t)((warp + k) * NT + n) * 4 + i) * 32 + lane]);
                        const int m = matrix_of_band(a, band);
                        const int r = (band - a.first_band[m]) * G.BH + rt * 16 + g + (i >> 1) * 8;
                        const int tok = (tile0 + n) * 8 + 2 * t + (i & 1);
                        if (n < nt && ok && r < a.rows[m] && tok < a.batch)
                            a.out[m][(size_t)tok * a.rows[m] + r] = v;
                    }
                }
            }
            if (kw > 1) consumers_sync();
#pragma unroll
            for (int n = 0; n < NT; n++) acc[n][0] = acc[n][1] = acc[n][2] = acc[n][3] = 0.0f;
        }
    }
    // A wait that gave up may leave copies in flight: let them land before the CTA's shared
    // memory is released (bounded, without the abort short-cut).
    __syncthreads();
    if (*abort_flag && tid == GM_CONSUMERS * 32) {
        (void)mbar_wait_bounded(act_bar, 0u, a.err, nullptr);
        for (int seq = issued > a.stages ? issued - a.stages : 0; seq < issued; seq++)
            (void)mbar_wait_bounded(&full[seq % a.stages], (uint32_t)(seq / a.stages) & 1u, a.err,
                                    nullptr);
    }
}

// Plan of one launch: sequences per CTA group, band height, stage size, ring depth.
struct GmPlan {
    int nt, rw, kc, stages, bands, groups, ctas;
    size_t smem;
};

int count_bands(const int* rows, int count, int bh) {
    long n = 0;
    for (int i = 0; i < count; i++) n += (rows[i] + bh - 1) / bh;
    return n > 0x7fffffffL ? 0x7fffffff : (int)n;
}

// Pass 0 looks for a plan that admits two CTAs per SM (twice the consumer warps to hide the
// latency of each block's MMA and scale steps; with several 8-sequence tiles, groups of at
// least two tiles and stages of at least 32 blocks), its ring cut to what fits in half the SM;
// pass 1 takes the largest group and the deepest ring that fit one CTA.
bool gm_plan(const int* rows, int count, int K, int batch, int num_sms, GmPlan* p) {
    const int nb = K / 32, tiles = (batch + 7) / 8;
    const size_t half = 114u * 1024u - 1024u;
    for (int pass = 0; pass < 2; pass++) {
        for (int nt = 4; nt >= 1; nt >>= 1) {
            if (nt > 1 && nt > tiles) continue;
            if (pass == 0 && tiles > 1 && nt < 2) continue;
            const int groups = (tiles + nt - 1) / nt;
            // the tallest band that still gives every SM a band
            int rw = 1;
            for (int c = GM_CONSUMERS; c > 1; c >>= 1)
                if ((long)count_bands(rows, count, 16 * c) * groups >= num_sms) {
                    rw = c;
                    break;
                }
            for (int rb = 2048; rb >= 512; rb >>= 1) {  // row-blocks per stage
                int kc = rb / (16 * rw) / 8 * 8;
                if (kc < 8) kc = 8;
                if (kc > nb) kc = nb;
                const GmGeom G = gm_geom(nt, K, rw, kc);
                const size_t fixed = 1024 + G.act_codes + G.act_aux + G.red + 256;
                const size_t limit = pass == 0 ? half : GM_SMEM_MAX;
                if (fixed + 2 * G.stage > limit) continue;
                // (pass 0 with several tiles: stages of at least 32 blocks, or the one-CTA plan)
                if (pass == 0 && tiles > 1 && kc < 32 && kc < nb) continue;
                int stages = (int)((limit - fixed) / G.stage);
                if (stages > GM_MAX_STAGES) stages = GM_MAX_STAGES;
                p->nt = nt;
                p->rw = rw;
                p->kc = kc;
                p->stages = stages;
                p->bands = count_bands(rows, count, G.BH);
                p->groups = groups;
                p->smem = fixed + (size_t)stages * G.stage;
                // CTAs per SM the shared memory admits (228 KB per SM, 1 KB reserved per CTA)
                int occ = (int)((228u * 1024u) / (p->smem + 1024));
                if (occ < 1) occ = 1;
                if (occ > 2) occ = 2;
                long ctas = ((long)num_sms * occ + groups - 1) / groups;
                if (ctas > p->bands) ctas = p->bands;
                if (ctas < 1) ctas = 1;
                p->ctas = (int)ctas;
                return true;
            }
        }
    }
    return false;
}

template <int NT, int KW>
int launch_ntkw(sulimo_ctx* ctx, const GmArgs& a, const GmMaps& maps, const GmPlan& pl) {
    static DeviceBits attr_done;
    if (!attr_done.test(ctx->device)) {
        int st = check_cuda(cudaFuncSetAttribute(gemv_mma_kernel<NT, KW>,
                                                 cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                 (int)GM_SMEM_MAX),
                            "gemv_mma smem attribute");
        if (st) return st;
        attr_done.set(ctx->device);
    }
    const cudaError_t e = launch_pdl(gemv_mma_kernel<NT, KW>, dim3((unsigned)pl.ctas, (unsigned)pl.groups),
                                     dim3(GM_THREADS), pl.smem, ctx->stream, a, maps);
    ctx->launches++;
    return check_cuda(e, "gemv_mma launch");
}

template <int NT>
int launch_nt(sulimo_ctx* ctx, const GmArgs& a, const GmMaps& maps, const GmPlan& pl) {
    switch (GM_CONSUMERS / pl.rw) {
        case 1: return launch_ntkw<NT, 1>(ctx, a, maps, pl);
        case 2: return launch_ntkw<NT, 2>(ctx, a, maps, pl);
        case 4: return launch_ntkw<NT, 4>(ctx, a, maps, pl);
        default: return launch_ntkw<NT, 8>(ctx, a, maps, pl);
    }
}

// Q8_0 block arrays [batch][nb][34] -> the staged form (one warp per block).
__global__ void __launch_bounds__(256)
    q8_stage_kernel(const uint8_t* __restrict__ src, size_t nblocks, int nb, int K,
                    int8_t* __restrict__ codes, int2* __restrict__ aux) {
    pdl_launch_dependents();
    pdl_wait_prerequisites();
    const int lane = threadIdx.x & 31;
    const size_t b = (size_t)blockIdx.x * 8 + (threadIdx.x >> 5);
    if (b >= nblocks) return;
    const size_t row = b / nb;
    const int blk = (int)(b % nb);
    const uint8_t* blkp = src + b * 34;
    const int q = (int)(int8_t)blkp[2 + lane];
    codes[row * K + (size_t)blk * 32 + lane] = (int8_t)q;
    int s = q;
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) s += __shfl_xor_sync(0xffffffffu, s, off);
    if (lane == 0) {
        const uint16_t dbits = (uint16_t)blkp[0] | ((uint16_t)blkp[1] << 8);
        aux[((row >> 3) * nb + blk) * 8 + (row & 7)] =
            make_int2(__float_as_int(f16_bits_to_f32(dbits)), 0x4B400000 - 8 * s);
    }
}

}  // namespace

size_t q8_staged_bytes(int batch, int K) {
    const size_t bp = (size_t)(batch + 7) / 8 * 8;
    return (bp * K + 255) / 256 * 256 + bp * (size_t)(K / 32) * 8;
}

Q8Out q8_staged_view(void* base, int batch, int K) {
    const size_t bp = (size_t)(batch + 7) / 8 * 8;
    uint8_t* p = reinterpret_cast<uint8_t*>(base);
    Q8Out o;
    o.aos = nullptr;
    o.codes = reinterpret_cast<int8_t*>(p);
    o.aux = reinterpret_cast<int2*>(p + (bp * K + 255) / 256 * 256);
    o.K = K;
    return o;
}

bool gemv_mma_applies(const GemvMatSrc* src, int count, int cols, int batch, int num_sms) {
    if (count < 1 || count > GM_MAX_MATS || cols <= 0 || cols % 256 || batch < 1 ||
        batch > 65535 * 8)
        return false;
    int rows[GM_MAX_MATS];
    for (int i = 0; i < count; i++) {
        if (!src[i].quants || !src[i].scales || !src[i].out || src[i].rows <= 0 ||
            ((uintptr_t)src[i].quants % 16) || ((uintptr_t)src[i].scales % 16))
            return false;
        rows[i] = src[i].rows;
    }
    GmPlan pl;
    return gm_plan(rows, count, cols, batch, num_sms, &pl);
}

int launch_gemv_mma_group(sulimo_ctx* ctx, const GemvMatSrc* src, int count, const Q8Out& x,
                          int cols, int batch, bool static_weights) {
    if (!gemv_mma_applies(src, count, cols, batch, ctx->num_sms) || !x.codes || !x.aux ||
        ((uintptr_t)x.codes % 16) || ((uintptr_t)x.aux % 16) || x.K != cols)
        return set_error(SULIMO_EINVAL, "batched tensor-core matvec does not apply to this shape");
    int rows[GM_MAX_MATS];
    for (int i = 0; i < count; i++) rows[i] = src[i].rows;
    GmPlan pl;
    gm_plan(rows, count, cols, batch, ctx->num_sms, &pl);
    const int nb = cols / 32, bh = 16 * pl.rw;
    GmArgs a;
    GmMaps maps;
    memset(&maps, 0, sizeof(maps));
    int band = 0;
    for (int i = 0; i < GM_MAX_MATS; i++) {
        const int k = i < count ? i : 0;
        a.out[i] = src[k].out;
        a.rows[i] = src[k].rows;
        a.first_band[i] = band;
        if (i >= count) continue;
        band += (src[i].rows + bh - 1) / bh;
        const uint64_t qdims[2] = {(uint64_t)nb * 16, (uint64_t)src[i].rows};
        const uint64_t qstr[1] = {(uint64_t)nb * 16};
        const uint32_t qbox[2] = {128, (uint32_t)bh};
        const uint64_t sdims[2] = {(uint64_t)nb, (uint64_t)src[i].rows};
        const uint64_t sstr[1] = {(uint64_t)nb * 2};
        const uint32_t sbox[2] = {64, (uint32_t)bh};
        int st = encode_tensor_map(&maps.q[i], CU_TENSOR_MAP_DATA_TYPE_UINT8, src[i].quants, 2,
                                   qdims, qstr, qbox, CU_TENSOR_MAP_SWIZZLE_128B);
        if (!st)
            st = encode_tensor_map(&maps.s[i], CU_TENSOR_MAP_DATA_TYPE_UINT16, src[i].scales, 2,
                                   sdims, sstr, sbox, CU_TENSOR_MAP_SWIZZLE_128B);
        if (st) return st;
    }
    a.count = count;
    a.codes = x.codes;
    a.aux = x.aux;
    a.K = cols;
    a.nb = nb;
    a.batch = batch;
    a.tiles = (batch + 7) / 8;
    a.rw = pl.rw;
    a.kc = pl.kc;
    a.stages = pl.stages;
    a.bands = pl.bands;
    a.static_weights = static_weights ? 1 : 0;
    a.err = ctx->d_error;
    switch (pl.nt) {
        case 4: return launch_nt<4>(ctx, a, maps, pl);
        case 2: return launch_nt<2>(ctx, a, maps, pl);
        default: return launch_nt<1>(ctx, a, maps, pl);
    }
}

int launch_q8_stage(sulimo_ctx* ctx, const void* x_q8, int batch, int K, const Q8Out& dst) {
    const size_t nblocks = (size_t)batch * (K / 32);
    const size_t grid = (nblocks + 7) / 8;
    if (grid > 0x7fffffffu) return set_error(SULIMO_EINVAL, "activation too large");
    const cudaError_t e = launch_pdl(q8_stage_kernel, dim3((unsigned)grid), dim3(256), 0,
                                     ctx->stream, reinterpret_cast<const uint8_t*>(x_q8), nblocks,
                                     K / 32, K, dst.codes, dst.aux);
    ctx->launches++;
    return check_cuda(e, "q8_stage launch");
}

}  // namespace sulimo
