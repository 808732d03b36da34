// gemv_q4_0_q8_0.cu — decode matvec Q4_0 (SoA) x Q8_0, bit-identical to the reference's AVX2
// kernel matvec_q4_0_q8_0_avx2 / vec_dot_q4_0_q8_0_avx2 (crates/sulimo-cpu/src/avx2.rs:113-189).
//
// The AVX2 kernel keeps eight fp32 lanes per row.  For block b, lane j holds the i32
//   s_j(b) = w[2j]x[2j] + w[2j+1]x[2j+1] + w[16+2j]x[16+2j] + w[17+2j]x[17+2j]   (w = nibble-8)
// (madd_epi16 pairs of the low and high 16-lane halves, avx2.rs:146-155) and accumulates
//   acc_j = fma(float(s_j(b)), d_w(b)*d_x(b), acc_j)          in block order (avx2.rs:158-159)
// then returns ((a0+a4)+(a1+a5)) + ((a2+a6)+(a3+a7))        (hsum_256, avx2.rs:333-342).
// s_j is an exact integer and d_w*d_x is exact in f32 (two 11-bit significands), so the only
// roundings are the FMAs and the final adds; this kernel performs exactly those, in that order.
//
// Work split (per CTA: ROWS rows of one batch vector, K processed in chunks of KB blocks):
//   stage x: the chunk's Q8_0 activation bytes are repacked into per-lane words
//            {x[2j],x[2j+1],x[16+2j],x[17+2j]} plus c_j = -8*sum(bytes) (the nibble offset);
//   phase 1: one thread per (row, block) loads the 16 quant bytes (one 128-bit load, coalesced
//            along the row) and the f16 scale, forms the 8 lane sums with dp4a and stores them
//            as f32 with d = d_w*d_x in shared memory;
//   phase 2: one thread per (row, lane) runs that lane's FMA chain over the chunk's blocks;
//   end:     the 8 lanes of a row are combined with hsum_256's tree through warp shuffles.
#include "sulimo_common.cuh"
#include "sulimo_internal.h"

namespace sulimo {
namespace {

constexpr int GEMV_THREADS = 256;
constexpr int GEMV_ROWS = 16;   // rows per CTA
constexpr int GEMV_KB = 64;     // Q4_0 blocks per K chunk
constexpr int S_STRIDE = GEMV_KB * 8 + 8;   // floats per row of lane sums (+8: bank skew)
constexpr int D_STRIDE = GEMV_KB + 1;
constexpr int ITEMS = (GEMV_ROWS * GEMV_KB + GEMV_THREADS - 1) / GEMV_THREADS;

struct __align__(16) GemvSmem {
    int xw[GEMV_KB][8];    // per-lane packed activation bytes
    int xc[GEMV_KB][8];    // -8 * sum of those bytes
    float xd[GEMV_KB];     // activation block scale
    float s[GEMV_ROWS][S_STRIDE];
    float d[GEMV_ROWS][D_STRIDE];
};

__global__ void __launch_bounds__(GEMV_THREADS)
    gemv_q4_0_q8_0_kernel(const uint16_t* __restrict__ wsc, const uint8_t* __restrict__ wq,
                          const uint8_t* __restrict__ xq8, int rows, int nb, int batch,
                          float* __restrict__ out) {
    pdl_launch_dependents();
    pdl_wait_prerequisites();
    __shared__ GemvSmem sm;
    const int tid = threadIdx.x;
    const int vec = blockIdx.x % batch;
    const int row0 = (blockIdx.x / batch) * GEMV_ROWS;
    const uint8_t* xv = xq8 + (size_t)vec * nb * 34;

    // phase-2 role: thread (r, j)
    const int pr = tid >> 3, pj = tid & 7;
    float acc = 0.0f;

    for (int c0 = 0; c0 < nb; c0 += GEMV_KB) {
        const int kbc = min(GEMV_KB, nb - c0);
        // ---- stage activations of this chunk ----
        for (int it = tid; it < kbc * 8; it += GEMV_THREADS) {
            const int b = it >> 3, j = it & 7;
            const uint16_t* blk = reinterpret_cast<const uint16_t*>(xv + (size_t)(c0 + b) * 34);
            uint32_t lo = __ldg(blk + 1 + j);      // bytes 2j, 2j+1 of qs
            uint32_t hi = __ldg(blk + 1 + 8 + j);  // bytes 16+2j, 17+2j of qs
            uint32_t w = lo | (hi << 16);
            int sum = (int)(int8_t)(w & 0xFF) + (int)(int8_t)((w >> 8) & 0xFF) +
                      (int)(int8_t)((w >> 16) & 0xFF) + (int)(int8_t)(w >> 24);
            sm.xw[b][j] = (int)w;
            sm.xc[b][j] = -8 * sum;
            if (j == 0) sm.xd[b] = f16_bits_to_f32(__ldg(blk));
        }
        __syncthreads();

        // ---- phase 1: integer lane sums, one (row, block) item per thread per step ----
        uint4 qv[ITEMS];
        uint16_t sv[ITEMS];
#pragma unroll
        for (int u = 0; u < ITEMS; u++) {
            const int item = tid + u * GEMV_THREADS;
            const int r = item / kbc, b = item - r * kbc;
            qv[u] = make_uint4(0, 0, 0, 0);
            sv[u] = 0;
            if (item < GEMV_ROWS * kbc && row0 + r < rows) {
                const size_t blk = (size_t)(row0 + r) * nb + c0 + b;
                qv[u] = __ldg(reinterpret_cast<const uint4*>(wq + blk * 16));
                sv[u] = __ldg(wsc + blk);
            }
        }
#pragma unroll
        for (int u = 0; u < ITEMS; u++) {
            const int item = tid + u * GEMV_THREADS;
            if (item < GEMV_ROWS * kbc) {
                const int r = item / kbc, b = item - r * kbc;
                const uint32_t words[4] = {qv[u].x, qv[u].y, qv[u].z, qv[u].w};
                float f[8];
#pragma unroll
                for (int w = 0; w < 4; w++) {
                    const uint32_t lo = words[w] & 0x0F0F0F0Fu;
                    const uint32_t hi = (words[w] >> 4) & 0x0F0F0F0Fu;
                    const uint32_t l0 = prmt(lo, hi, 0x5410);  // lane 2w
                    const uint32_t l1 = prmt(lo, hi, 0x7632);  // lane 2w+1
                    f[2 * w] = (float)dp4a_us(l0, (uint32_t)sm.xw[b][2 * w], sm.xc[b][2 * w]);
                    f[2 * w + 1] =
                        (float)dp4a_us(l1, (uint32_t)sm.xw[b][2 * w + 1], sm.xc[b][2 * w + 1]);
                }
                float4* dst = reinterpret_cast<float4*>(&sm.s[r][b * 8]);
                dst[0] = make_float4(f[0], f[1], f[2], f[3]);
                dst[1] = make_float4(f[4], f[5], f[6], f[7]);
                sm.d[r][b] = __fmul_rn(f16_bits_to_f32(sv[u]), sm.xd[b]);
            }
        }
        __syncthreads();

        // ---- phase 2: the lane's FMA chain over this chunk, in block order ----
        if (pr < GEMV_ROWS) {
            const float* sr = &sm.s[pr][pj];
            const float* dr = &sm.d[pr][0];
#pragma unroll 8
            for (int b = 0; b < kbc; b++) acc = __fmaf_rn(sr[b * 8], dr[b], acc);
        }
        __syncthreads();
    }

    // ---- hsum_256 tree: ((a0+a4)+(a1+a5)) + ((a2+a6)+(a3+a7)) ----
    if (tid < GEMV_ROWS * 8) {
        // all threads of the participating warps execute the shuffles
        float t = __fadd_rn(acc, __shfl_xor_sync(0xffffffffu, acc, 4));   // j<4: a_j + a_{j+4}
        float u2 = __fadd_rn(t, __shfl_xor_sync(0xffffffffu, t, 1));      // j=0: (a0+a4)+(a1+a5)
        float v = __fadd_rn(u2, __shfl_xor_sync(0xffffffffu, u2, 2));     // j=0: + ((a2+a6)+(a3+a7))
        if (pj == 0 && row0 + pr < rows) out[(size_t)vec * rows + row0 + pr] = v;
    }
}

// ---------------------------------------------------------------------------------------------
// Streaming form for K a multiple of 256 and 16-byte aligned scales (every projection of the supported models).
//
// CTA: ROWS rows (64, 32 or 16: chosen so the launch covers the SMs) x 4 threads per row
// (thread p of a row owns AVX2 lanes 2p and 2p+1, i.e. quant word p of every block) + 1 producer
// warp.  The producer streams the rows' quants and scales through a ring of TS stages of 8
// blocks with TMA (quants 128-byte swizzled, so the 4 word reads of 8 rows hit 32 distinct
// banks); the activations of NV vectors are packed into per-lane words in shared memory once
// per CTA.  Each thread keeps 2 x NV fp32 lane accumulators and applies exactly the AVX2 FMA
// sequence; the row's 8 lanes are combined with hsum_256's tree through shuffles inside the
// 4-thread group.  One launch can cover up to three matrices that share the activations (the
// decode step's q/k/v and gate/up projections): the CTA index picks the matrix.
constexpr int TS_BLOCKS = 8;                     // Q4_0 blocks per stage (K = 256)
constexpr int TS_MAX_MATS = 3;

// Shared memory: the stages' quant tiles first (each ROWS x 128 bytes, a multiple of the
// 1024-byte swizzle atom, so every tile starts on an atom), then the stages' scale tiles.
// Ring depth: 8 stages of 64 rows; narrower tiles get proportionally more stages so every CTA
// keeps the same ~72 KB of weights in flight (the small decode matrices are latency-bound).
template <int ROWS>
struct TsShape {
    static constexpr int THREADS = ROWS * 4 + 32;  // + producer warp
    static constexpr int STAGES = 8 * 64 / ROWS;
    static constexpr uint32_t Q_BYTES = ROWS * TS_BLOCKS * 16;
    static constexpr uint32_t S_BYTES = ROWS * TS_BLOCKS * 2;
    static constexpr uint32_t STAGE_BYTES = Q_BYTES + S_BYTES;
    static_assert(Q_BYTES % 1024 == 0, "swizzled quant tiles must start on 1024-byte atoms");
};

struct GemvMat {
    CUtensorMap q, s;  // quants [rows][nb*16] (128-byte swizzle), scales [rows][nb] (u16)
    float* out;        // [batch][rows]
    int rows, tile0;   // first CTA (x) index of this matrix
};

struct GemvGroup {
    GemvMat m[TS_MAX_MATS];
    int count;
};

// exact int -> float for |s| < 2^22: 1.5*2^23 + s has an integer ulp
__device__ __forceinline__ float small_int_to_float(int s) {
    return __fsub_rn(__int_as_float(0x4B400000 + s), 12582912.0f);
}

template <int NV, int ROWS>
__global__ void __launch_bounds__(TsShape<ROWS>::THREADS)
    gemv_q4_0_q8_0_tma_kernel(const __grid_constant__ GemvGroup grp,
                              const uint8_t* __restrict__ xq8, int nb, int batch,
                              int static_weights, int* __restrict__ err) {
    using T = TsShape<ROWS>;
    pdl_launch_dependents();
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    const uint32_t raw = smem_u32(smem_raw);
    uint8_t* sm = smem_raw + ((1024u - (raw & 1023u)) & 1023u);
    uint8_t* qtiles = sm;                                   // T::STAGES x Q_BYTES
    uint8_t* stiles = sm + T::STAGES * T::Q_BYTES;          // T::STAGES x S_BYTES
    uint64_t* full = reinterpret_cast<uint64_t*>(sm + T::STAGES * T::STAGE_BYTES);
    uint64_t* empty = full + T::STAGES;
    volatile int* abort_flag = reinterpret_cast<volatile int*>(empty + T::STAGES);
    int* xw = reinterpret_cast<int*>(empty + T::STAGES + 1);        // [NV][nb][8]
    int* xc = xw + NV * nb * 8;                                      // [NV][nb][8]
    float* xs = reinterpret_cast<float*>(xc + NV * nb * 8);          // [NV][nb]

    int mi = 0;
#pragma unroll
    for (int i = 1; i < TS_MAX_MATS; i++)
        if (i < grp.count && (int)blockIdx.x >= grp.m[i].tile0) mi = i;
    const GemvMat& M = grp.m[mi];
    const int rows = M.rows;
    const int tid = threadIdx.x;
    const int row0 = ((int)blockIdx.x - M.tile0) * ROWS;
    const int v0 = blockIdx.y * NV;
    const int nchunks = nb / TS_BLOCKS;

    // The producer thread sets up the ring.  When the caller vouches that the weights are not
    // written by the previous kernel of the stream (a decode step's static parameters), it also
    // issues the first ring pass of weight tiles before griddepcontrol.wait, so the weight
    // stream overlaps the previous kernel's tail; everything else (and always the
    // activations) is read only after the wait.
    int prefetched = 0;
    if (tid == ROWS * 4) {
        for (int s = 0; s < T::STAGES; s++) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], ROWS * 4);
        }
        *abort_flag = 0;
        fence_barrier_init();
        prefetch_tensormap(&M.q);
        prefetch_tensormap(&M.s);
        if (static_weights) {
            for (int c = 0; c < nchunks && c < T::STAGES; c++) {
                mbar_arrive_expect_tx(&full[c], T::STAGE_BYTES);
                tma_load_2d(qtiles + c * T::Q_BYTES, &M.q, c * TS_BLOCKS * 16, row0, &full[c]);
                tma_load_2d(stiles + c * T::S_BYTES, &M.s, c * TS_BLOCKS, row0, &full[c]);
            }
            prefetched = nchunks < T::STAGES ? nchunks : T::STAGES;
        }
    }
    pdl_wait_prerequisites();
    __syncthreads();

    if (tid >= ROWS * 4) {
        // ------------------------------ producer warp ------------------------------
        if (tid == ROWS * 4) {
            int issued = prefetched;
            for (int c = prefetched; c < nchunks; c++) {
                const int s = c % T::STAGES;
                const uint32_t ph = (uint32_t)(c / T::STAGES) & 1u;
                if (!mbar_wait_bounded(&empty[s], ph ^ 1u, err, abort_flag)) break;
                mbar_arrive_expect_tx(&full[s], T::STAGE_BYTES);
                tma_load_2d(qtiles + s * T::Q_BYTES, &M.q, c * TS_BLOCKS * 16, row0, &full[s]);
                tma_load_2d(stiles + s * T::S_BYTES, &M.s, c * TS_BLOCKS, row0, &full[s]);
                issued = c + 1;
            }
            if (*abort_flag)  // the issued copies must land before the CTA releases its smem
                for (int c = (issued > T::STAGES ? issued - T::STAGES : 0); c < issued; c++)
                    mbar_wait_bounded(&full[c % T::STAGES], (uint32_t)(c / T::STAGES) & 1u, err,
                                      nullptr);
        }
        return;  // the consumers synchronize among themselves (named barrier 1) from here on
    }

    // ---- pack the activations: lane j of block b -> {x[2j],x[2j+1],x[16+2j],x[17+2j]} ----
    for (int it = tid; it < NV * nb * 8; it += ROWS * 4) {
        const int v = it / (nb * 8), rem = it - v * nb * 8;
        const int b = rem >> 3, j = rem & 7;
        uint32_t w = 0;
        float d = 0.0f;
        if (v0 + v < batch) {
            const uint16_t* blk =
                reinterpret_cast<const uint16_t*>(xq8 + ((size_t)(v0 + v) * nb + b) * 34);
            w = (uint32_t)__ldg(blk + 1 + j) | ((uint32_t)__ldg(blk + 9 + j) << 16);
            if (j == 0) d = f16_bits_to_f32(__ldg(blk));
        }
        const int sum = (int)(int8_t)(w & 0xFF) + (int)(int8_t)((w >> 8) & 0xFF) +
                        (int)(int8_t)((w >> 16) & 0xFF) + (int)(int8_t)(w >> 24);
        xw[it] = (int)w;
        xc[it] = -8 * sum;
        if (j == 0) xs[v * nb + b] = d;
    }
    asm volatile("bar.sync 1, %0;" ::"r"(ROWS * 4) : "memory");  // consumers only

    const int rl = tid >> 2, p = tid & 3;
    float acc[NV][2];
#pragma unroll
    for (int v = 0; v < NV; v++) acc[v][0] = acc[v][1] = 0.0f;

    for (int c = 0; c < nchunks; c++) {
        const int s = c % T::STAGES;
        const uint32_t ph = (uint32_t)(c / T::STAGES) & 1u;
        if (!mbar_wait_bounded(&full[s], ph, err, abort_flag)) break;
        const uint8_t* qst = qtiles + s * T::Q_BYTES + rl * 128;
        const uint16_t* sst = reinterpret_cast<const uint16_t*>(stiles + s * T::S_BYTES) + rl * 8;
#pragma unroll
        for (int b = 0; b < TS_BLOCKS; b++) {
            const int kb = c * TS_BLOCKS + b;
            // 128-byte swizzle: the 16-byte chunk b of row rl sits at chunk b ^ (rl & 7)
            const uint32_t word =
                *reinterpret_cast<const uint32_t*>(qst + ((b ^ (rl & 7)) << 4) + p * 4);
            const float dw = f16_bits_to_f32(sst[b]);
            const uint32_t lo = word & 0x0F0F0F0Fu;
            const uint32_t hi = (word >> 4) & 0x0F0F0F0Fu;
            const uint32_t l0 = prmt(lo, hi, 0x5410);  // lane 2p
            const uint32_t l1 = prmt(lo, hi, 0x7632);  // lane 2p+1
#pragma unroll
            for (int v = 0; v < NV; v++) {
                const int2 xv = *reinterpret_cast<const int2*>(xw + (v * nb + kb) * 8 + 2 * p);
                const int2 cv = *reinterpret_cast<const int2*>(xc + (v * nb + kb) * 8 + 2 * p);
                const float d = __fmul_rn(dw, xs[v * nb + kb]);
                acc[v][0] = __fmaf_rn(small_int_to_float(dp4a_us(l0, (uint32_t)xv.x, cv.x)), d,
                                      acc[v][0]);
                acc[v][1] = __fmaf_rn(small_int_to_float(dp4a_us(l1, (uint32_t)xv.y, cv.y)), d,
                                      acc[v][1]);
            }
        }
        mbar_arrive(&empty[s]);
    }

    // hsum_256: ((a0+a4)+(a1+a5)) + ((a2+a6)+(a3+a7)); thread p holds lanes 2p, 2p+1
    const int row = row0 + rl;
#pragma unroll
    for (int v = 0; v < NV; v++) {
        const float u0 = __fadd_rn(acc[v][0], __shfl_xor_sync(0xffffffffu, acc[v][0], 2));
        const float u1 = __fadd_rn(acc[v][1], __shfl_xor_sync(0xffffffffu, acc[v][1], 2));
        const float w = __fadd_rn(u0, u1);
        const float r = __fadd_rn(w, __shfl_xor_sync(0xffffffffu, w, 1));
        if (p == 0 && row < rows && v0 + v < batch && !*abort_flag)
            M.out[(size_t)(v0 + v) * rows + row] = r;
    }
}

template <int NV, int ROWS>
size_t gemv_tma_smem(int nb) {
    using T = TsShape<ROWS>;
    return 1024 + (size_t)T::STAGES * T::STAGE_BYTES + 8 * (2 * T::STAGES + 1) +
           (size_t)NV * nb * (8 * 4 * 2 + 4);
}

template <int NV, int ROWS>
int launch_gemv_tma(sulimo_ctx* ctx, const GemvGroup& grp, int tiles, const uint8_t* xq8, int nb,
                    int batch, int static_weights) {
    const size_t smem = gemv_tma_smem<NV, ROWS>(nb);
    static DeviceBits done;  // per device
    if (!done.test(ctx->device)) {
        int st = check_cuda(cudaFuncSetAttribute(gemv_q4_0_q8_0_tma_kernel<NV, ROWS>,
                                                 cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                 227 * 1024),
                            "gemv smem attribute");
        if (st) return st;
        done.set(ctx->device);
    }
    dim3 grid((unsigned)tiles, (batch + NV - 1) / NV);
    (void)launch_pdl(gemv_q4_0_q8_0_tma_kernel<NV, ROWS>, grid, dim3(TsShape<ROWS>::THREADS), smem,
                     ctx->stream, grp, xq8, nb, batch, static_weights, ctx->d_error);
    ctx->launches++;
    return check_cuda(cudaGetLastError(), "gemv_q4_0_q8_0_tma launch");
}

template <int ROWS>
int launch_gemv_tma_rows(sulimo_ctx* ctx, GemvGroup& grp, const GemvMatSrc* src, int count,
                         const uint8_t* xq8, int nb, int batch, int nv, int sw) {
    int tiles = 0;
    for (int i = 0; i < count; i++) {
        GemvMat& M = grp.m[i];
        const uint64_t qd[2] = {(uint64_t)nb * 16, (uint64_t)src[i].rows};
        const uint64_t qs[1] = {(uint64_t)nb * 16};
        const uint32_t qb[2] = {TS_BLOCKS * 16, (uint32_t)ROWS};
        int st = encode_tensor_map(&M.q, CU_TENSOR_MAP_DATA_TYPE_UINT8, src[i].quants, 2, qd, qs,
                                   qb, CU_TENSOR_MAP_SWIZZLE_128B);
        if (st) return st;
        const uint64_t sd[2] = {(uint64_t)nb, (uint64_t)src[i].rows};
        const uint64_t ss[1] = {(uint64_t)nb * 2};
        const uint32_t sbx[2] = {TS_BLOCKS, (uint32_t)ROWS};
        st = encode_tensor_map(&M.s, CU_TENSOR_MAP_DATA_TYPE_UINT16, src[i].scales, 2, sd, ss, sbx,
                               CU_TENSOR_MAP_SWIZZLE_NONE);
        if (st) return st;
        M.out = src[i].out;
        M.rows = src[i].rows;
        M.tile0 = tiles;
        tiles += (src[i].rows + ROWS - 1) / ROWS;
    }
    for (int i = count; i < TS_MAX_MATS; i++) grp.m[i] = grp.m[0];
    grp.count = count;
    switch (nv) {
        case 8: return launch_gemv_tma<8, ROWS>(ctx, grp, tiles, xq8, nb, batch, sw);
        case 4: return launch_gemv_tma<4, ROWS>(ctx, grp, tiles, xq8, nb, batch, sw);
        case 2: return launch_gemv_tma<2, ROWS>(ctx, grp, tiles, xq8, nb, batch, sw);
        default: return launch_gemv_tma<1, ROWS>(ctx, grp, tiles, xq8, nb, batch, sw);
    }
}

}  // namespace

// Streams 1..3 matrices of the same K against the same activations in one launch; false when
// the streaming form does not apply (K not a multiple of 256, scales not 16-byte aligned,
// activations too large for shared memory).
int launch_gemv_group(sulimo_ctx* ctx, const GemvMatSrc* src, int count, const void* x_q8,
                      int cols, int batch, bool* handled, bool static_weights) {
    *handled = false;
    const int nb = cols / 32;
    if (count < 1 || count > TS_MAX_MATS || nb % TS_BLOCKS != 0) return SULIMO_OK;
    int total_rows = 0;
    for (int i = 0; i < count; i++) {
        if (((uintptr_t)src[i].scales % 16) != 0 || src[i].rows <= 0) return SULIMO_OK;
        total_rows += src[i].rows;
    }
    int nv = 8;  // vectors per weight pass: <= batch, packed activations <= 96 KB
    while (nv > 1 && (nv > batch || (size_t)nv * nb * 68 > 96 * 1024)) nv >>= 1;
    if ((size_t)nv * nb * 68 > 96 * 1024) return SULIMO_OK;
    *handled = true;
    const int sw = static_weights ? 1 : 0;
    // rows per CTA: 64 unless that leaves more than half of the SMs idle (measured: 32-row
    // tiles make the one-wave 8960-row config-1 matvec ~1.4x slower, so narrower tiles only
    // serve the small decode matrices)
    const int vec_groups = (batch + nv - 1) / nv;
    const uint8_t* x = reinterpret_cast<const uint8_t*>(x_q8);
    GemvGroup grp;
    const size_t half_sms = (size_t)ctx->num_sms / 2;
    if ((size_t)(total_rows / 64) * vec_groups >= half_sms)
        return launch_gemv_tma_rows<64>(ctx, grp, src, count, x, nb, batch, nv, sw);
    if ((size_t)(total_rows / 32) * vec_groups >= half_sms)
        return launch_gemv_tma_rows<32>(ctx, grp, src, count, x, nb, batch, nv, sw);
    return launch_gemv_tma_rows<16>(ctx, grp, src, count, x, nb, batch, nv, sw);
}

int launch_gemv_static(sulimo_ctx* ctx, const void* w_scales, const void* w_quants,
                       const void* x_q8, int rows, int cols, int batch, float* out) {
    const GemvMatSrc src = {w_scales, w_quants, out, rows};
    bool handled = false;
    const int st = launch_gemv_group(ctx, &src, 1, x_q8, cols, batch, &handled, true);
    if (handled || st) return st;
    return launch_gemv_q4_0_q8_0(ctx, w_scales, w_quants, x_q8, rows, cols, batch, out);
}

int launch_gemv_q4_0_q8_0(sulimo_ctx* ctx, const void* w_scales, const void* w_quants,
                          const void* x_q8, int rows, int cols, int batch, float* out) {
    const int nb = cols / 32;
    const GemvMatSrc src = {w_scales, w_quants, out, rows};
    bool handled = false;
    const int st = launch_gemv_group(ctx, &src, 1, x_q8, cols, batch, &handled, false);
    if (handled || st) return st;
    const size_t tiles = ((size_t)rows + GEMV_ROWS - 1) / GEMV_ROWS;
    const size_t grid = tiles * (size_t)batch;
    if (grid > 0x7fffffffu) return set_error(SULIMO_EINVAL, "gemv grid too large");
    (void)launch_pdl(gemv_q4_0_q8_0_kernel, dim3((unsigned)grid), dim3(GEMV_THREADS), 0,
                     ctx->stream, reinterpret_cast<const uint16_t*>(w_scales),
                     reinterpret_cast<const uint8_t*>(w_quants),
                     reinterpret_cast<const uint8_t*>(x_q8), rows, nb, batch, out);
    ctx->launches++;
    return check_cuda(cudaGetLastError(), "gemv_q4_0_q8_0 launch");
}

}  // namespace sulimo
