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

}  // namespace

int launch_gemv_q4_0_q8_0(sulimo_ctx* ctx, const void* w_scales, const void* w_quants,
                          const void* x_q8, int rows, int cols, int batch, float* out) {
    const int nb = cols / 32;
    const size_t tiles = ((size_t)rows + GEMV_ROWS - 1) / GEMV_ROWS;
    const size_t grid = tiles * (size_t)batch;
    if (grid > 0x7fffffffu) return set_error(SULIMO_EINVAL, "gemv grid too large");
    gemv_q4_0_q8_0_kernel<<<(unsigned)grid, GEMV_THREADS, 0, ctx->stream>>>(
        reinterpret_cast<const uint16_t*>(w_scales), reinterpret_cast<const uint8_t*>(w_quants),
        reinterpret_cast<const uint8_t*>(x_q8), rows, nb, batch, out);
    ctx->launches++;
    return check_cuda(cudaGetLastError(), "gemv_q4_0_q8_0 launch");
}

}  // namespace sulimo
