// matvec_dense.cu — the F32 / F16 branches of the decode matvec.
//
// apply_matvec (crates/sulimo-engine/src/forward_pass.rs:509-527) routes a Q4_0 tensor to the
// Q4_0 x Q8_0 matvec and a raw F32 or F16 tensor to dispatch_matvec_f32 / dispatch_matvec_f16
// (crates/sulimo-cpu/src/avx2.rs:72-104), whose AVX2 kernels (avx2.rs:259-331) compute, per
// row r, eight fp32 lanes acc_j = fma(w[r][8c + j], x[8c + j], acc_j) over c = 0 .. cols/8 - 1
// in order, reduce them with hsum_256 ((a0 + a4) + (a1 + a5)) + ((a2 + a6) + (a3 + a7)), then
// add the tail columns cols/8*8 .. cols-1 one by one (multiply, then add).  The F16 kernel
// widens the weights with F16C (exact).
//
// Here eight threads carry a row's eight lanes with the same FMA chains, and the add tree is
// the same, so every output is bit-identical to the reference's AVX2 kernel.  Batched: each
// weight load serves NV activation vectors.  HBM-bound (rows * cols * sizeof(W) bytes); the
// chains are long but every row is independent.
#include "sulimo_common.cuh"
#include "sulimo_internal.h"

namespace sulimo {
namespace {

constexpr int MVD_THREADS = 256;  // 32 rows per CTA

__device__ __forceinline__ float widen(float v) { return v; }
__device__ __forceinline__ float widen(__half v) { return __half2float(v); }

template <typename W, int NV>
__global__ void __launch_bounds__(MVD_THREADS)
    matvec_dense_kernel(const W* __restrict__ w, const float* __restrict__ x, int rows, int cols,
                        int batch, int v0, float* __restrict__ out) {
    pdl_launch_dependents();
    pdl_wait_prerequisites();
    const int t = blockIdx.x * MVD_THREADS + threadIdx.x;
    const int row = t >> 3, j = t & 7;
    const bool live = row < rows;
    const int chunks = cols >> 3;
    const W* wr = w + (size_t)(live ? row : 0) * cols;
    float acc[NV];
#pragma unroll
    for (int v = 0; v < NV; v++) acc[v] = 0.0f;
    if (live) {
#pragma unroll 4
        for (int c = 0; c < chunks; c++) {
            const float wv = widen(wr[8 * c + j]);
#pragma unroll
            for (int v = 0; v < NV; v++)
                if (v0 + v < batch)
                    acc[v] = __fmaf_rn(wv, __ldg(x + (size_t)(v0 + v) * cols + 8 * c + j), acc[v]);
        }
    }
    // hsum_256: lane j + lane j^4, then pairs (0,1) (2,3), then the two halves
#pragma unroll
    for (int v = 0; v < NV; v++) {
        float s = acc[v];
        s = __fadd_rn(s, __shfl_xor_sync(0xffffffffu, s, 4));
        s = __fadd_rn(s, __shfl_xor_sync(0xffffffffu, s, 1));
        s = __fadd_rn(s, __shfl_xor_sync(0xffffffffu, s, 2));
        if (live && j == 0 && v0 + v < batch) {
            const float* xv = x + (size_t)(v0 + v) * cols;
            for (int c = chunks * 8; c < cols; c++) s = __fadd_rn(s, __fmul_rn(widen(wr[c]), xv[c]));
            out[(size_t)(v0 + v) * rows + row] = s;
        }
    }
}

template <typename W>
int launch_dense(sulimo_ctx* ctx, const W* w, const float* x, int rows, int cols, int batch,
                 float* out) {
    const unsigned grid = (unsigned)(((size_t)rows * 8 + MVD_THREADS - 1) / MVD_THREADS);
    for (int v0 = 0; v0 < batch; v0 += 4) {
        cudaError_t e = batch - v0 >= 4 || batch - v0 == 3
                            ? launch_pdl(matvec_dense_kernel<W, 4>, dim3(grid), dim3(MVD_THREADS), 0,
                                         ctx->stream, w, x, rows, cols, batch, v0, out)
                            : launch_pdl(matvec_dense_kernel<W, 2>, dim3(grid), dim3(MVD_THREADS), 0,
                                         ctx->stream, w, x, rows, cols, batch, v0, out);
        ctx->launches++;
        int st = check_cuda(e, "matvec_dense launch");
        if (st) return st;
    }
    return SULIMO_OK;
}

}  // namespace

int launch_matvec_dense(sulimo_ctx* ctx, int wtype, const void* w, const float* x, int rows,
                        int cols, int batch, float* out) {
    if (wtype == SULIMO_GGML_F32)
        return launch_dense(ctx, reinterpret_cast<const float*>(w), x, rows, cols, batch, out);
    return launch_dense(ctx, reinterpret_cast<const __half*>(w), x, rows, cols, batch, out);
}

}  // namespace sulimo
