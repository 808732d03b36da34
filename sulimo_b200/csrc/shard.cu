// shard.cu — layout kernel of the row-sharded projection (multi-GPU).
//
// A Q4_0 projection [F][K] is split into `world` contiguous row (feature) ranges of `fs` rows
// (the last one may be shorter); rank r computes Y_r = X W_r^T as [M][fs] and an all-gather
// (NCCL) concatenates the ranks' results shard-major: G[world][M][fs].  unshard_rows_kernel
// writes the row-major Y[M][F] the single-GPU GEMM produces: Y[t][r*fs + j] = G[r][t][j] for
// j < rows of shard r.  Memory-bound; 16-byte copies when every row segment is 16-byte aligned,
// element copies otherwise.
#include "sulimo_common.cuh"
#include "sulimo_internal.h"

namespace sulimo {
namespace {

// One CTA row per (token t, shard r); threads stride over the shard's row segment.
template <typename V>
__global__ void __launch_bounds__(256)
    unshard_rows_kernel(const V* __restrict__ g, V* __restrict__ y, int world, int m_tokens,
                        size_t fs_v, size_t f_v, size_t last_v) {
    pdl_launch_dependents();
    pdl_wait_prerequisites();
    const int t = blockIdx.x, r = blockIdx.y;
    const size_t len = (r == world - 1) ? last_v : fs_v;
    const V* src = g + ((size_t)r * m_tokens + t) * fs_v;
    V* dst = y + (size_t)t * f_v + (size_t)r * fs_v;
    for (size_t j = threadIdx.x; j < len; j += blockDim.x) dst[j] = src[j];
}

}  // namespace

int launch_unshard_rows(sulimo_ctx* ctx, const void* gathered, void* out, int world,
                        int m_tokens, size_t fs, size_t f, int elem_size) {
    const size_t last = f - (size_t)(world - 1) * fs;
    const size_t fs_b = fs * elem_size, f_b = f * elem_size, last_b = last * elem_size;
    const bool v16 = fs_b % 16 == 0 && f_b % 16 == 0 && last_b % 16 == 0 &&
                     (uintptr_t)gathered % 16 == 0 && (uintptr_t)out % 16 == 0;
    dim3 grid((unsigned)m_tokens, (unsigned)world);
    cudaError_t e;
    if (v16)
        e = launch_pdl(unshard_rows_kernel<uint4>, grid, dim3(256), 0, ctx->stream,
                       reinterpret_cast<const uint4*>(gathered), reinterpret_cast<uint4*>(out),
                       world, m_tokens, fs_b / 16, f_b / 16, last_b / 16);
    else if (elem_size == 4)
        e = launch_pdl(unshard_rows_kernel<uint32_t>, grid, dim3(256), 0, ctx->stream,
                       reinterpret_cast<const uint32_t*>(gathered),
                       reinterpret_cast<uint32_t*>(out), world, m_tokens, fs, f, last);
    else
        e = launch_pdl(unshard_rows_kernel<uint16_t>, grid, dim3(256), 0, ctx->stream,
                       reinterpret_cast<const uint16_t*>(gathered),
                       reinterpret_cast<uint16_t*>(out), world, m_tokens, fs, f, last);
    ctx->launches++;
    return check_cuda(e, "unshard_rows launch");
}

}  // namespace sulimo
