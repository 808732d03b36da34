// repack_q4_0.cu — GGUF Q4_0 blocks (array of structures) to the SoA layout every kernel of this
// library reads, on the device.
//
// repack_q4_0_aos_to_soa (crates/sulimo-core/src/repack.rs:45-81): block b of the source is 18
// bytes, [d: f16][qs: 16 bytes]; it becomes scales[b] (2 bytes) and quants[16 b .. 16 b + 16].
// The reference repacks on the host at load time; here a model file's tensor data, copied to the
// device as it lies in the file, is repacked there (no host pass over the weights).
// HBM-bound: 18 bytes read and 18 written per block.  A CTA stages 256 consecutive blocks
// (4608 bytes) through shared memory with 16-byte loads when the source is 16-byte aligned (the
// block stream's own alignment is 2), then writes each block's quants as one 16-byte store and
// its scale as one 2-byte store.
#include "sulimo_common.cuh"
#include "sulimo_internal.h"

namespace sulimo {
namespace {

constexpr int RP_THREADS = 256;  // one block per thread
constexpr int RP_BYTES = RP_THREADS * 18;

__global__ void __launch_bounds__(RP_THREADS)
    repack_q4_0_kernel(const uint8_t* __restrict__ src, size_t nblocks, bool src16,
                       uint16_t* __restrict__ scales, uint8_t* __restrict__ quants) {
    // No griddepcontrol.launch_dependents: the GEMMs and matvecs read their weights before
    // their own programmatic wait, so the kernel that writes weights lets its dependents start
    // only when it has completed.
    pdl_wait_prerequisites();
    __shared__ __align__(16) uint8_t tile[RP_BYTES];
    const size_t b0 = (size_t)blockIdx.x * RP_THREADS;
    const size_t nb = min((size_t)RP_THREADS, nblocks - b0);
    const uint8_t* s = src + b0 * 18;
    const size_t bytes = nb * 18;
    if (src16) {
        // the tile's start is 16-byte aligned when src is (4608 = 288 * 16)
        const size_t n16 = bytes / 16;
        for (size_t i = threadIdx.x; i < n16; i += RP_THREADS)
            reinterpret_cast<uint4*>(tile)[i] = __ldg(reinterpret_cast<const uint4*>(s) + i);
        for (size_t i = n16 * 16 + threadIdx.x; i < bytes; i += RP_THREADS) tile[i] = s[i];
    } else {
        for (size_t i = threadIdx.x; i < bytes / 2; i += RP_THREADS)
            reinterpret_cast<uint16_t*>(tile)[i] = __ldg(reinterpret_cast<const uint16_t*>(s) + i);
    }
    __syncthreads();
    if ((size_t)threadIdx.x < nb) {
        const uint8_t* blk = tile + threadIdx.x * 18;
        const uint16_t* w = reinterpret_cast<const uint16_t*>(blk);  // 18-byte blocks: 2-aligned
        scales[b0 + threadIdx.x] = w[0];
        uint4 q;
        q.x = (uint32_t)w[1] | ((uint32_t)w[2] << 16);
        q.y = (uint32_t)w[3] | ((uint32_t)w[4] << 16);
        q.z = (uint32_t)w[5] | ((uint32_t)w[6] << 16);
        q.w = (uint32_t)w[7] | ((uint32_t)w[8] << 16);
        reinterpret_cast<uint4*>(quants)[b0 + threadIdx.x] = q;
    }
}

}  // namespace

int launch_repack_q4_0(sulimo_ctx* ctx, const void* src_aos, size_t nblocks, void* dst_scales,
                       void* dst_quants) {
    if (nblocks == 0) return SULIMO_OK;
    const size_t grid = (nblocks + RP_THREADS - 1) / RP_THREADS;
    if (grid > 0x7fffffffu) return set_error(SULIMO_EINVAL, "too many blocks");
    const bool src16 = ((uintptr_t)src_aos % 16) == 0;
    const cudaError_t e =
        launch_pdl(repack_q4_0_kernel, dim3((unsigned)grid), dim3(RP_THREADS), 0, ctx->stream,
                   reinterpret_cast<const uint8_t*>(src_aos), nblocks, src16,
                   reinterpret_cast<uint16_t*>(dst_scales), reinterpret_cast<uint8_t*>(dst_quants));
    ctx->launches++;
    return check_cuda(e, "repack_q4_0 launch");
}

}  // namespace sulimo
