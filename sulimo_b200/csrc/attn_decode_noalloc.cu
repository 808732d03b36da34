// attn_decode_noalloc.cu — decode attention for callers that may not allocate device memory.
//
// The regular entry point (sulimo_cuda_attn_decode_q8_0) keeps its split-K partial results in a
// per-context workspace that it grows with cudaMalloc the first time a larger problem arrives.
// Some callers cannot let that happen:
//   - a decode loop run under a no-allocation rule.  Sulimo's CPU decode step is built to make
//     zero heap allocations per token (its forward pass keeps every buffer in pre-sized
//     scratch); an engine carrying that rule over to the GPU cannot have a library call
//     cudaMalloc in the middle of a token, where the allocation would also stall the stream;
//   - hosts whose device memory is planned up front.  Sulimo sizes one fixed arena from a memory
//     budget before loading; a caller working from such a plan has no room for allocations the
//     library makes on its own.
// This entry point keeps the partials in a fixed array compiled into the library instead.  The
// array is a file-scope __device__ variable, so every GPU that loads the library reserves it
// (ATTN_NOALLOC_SCRATCH_BYTES) until the process exits, whether or not it is used.
#include <mutex>
#include <string>

#include "sulimo_common.cuh"
#include "sulimo_internal.h"

namespace {

constexpr size_t ATTN_NOALLOC_SCRATCH_FLOATS = (size_t)1 << 19;  // 2 MiB of fp32 partials

static __device__ __align__(256) float g_attn_noalloc_scratch[ATTN_NOALLOC_SCRATCH_FLOATS];

// Host code cannot use the array's name as a device address: the name is a host-side stand-in.
// The device address is looked up once per device (with that device current) and cached.
std::mutex g_scratch_mu;
float* g_scratch_ptr[64] = {};

int scratch_for_device(int device, float** out) {
    if (device < 0 || device >= 64) return sulimo::set_error(SULIMO_ENODEV, "device index >= 64");
    std::lock_guard<std::mutex> lock(g_scratch_mu);
    if (!g_scratch_ptr[device]) {
        void* p = nullptr;
        cudaError_t e = cudaGetSymbolAddress(&p, g_attn_noalloc_scratch);
        if (e != cudaSuccess) return sulimo::check_cuda(e, "cudaGetSymbolAddress(attention scratch)");
        g_scratch_ptr[device] = reinterpret_cast<float*>(p);
    }
    *out = g_scratch_ptr[device];
    return SULIMO_OK;
}

bool aligned_to(const void* p, size_t a) { return ((uintptr_t)p % a) == 0; }

}  // namespace

extern "C" int sulimo_cuda_attn_decode_q8_0_noalloc(sulimo_ctx* ctx, const float* q,
                                                    const void* k_ring, const void* v_ring,
                                                    size_t seq_stride_bytes, size_t capacity,
                                                    size_t context_len, int head_count,
                                                    int head_count_kv, int head_dim, int batch,
                                                    float softcap, float* out) {
    using sulimo::set_error;
    if (!ctx) return set_error(SULIMO_EINVAL, "null context");
    if (head_count <= 0 || head_count_kv <= 0 || head_count % head_count_kv != 0)
        return set_error(SULIMO_EINVAL, "head_count must be a positive multiple of head_count_kv");
    if (head_dim <= 0 || head_dim % 32 != 0 || head_dim > 256)
        return set_error(SULIMO_EINVAL, "head_dim must be a multiple of 32 in [32, 256]");
    if (head_count / head_count_kv > 8)
        return set_error(SULIMO_EINVAL, "at most 8 query heads per KV head");
    if (batch < 0 || capacity == 0) return set_error(SULIMO_EINVAL, "bad batch / capacity");
    if (batch == 0) return SULIMO_OK;
    if (!q || !k_ring || !v_ring || !out) return set_error(SULIMO_EINVAL, "null pointer");
    if (!aligned_to(q, 16) || !aligned_to(out, 16) || !aligned_to(k_ring, 2) ||
        !aligned_to(v_ring, 2) || seq_stride_bytes % 2 != 0)
        return set_error(SULIMO_EALIGN, "q/out 16-byte aligned, rings 2-byte aligned");

    // Fit the split count to the fixed scratch: fewer splits than the workspace path would
    // pick when needed, never fewer than the kernel's minimum (256 positions per split).
    int min_splits = 1, splits = 1;
    sulimo::attn_decode_split_range(context_len, head_count_kv, batch, ctx->num_sms, &min_splits,
                                    &splits);
    const size_t per_split = (size_t)batch * head_count * (head_dim + 2);
    const size_t fit = ATTN_NOALLOC_SCRATCH_FLOATS / per_split;
    if (fit < (size_t)min_splits)
        return set_error(SULIMO_EINVAL,
                         "problem too large for the fixed attention scratch: needs " +
                             std::to_string(per_split * min_splits) + " floats (batch * heads * " +
                             "ceil(context_len / 256) * (head_dim + 2)), limit " +
                             std::to_string(ATTN_NOALLOC_SCRATCH_FLOATS));
    if ((size_t)splits > fit) splits = (int)fit;
    if (splits < min_splits) splits = min_splits;

    cudaError_t e = cudaSetDevice(ctx->device);
    if (e != cudaSuccess) return sulimo::check_cuda(e, "cudaSetDevice");
    float* scratch = nullptr;
    int st = scratch_for_device(ctx->device, &scratch);
    if (st) return st;
    return sulimo::launch_attn_decode_with_splits(ctx, q, k_ring, v_ring, seq_stride_bytes,
                                                  capacity, context_len, head_count,
                                                  head_count_kv, head_dim, batch, softcap, out,
                                                  scratch, splits);
}
