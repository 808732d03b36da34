// q8_0.cu — Q8_0 quantization, Q8_0 KV-ring store, Q4_0 row dequant and integer block sums.
//
// All of these are byte/bit-exact restatements of the reference's CPU functions:
//   quantize_f32_to_q8_0      crates/sulimo-core/src/kv_cache.rs:162-192
//   KvCache::store_key/value  kv_cache.rs:93-110, GPU writer kv_store_q8_0 kernels/prefill.cl:72-116
//   dequantize_q4_0_soa       crates/sulimo-core/src/repack.rs:107-131
//   lookup_token_embedding_f16 crates/sulimo-engine/src/scheduler.rs:329-357
//   block_sum of vec_dot_q4_0_q8_0_scalar crates/sulimo-cpu/src/scalar.rs:189-199
// One warp quantizes one 32-value block: lane i owns value i, the block's max|x| is a warp max.
#include "sulimo_common.cuh"
#include "sulimo_internal.h"

namespace sulimo {
namespace {

__global__ void __launch_bounds__(256) quantize_q8_0_kernel(const float* __restrict__ src,
                                                            uint8_t* __restrict__ dst,
                                                            size_t nblocks) {
    pdl_launch_dependents();
    pdl_wait_prerequisites();
    const int lane = threadIdx.x & 31;
    size_t w = (size_t)blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;
    const size_t stride = (size_t)gridDim.x * (blockDim.x / 32);
    for (; w < nblocks; w += stride) quantize_block_warp(__ldg(src + w * 32 + lane), dst + w * 34, lane);
}

template <typename T>
__device__ __forceinline__ float to_f32(T v);
template <>
__device__ __forceinline__ float to_f32<float>(float v) { return v; }
template <>
__device__ __forceinline__ float to_f32<__half>(__half v) { return __half2float(v); }

// act [n][bpp*32]; token t, block b -> ring slot (start_pos+t) % capacity, byte b*34.
template <typename T>
__global__ void __launch_bounds__(256) kv_store_q8_0_kernel(const T* __restrict__ act,
                                                            uint8_t* __restrict__ kv,
                                                            size_t start_pos, size_t capacity,
                                                            size_t bpp, size_t n) {
    pdl_launch_dependents();
    pdl_wait_prerequisites();
    const int lane = threadIdx.x & 31;
    size_t w = (size_t)blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;
    const size_t stride = (size_t)gridDim.x * (blockDim.x / 32);
    const size_t total = n * bpp;
    for (; w < total; w += stride) {
        size_t t = w / bpp, b = w % bpp;
        size_t slot = (start_pos + t) % capacity;
        float v = to_f32<T>(act[w * 32 + lane]);
        quantize_block_warp(v, kv + slot * bpp * 34 + b * 34, lane);
    }
}

// One thread per (row, block, byte i): writes weights i and i+16 of the block.  MODE:
// DEQUANT_F32 exact f32 (dequantize_q4_0_soa, repack.rs:107-131), DEQUANT_F16 f16
// (lookup_token_embedding_f16, scheduler.rs:345-357), DEQUANT_F16_WIDE that f16 value stored
// as f32 (the f16 embedding row widened into an fp32 residual stream).
template <int MODE>
__global__ void __launch_bounds__(256) dequant_rows_kernel(const uint16_t* __restrict__ scales,
                                                           const uint8_t* __restrict__ quants,
                                                           int nb, const int32_t* __restrict__ rows,
                                                           int count, void* __restrict__ out) {
    pdl_launch_dependents();
    pdl_wait_prerequisites();
    size_t idx = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    size_t total = (size_t)count * nb * 16;
    if (idx >= total) return;
    int i = (int)(idx % 16);
    size_t rb = idx / 16;
    int b = (int)(rb % nb);
    int c = (int)(rb / nb);
    size_t r = (size_t)rows[c];
    size_t blk = r * nb + b;
    float d = f16_bits_to_f32(scales[blk]);
    uint8_t byte = quants[blk * 16 + i];
    float w0 = __fmul_rn((float)((int)(byte & 0x0F) - 8), d);
    float w1 = __fmul_rn((float)((int)(byte >> 4) - 8), d);
    size_t o = (size_t)c * nb * 32 + (size_t)b * 32 + i;
    if (MODE == DEQUANT_F16) {
        __half* oh = reinterpret_cast<__half*>(out);
        oh[o] = __float2half_rn(w0);
        oh[o + 16] = __float2half_rn(w1);
    } else if (MODE == DEQUANT_F16_WIDE) {
        float* of = reinterpret_cast<float*>(out);
        of[o] = __half2float(__float2half_rn(w0));
        of[o + 16] = __half2float(__float2half_rn(w1));
    } else {
        float* of = reinterpret_cast<float*>(out);
        of[o] = w0;
        of[o + 16] = w1;
    }
}

// out[r*nb+b] = sum_i (w_i-8)*x_i as i32.
__global__ void __launch_bounds__(256) block_sums_kernel(const uint8_t* __restrict__ wq,
                                                         const uint8_t* __restrict__ xq8, int rows,
                                                         int nb, int32_t* __restrict__ out) {
    pdl_launch_dependents();
    pdl_wait_prerequisites();
    size_t idx = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (idx >= (size_t)rows * nb) return;
    int b = (int)(idx % nb);
    const uint8_t* w = wq + idx * 16;
    const int8_t* x = reinterpret_cast<const int8_t*>(xq8 + (size_t)b * 34 + 2);
    int s = 0;
#pragma unroll
    for (int i = 0; i < 16; i++) s += ((int)(w[i] & 0x0F) - 8) * x[i] + ((int)(w[i] >> 4) - 8) * x[i + 16];
    out[idx] = s;
}

int grid_for(size_t warps_needed, int num_sms) {
    size_t ctas = (warps_needed + 7) / 8;
    size_t cap = (size_t)num_sms * 16;
    if (ctas > cap) ctas = cap;
    if (ctas < 1) ctas = 1;
    return (int)ctas;
}

}  // namespace

int launch_quantize_q8_0(sulimo_ctx* ctx, const float* src, void* dst, size_t n) {
    size_t nb = n / 32;
    cudaError_t le = launch_pdl(quantize_q8_0_kernel, dim3(grid_for(nb, ctx->num_sms)), dim3(256),
                                0, ctx->stream, src, reinterpret_cast<uint8_t*>(dst), nb);
    if (le != cudaSuccess) return check_cuda(le, "quantize_q8_0 launch");
    ctx->launches++;
    return check_cuda(cudaGetLastError(), "quantize_q8_0 launch");
}

int launch_kv_store_q8_0(sulimo_ctx* ctx, const void* act, int act_dtype, void* kv,
                         size_t start_pos, size_t capacity, size_t bpp, size_t n) {
    int g = grid_for(n * bpp, ctx->num_sms);
    if (act_dtype == SULIMO_ACT_F16)
        (void)launch_pdl(kv_store_q8_0_kernel<__half>, dim3(g), dim3(256), 0, ctx->stream,
                         reinterpret_cast<const __half*>(act), reinterpret_cast<uint8_t*>(kv),
                         start_pos, capacity, bpp, n);
    else
        (void)launch_pdl(kv_store_q8_0_kernel<float>, dim3(g), dim3(256), 0, ctx->stream,
                         reinterpret_cast<const float*>(act), reinterpret_cast<uint8_t*>(kv),
                         start_pos, capacity, bpp, n);
    ctx->launches++;
    return check_cuda(cudaGetLastError(), "kv_store_q8_0 launch");
}

int launch_dequant_rows(sulimo_ctx* ctx, const void* scales, const void* quants, int cols,
                        const int32_t* row_ids, int count, void* out, int out_dtype) {
    int nb = cols / 32;
    size_t total = (size_t)count * nb * 16;
    int g = (int)((total + 255) / 256);
    const uint16_t* sc = reinterpret_cast<const uint16_t*>(scales);
    const uint8_t* qu = reinterpret_cast<const uint8_t*>(quants);
    if (out_dtype == SULIMO_OUT_F16)
        (void)launch_pdl(dequant_rows_kernel<DEQUANT_F16>, dim3(g), dim3(256), 0, ctx->stream, sc,
                         qu, nb, row_ids, count, out);
    else if (out_dtype == DEQUANT_F16_WIDE)
        (void)launch_pdl(dequant_rows_kernel<DEQUANT_F16_WIDE>, dim3(g), dim3(256), 0, ctx->stream,
                         sc, qu, nb, row_ids, count, out);
    else
        (void)launch_pdl(dequant_rows_kernel<DEQUANT_F32>, dim3(g), dim3(256), 0, ctx->stream, sc,
                         qu, nb, row_ids, count, out);
    ctx->launches++;
    return check_cuda(cudaGetLastError(), "dequant_rows launch");
}

int launch_block_sums(sulimo_ctx* ctx, const void* w_quants, const void* x_q8, int rows, int cols,
                      int32_t* out) {
    int nb = cols / 32;
    size_t total = (size_t)rows * nb;
    block_sums_kernel<<<(int)((total + 255) / 256), 256, 0, ctx->stream>>>(
        reinterpret_cast<const uint8_t*>(w_quants), reinterpret_cast<const uint8_t*>(x_q8), rows,
        nb, out);
    ctx->launches++;
    return check_cuda(cudaGetLastError(), "block_sums launch");
}

}  // namespace sulimo
