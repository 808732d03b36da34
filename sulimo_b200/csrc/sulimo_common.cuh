// sulimo_common.cuh — shared device helpers for the sm_100a kernels of libsulimo_cuda.
#pragma once

#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/sulimo_cuda.h"
#include "sulimo_internal.h"

// Device error codes written to the context's error word (first writer wins).
#define SULIMO_DEVERR_WAIT_TIMEOUT 1
#define SULIMO_DEVERR_BAD_ARG 2

// A bounded wait gives up after this many nanoseconds of %globaltimer and records an error
// instead of hanging the GPU.  Kernels of this library finish in micro- to milliseconds.
#define SULIMO_WAIT_LIMIT_NS 2000000000ull

namespace sulimo {

__device__ __forceinline__ uint64_t globaltimer_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ void record_device_error(int* err, int code) {
    if (err) atomicCAS(err, 0, code);
}

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// ---- mbarrier -------------------------------------------------------------------------
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}

__device__ __forceinline__ void fence_barrier_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
                 "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

// Waits for the phase with the given parity.  Returns false (and records an error) if the
// phase does not complete within SULIMO_WAIT_LIMIT_NS; *abort short-circuits the wait when
// another role of the same CTA already gave up.
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, uint32_t parity, int* err,
                                                  volatile int* abort_flag) {
    if (mbar_try_wait(bar, parity)) return true;
    uint64_t t0 = globaltimer_ns();
    uint32_t spins = 0;
    while (true) {
        if (mbar_try_wait(bar, parity)) return true;
        if ((++spins & 63u) == 0) {
            if (abort_flag && *abort_flag) return false;
            if (globaltimer_ns() - t0 > SULIMO_WAIT_LIMIT_NS) {
                record_device_error(err, SULIMO_DEVERR_WAIT_TIMEOUT);
                if (abort_flag) *abort_flag = 1;
                return false;
            }
        }
    }
}

// ---- TMA (no multicast anywhere in this library) -------------------------------------------
__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int c0, int c1,
                                            uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%2, %3}], [%4];" ::"r"(smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(smem_u32(bar))
        : "memory");
}

__device__ __forceinline__ void tma_load_3d(void* dst, const CUtensorMap* map, int c0, int c1,
                                            int c2, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%2, %3, %4}], [%5];" ::"r"(smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2), "r"(smem_u32(bar))
        : "memory");
}

// Contiguous global -> shared copy by the TMA unit (no tensor map); 16-byte aligned addresses,
// size a multiple of 16.
__device__ __forceinline__ void bulk_load(void* dst, const void* src, uint32_t bytes,
                                          uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::
            "r"(smem_u32(dst)),
        "l"(src), "r"(bytes), "r"(smem_u32(bar))
        : "memory");
}

__device__ __forceinline__ void prefetch_tensormap(const CUtensorMap* map) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// ---- programmatic dependent launch ------------------------------------------------------
// A kernel launched with the programmatic-stream-serialization attribute may start while the
// previous kernel of the stream still runs; it must wait here before its first global read or
// write of data that kernel touches.  Without the attribute both are no-ops.
__device__ __forceinline__ void pdl_wait_prerequisites() {
    asm volatile("griddepcontrol.wait;" ::: "memory");
}

// Lets the next programmatically dependent kernel of the stream begin launching (it still
// waits for this grid's completion in pdl_wait_prerequisites).
__device__ __forceinline__ void pdl_launch_dependents() {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// ---- Q8_0 ----------------------------------------------------------------------------------
// Quantizes the 32 values of a block held one per lane exactly as quantize_f32_to_q8_0
// (crates/sulimo-core/src/kv_cache.rs:162-192): d = max|x|/127 (IEEE f32), stored as f16 RNE;
// id = 1/d from the f32 d; q = clamp(roundf(x*id), -128, 127).  Returns this lane's code and
// the f32 d in *d_out (every lane).
__device__ __forceinline__ int q8_quantize_lane(float v, float* d_out) {
    float a = fabsf(v);  // fmaxf drops NaN like the reference's `a > max_abs` test
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) a = fmaxf(a, __shfl_xor_sync(0xffffffffu, a, off));
    const float d = __fdiv_rn(a, 127.0f);
    const float id = (d != 0.0f) ? __fdiv_rn(1.0f, d) : 0.0f;
    float q = roundf(__fmul_rn(v, id));
    if (q != q) q = 0.0f;  // f32 NaN `as i8` == 0
    q = fminf(fmaxf(q, -128.0f), 127.0f);
    *d_out = d;
    return (int)q;
}

// The 34-byte Q8_0 block [d: f16][32 x i8] of the 32 values held one per lane.
__device__ __forceinline__ void quantize_block_warp(float v, uint8_t* dst, int lane) {
    float d;
    const int q = q8_quantize_lane(v, &d);
    dst[2 + lane] = (uint8_t)(int8_t)q;
    // the f16 scale as one 2-byte store (blocks are 34 bytes, so dst is 2-byte aligned)
    if (lane == 0) *reinterpret_cast<__half*>(dst) = __float2half_rn(d);
}

// Writes the block as Q8Out asks: the block array and / or the staged form (the staged
// aux word needs the block's code sum: one warp reduction).
__device__ __forceinline__ void q8_store_block(const Q8Out& o, float v, size_t row, int blk,
                                               int lane) {
    float d;
    const int q = q8_quantize_lane(v, &d);
    const __half dh = __float2half_rn(d);
    const int nb = o.K / 32;
    if (o.aos) {
        uint8_t* dst = o.aos + (row * nb + blk) * 34;
        dst[2 + lane] = (uint8_t)(int8_t)q;
        if (lane == 0) *reinterpret_cast<__half*>(dst) = dh;
    }
    if (o.codes) {
        o.codes[row * o.K + (size_t)blk * 32 + lane] = (int8_t)q;
        int s = q;
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) s += __shfl_xor_sync(0xffffffffu, s, off);
        if (lane == 0)
            o.aux[((row >> 3) * nb + blk) * 8 + (row & 7)] =
                make_int2(__float_as_int(__half2float(dh)), 0x4B400000 - 8 * s);
    }
}

// ---- misc ------------------------------------------------------------------------------
__device__ __forceinline__ void fence_proxy_async_smem() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
    uint32_t r;
    asm("prmt.b32 %0, %1, %2, %3;" : "=r"(r) : "r"(a), "r"(b), "r"(sel));
    return r;
}

// sum_i a.u8[i] * b.s8[i] + c  (unsigned x signed 4-way byte dot product)
__device__ __forceinline__ int dp4a_us(uint32_t a, uint32_t b, int c) {
    int r;
    asm("dp4a.u32.s32 %0, %1, %2, %3;" : "=r"(r) : "r"(a), "r"(b), "r"(c));
    return r;
}

__device__ __forceinline__ float f16_bits_to_f32(uint16_t h) {
    return __half2float(__ushort_as_half(h));
}

}  // namespace sulimo
