// tc_sm100.cuh — tcgen05 / TMA helpers shared by the Q4_0 prefill GEMM kernels (the one-CTA
// form in gemm_q4_0_tc.cu and the CTA-pair form in gemm_q4_0_pair.cu): fences, TMA tensor
// stores and bulk groups, the 128-byte-swizzle shared-memory descriptor, TMEM loads / stores,
// the Q4_0 block dequant into f16 TMEM columns and the ordered split-K reduction.
#pragma once

#include "sulimo_common.cuh"

namespace sulimo {
namespace {

// ---- tcgen05 / TMA wrappers ----------------------------------------------------------------
__device__ __forceinline__ void tc_fence_before() {
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

__device__ __forceinline__ void tma_store_2d(const CUtensorMap* map, int c0, int c1,
                                             const void* src) {
    asm volatile(
        "cp.async.bulk.tensor.2d.global.shared::cta.tile.bulk_group [%0, {%1, %2}], [%3];" ::"l"(
            reinterpret_cast<uint64_t>(map)),
        "r"(c0), "r"(c1), "r"(smem_u32(src))
        : "memory");
}

__device__ __forceinline__ void tma_store_3d(const CUtensorMap* map, int c0, int c1, int c2,
                                             const void* src) {
    asm volatile(
        "cp.async.bulk.tensor.3d.global.shared::cta.tile.bulk_group [%0, {%1, %2, %3}], [%4];" ::
            "l"(reinterpret_cast<uint64_t>(map)),
        "r"(c0), "r"(c1), "r"(c2), "r"(smem_u32(src))
        : "memory");
}

__device__ __forceinline__ void bulk_commit() {
    asm volatile("cp.async.bulk.commit_group;" ::: "memory");
}

// Waits until the committed bulk stores have read their shared-memory sources (the global
// writes complete on their own before the grid is complete).
__device__ __forceinline__ void bulk_wait_read_all() {
    asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
}

// Waits until the committed bulk stores' global writes are complete and visible to this thread.
__device__ __forceinline__ void bulk_wait_all() {
    asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
}

__device__ __forceinline__ void named_barrier_sync(int id, int threads) {
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}

// Shared-memory matrix descriptor: K-major, 128-byte swizzle, 8-row groups 1024 bytes apart.
__device__ __forceinline__ uint64_t sw128_desc(uint32_t saddr) {
    uint64_t d = 0;
    d |= (uint64_t)((saddr >> 4) & 0x3FFFu);  // start address
    d |= (uint64_t)1 << 16;                    // leading byte offset (unused for SW128 K-major)
    d |= (uint64_t)(1024 >> 4) << 32;          // stride byte offset
    d |= (uint64_t)1 << 46;                    // descriptor version (sm_100)
    d |= (uint64_t)2 << 61;                    // SWIZZLE_128B
    return d;
}


__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t* v) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, "
        "%11, %12, %13, %14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, "
        "%28, %29, %30, %31, %32};" ::"r"(taddr),
        "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]),
        "r"(v[8]), "r"(v[9]), "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]),
        "r"(v[15]), "r"(v[16]), "r"(v[17]), "r"(v[18]), "r"(v[19]), "r"(v[20]), "r"(v[21]),
        "r"(v[22]), "r"(v[23]), "r"(v[24]), "r"(v[25]), "r"(v[26]), "r"(v[27]), "r"(v[28]),
        "r"(v[29]), "r"(v[30]), "r"(v[31])
        : "memory");
}

__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t* v) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, "
        "%11, %12, %13, %14, %15, %16};" ::"r"(taddr),
        "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]),
        "r"(v[8]), "r"(v[9]), "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]),
        "r"(v[15])
        : "memory");
}

__device__ __forceinline__ void tmem_st_wait() {
    asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

// Loads 32 columns of this warp's 32 TMEM lanes and waits for them; the wait carries the
// registers as operands so no use can be scheduled before it.
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&v)[32]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, "
        "%11, %12, %13, %14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, "
        "%28, %29, %30, %31}, [%32];"
        : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]),
          "=r"(v[7]), "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]),
          "=r"(v[13]), "=r"(v[14]), "=r"(v[15]), "=r"(v[16]), "=r"(v[17]), "=r"(v[18]),
          "=r"(v[19]), "=r"(v[20]), "=r"(v[21]), "=r"(v[22]), "=r"(v[23]), "=r"(v[24]),
          "=r"(v[25]), "=r"(v[26]), "=r"(v[27]), "=r"(v[28]), "=r"(v[29]), "=r"(v[30]),
          "=r"(v[31])
        : "r"(taddr)
        : "memory");
    asm volatile("tcgen05.wait::ld.sync.aligned;"
                 : "+r"(v[0]), "+r"(v[1]), "+r"(v[2]), "+r"(v[3]), "+r"(v[4]), "+r"(v[5]),
                   "+r"(v[6]), "+r"(v[7]), "+r"(v[8]), "+r"(v[9]), "+r"(v[10]), "+r"(v[11]),
                   "+r"(v[12]), "+r"(v[13]), "+r"(v[14]), "+r"(v[15]), "+r"(v[16]), "+r"(v[17]),
                   "+r"(v[18]), "+r"(v[19]), "+r"(v[20]), "+r"(v[21]), "+r"(v[22]), "+r"(v[23]),
                   "+r"(v[24]), "+r"(v[25]), "+r"(v[26]), "+r"(v[27]), "+r"(v[28]), "+r"(v[29]),
                   "+r"(v[30]), "+r"(v[31])
                 :
                 : "memory");
}

// Starts a load of 32 columns of this warp's 32 TMEM lanes without waiting for it; complete it
// with tmem_ld_wait_carry on the same registers.
__device__ __forceinline__ void tmem_ld32_issue(uint32_t taddr, uint32_t (&v)[32]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, "
        "%11, %12, %13, %14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, "
        "%28, %29, %30, %31}, [%32];"
        : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]),
          "=r"(v[7]), "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]),
          "=r"(v[13]), "=r"(v[14]), "=r"(v[15]), "=r"(v[16]), "=r"(v[17]), "=r"(v[18]),
          "=r"(v[19]), "=r"(v[20]), "=r"(v[21]), "=r"(v[22]), "=r"(v[23]), "=r"(v[24]),
          "=r"(v[25]), "=r"(v[26]), "=r"(v[27]), "=r"(v[28]), "=r"(v[29]), "=r"(v[30]),
          "=r"(v[31])
        : "r"(taddr)
        : "memory");
}

// Waits for this thread's TMEM loads in flight; carrying the registers as operands keeps every
// use of them after the wait.
__device__ __forceinline__ void tmem_ld_wait_carry(uint32_t (&v)[32]) {
    asm volatile("tcgen05.wait::ld.sync.aligned;"
                 : "+r"(v[0]), "+r"(v[1]), "+r"(v[2]), "+r"(v[3]), "+r"(v[4]), "+r"(v[5]),
                   "+r"(v[6]), "+r"(v[7]), "+r"(v[8]), "+r"(v[9]), "+r"(v[10]), "+r"(v[11]),
                   "+r"(v[12]), "+r"(v[13]), "+r"(v[14]), "+r"(v[15]), "+r"(v[16]), "+r"(v[17]),
                   "+r"(v[18]), "+r"(v[19]), "+r"(v[20]), "+r"(v[21]), "+r"(v[22]), "+r"(v[23]),
                   "+r"(v[24]), "+r"(v[25]), "+r"(v[26]), "+r"(v[27]), "+r"(v[28]), "+r"(v[29]),
                   "+r"(v[30]), "+r"(v[31])
                 :
                 : "memory");
}

// 16 quant bytes of one Q4_0 block -> 16 packed f16x2 words (TMEM columns of the block):
// column c holds weights k = 2c, 2c+1 of the block; weights 0..15 are the low nibbles of
// bytes 0..15, weights 16..31 the high nibbles (repack.rs:122-129).
__device__ __forceinline__ void dequant_block(const uint4 q, uint32_t dbits, uint32_t* col) {
    const __half2 d2 = __halves2half2(__ushort_as_half((uint16_t)dbits),
                                      __ushort_as_half((uint16_t)dbits));
    const __half2 k1032 = __halves2half2(__ushort_as_half(0x6408), __ushort_as_half(0x6408));
    const uint32_t words[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
    for (int w = 0; w < 4; w++) {
        const uint32_t lo = words[w] & 0x0F0F0F0Fu;
        const uint32_t hi = (words[w] >> 4) & 0x0F0F0F0Fu;
        // {0x6400 | nibble} is the f16 value 1024 + nibble; minus 1032 gives nibble - 8 exactly.
        const uint32_t p[4] = {prmt(lo, 0x64646464u, 0x4140), prmt(lo, 0x64646464u, 0x4342),
                               prmt(hi, 0x64646464u, 0x4140), prmt(hi, 0x64646464u, 0x4342)};
        __half2 h[4];
#pragma unroll
        for (int e = 0; e < 4; e++) {
            h[e] = __hmul2(__hsub2(*reinterpret_cast<const __half2*>(&p[e]), k1032), d2);
        }
        col[2 * w] = *reinterpret_cast<uint32_t*>(&h[0]);
        col[2 * w + 1] = *reinterpret_cast<uint32_t*>(&h[1]);
        col[8 + 2 * w] = *reinterpret_cast<uint32_t*>(&h[2]);
        col[8 + 2 * w + 1] = *reinterpret_cast<uint32_t*>(&h[3]);
    }
}

// The exact-weight form of dequant_block: the same column layout, each weight w = d*(q-8)
// (exact in fp32: an 11-bit scale times an integer in [-8, 7]) as hi = f16(w) in `hi` and
// lo = f16(w - hi) in `lo`.  w - hi is exact in fp32 and is a multiple of the scale's last
// bit, so it is exact in f16 as well (subnormal included): hi + lo == w.
__device__ __forceinline__ void dequant_block_exact(const uint4 q, uint32_t dbits, uint32_t* hi,
                                                    uint32_t* lo) {
    const float d = __half2float(__ushort_as_half((uint16_t)dbits));
    const __half2 k1032 = __halves2half2(__ushort_as_half(0x6408), __ushort_as_half(0x6408));
    const uint32_t words[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
    for (int w = 0; w < 4; w++) {
        const uint32_t lo4 = words[w] & 0x0F0F0F0Fu;
        const uint32_t hi4 = (words[w] >> 4) & 0x0F0F0F0Fu;
        const uint32_t p[4] = {prmt(lo4, 0x64646464u, 0x4140), prmt(lo4, 0x64646464u, 0x4342),
                               prmt(hi4, 0x64646464u, 0x4140), prmt(hi4, 0x64646464u, 0x4342)};
        const int col[4] = {2 * w, 2 * w + 1, 8 + 2 * w, 8 + 2 * w + 1};
#pragma unroll
        for (int e = 0; e < 4; e++) {
            // q - 8 exactly (as in dequant_block), then w in fp32
            const float2 qm = __half22float2(
                __hsub2(*reinterpret_cast<const __half2*>(&p[e]), k1032));
            const float w0 = qm.x * d, w1 = qm.y * d;
            const __half2 h = __floats2half2_rn(w0, w1);
            const float2 hf = __half22float2(h);
            const __half2 l = __floats2half2_rn(w0 - hf.x, w1 - hf.y);
            hi[col[e]] = *reinterpret_cast<const uint32_t*>(&h);
            lo[col[e]] = *reinterpret_cast<const uint32_t*>(&l);
        }
    }
}

// Partial sums of split-K CTAs go to an fp32 workspace [split][n][m]; this kernel adds the
// splits in index order (deterministic) and writes f16 or f32 results.  Launched as a
// programmatic dependent of the GEMM: its CTAs wait for the partials in griddepcontrol.wait.
// Each thread issues the loads of all its splits (up to SPLITK_BATCH at a time) before the
// first add, so the partials cost one L2 round trip, not one per split.
constexpr int SPLITK_BATCH = 8;
template <bool OUT_F32>
__global__ void __launch_bounds__(256)
    splitk_reduce_kernel(const float* __restrict__ ws, void* __restrict__ out, size_t nm,
                         int splits) {
    pdl_launch_dependents();
    pdl_wait_prerequisites();
    const size_t i4 = ((size_t)blockIdx.x * blockDim.x + threadIdx.x) * 4;
    if (i4 >= nm) return;
    float4 acc = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
    for (int z0 = 0; z0 < splits; z0 += SPLITK_BATCH) {
        float4 p[SPLITK_BATCH];
#pragma unroll
        for (int j = 0; j < SPLITK_BATCH; j++)
            if (z0 + j < splits)
                p[j] = __ldcg(reinterpret_cast<const float4*>(ws + (size_t)(z0 + j) * nm + i4));
#pragma unroll
        for (int j = 0; j < SPLITK_BATCH; j++) {
            if (z0 + j >= splits) break;
            if (z0 + j == 0) {
                acc = p[j];
            } else {
                acc.x += p[j].x;
                acc.y += p[j].y;
                acc.z += p[j].z;
                acc.w += p[j].w;
            }
        }
    }
    if (OUT_F32) {
        *reinterpret_cast<float4*>(reinterpret_cast<float*>(out) + i4) = acc;
    } else {
        __half2 a = __floats2half2_rn(acc.x, acc.y), b = __floats2half2_rn(acc.z, acc.w);
        uint2 v = make_uint2(*reinterpret_cast<uint32_t*>(&a), *reinterpret_cast<uint32_t*>(&b));
        *reinterpret_cast<uint2*>(reinterpret_cast<__half*>(out) + i4) = v;
    }
}

// A tiled 2-D tensor map (inner dimension first; row pitch in bytes).
inline int encode_2d(CUtensorMap* map, CUtensorMapDataType dt, const void* base, uint64_t inner,
                     uint64_t outer, uint64_t row_bytes, uint32_t box_inner, uint32_t box_outer,
                     CUtensorMapSwizzle swz) {
    const uint64_t dims[2] = {inner, outer};
    const uint32_t box[2] = {box_inner, box_outer};
    return encode_tensor_map(map, dt, base, 2, dims, &row_bytes, box, swz);
}

}  // namespace
}  // namespace sulimo
