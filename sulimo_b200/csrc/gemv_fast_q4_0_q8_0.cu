// gemv_fast_q4_0_q8_0.cu — decode matvec Q4_0 (SoA) x Q8_0 in "fast mode": the same exact
// integer block sums as the reference (avx2.rs:113-164 / scalar.rs:173-205), but each row's
// blocks are spread over the 32 lanes of a warp whose fp32 partial sums are combined in a fixed
// tree.
//
// Per block b of row r (weights w = nibble - 8, activations x, scales d_w, d_x):
//   s(b) = sum_i w_i x_i                         exact int32 (dp4a, offset -8 * sum x folded in)
//   acc_l += float(s(b)) * (d_w * d_x)           one fp32 FMA; lane l owns blocks b = l mod 32
//   y_r = butterfly sum of acc_0..acc_31 (xor 16, 8, 4, 2, 1)
// This differs from the AVX2 kernel only in the grouping of the fp32 additions (the AVX2 kernel
// keeps 8 per-lane FMA chains over all blocks), so results agree to fp32 rounding (the parity
// tests bound the relative error) and are deterministic for a given shape.  The bit-exact
// AVX2-order kernel stays the default of sulimo_cuda_gemv_q4_0_q8_0: its order admits only 8
// sequential chains per row, which keeps a batch-1 matvec latency-bound.
//
// Register streaming, no shared-memory ring: a warp owns R (1 or 2) rows per iteration and
// loads their quants (16 B per lane per block, coalesced along the row) and scales into
// registers, issuing the next rows' loads before it computes the current ones.  For static
// weights (a decode step's model parameters) the first rows are loaded before
// griddepcontrol.wait, so the weight stream overlaps the previous kernel; after the wait the
// CTA only stages the Q8_0 activations in shared memory (8 aligned words + {d_x, -8 * sum x}
// per block) and computes.
// Up to three matrices sharing the activations (q/k/v, gate/up) go in one launch: their rows
// are numbered consecutively and each row picks its matrix.
#include "sulimo_common.cuh"
#include "sulimo_internal.h"

namespace sulimo {
namespace {

constexpr int GR_THREADS = 256;
constexpr int GR_WARPS = GR_THREADS / 32;
constexpr int GR_MAX_MATS = 3;
constexpr int GR_MAX_BPL = 9;     // blocks per lane: K <= 9216
constexpr int GR_MAX_NV = 8;
constexpr size_t GR_ACT_LIMIT = 48 * 1024;
constexpr int GR_BIAS = 0x4B400000;  // bits of 1.5 * 2^23: int add on these bits is exact

struct GrGroup {
    const uint16_t* scales[GR_MAX_MATS];
    const uint8_t* quants[GR_MAX_MATS];
    float* out[GR_MAX_MATS];
    int rows[GR_MAX_MATS];
    int first_row[GR_MAX_MATS];  // global row index of the matrix's row 0
    int count, total_rows;
};

template <int BPL>
struct RowRegs {
    uint4 q[BPL];
    uint16_t s[BPL];
};

template <int BPL>
__device__ __forceinline__ void load_row(const GrGroup& grp, int r, int nb, int lane,
                                         RowRegs<BPL>& w) {
    int m = 0;
#pragma unroll
    for (int i = 1; i < GR_MAX_MATS; i++)
        if (i < grp.count && r >= grp.first_row[i]) m = i;
    const size_t lr = (size_t)(r - grp.first_row[m]);
    const uint4* q = reinterpret_cast<const uint4*>(grp.quants[m]) + lr * nb;
    const uint16_t* s = grp.scales[m] + lr * nb;
#pragma unroll
    for (int j = 0; j < BPL; j++) {
        const int b = lane + 32 * j;
        if (b < nb) {
            w.q[j] = __ldg(q + b);
            w.s[j] = __ldg(s + b);
        } else {
            w.q[j] = make_uint4(0, 0, 0, 0);
            w.s[j] = 0;
        }
    }
}

// R rows (r0 .. r0 + R - 1, those below total) against the staged activations: lane partials,
// butterfly sums, stores.  The rows share every activation load (shared memory traffic per row
// falls by R when several vectors are staged); each row accumulates its blocks in the same
// order for any R.
template <int BPL, int NV, int R>
__device__ __forceinline__ void rows_dot(const GrGroup& grp, const RowRegs<BPL> (&w)[R], int r0,
                                         int nb, int lane, int v0, int nv, const uint4* xw,
                                         const int2* aux) {
    float acc[R][NV];
#pragma unroll
    for (int k = 0; k < R; k++)
#pragma unroll
        for (int v = 0; v < NV; v++) acc[k][v] = 0.0f;
#pragma unroll
    for (int j = 0; j < BPL; j++) {
        const int b = lane + 32 * j;
        if (b < nb) {
            uint32_t lo[R][4], hi[R][4];
            float dw[R];
#pragma unroll
            for (int k = 0; k < R; k++) {
                const uint32_t qw[4] = {w[k].q[j].x, w[k].q[j].y, w[k].q[j].z, w[k].q[j].w};
#pragma unroll
                for (int i = 0; i < 4; i++) {
                    lo[k][i] = qw[i] & 0x0F0F0F0Fu;         // weights 4i..4i+3 -> x bytes 4i..
                    hi[k][i] = (qw[i] >> 4) & 0x0F0F0F0Fu;  // weights 16+4i.. -> x 16+4i..
                }
                dw[k] = f16_bits_to_f32(w[k].s[j]);
            }
#pragma unroll
            for (int v = 0; v < NV; v++) {
                const int vb = v * nb + b;
                const uint4 x0 = xw[2 * vb], x1 = xw[2 * vb + 1];
                const int2 ax = aux[vb];
                const float dx = __int_as_float(ax.x);
#pragma unroll
                for (int k = 0; k < R; k++) {
                    int sacc = ax.y;
                    sacc = dp4a_us(lo[k][0], x0.x, sacc);
                    sacc = dp4a_us(lo[k][1], x0.y, sacc);
                    sacc = dp4a_us(lo[k][2], x0.z, sacc);
                    sacc = dp4a_us(lo[k][3], x0.w, sacc);
                    sacc = dp4a_us(hi[k][0], x1.x, sacc);
                    sacc = dp4a_us(hi[k][1], x1.y, sacc);
                    sacc = dp4a_us(hi[k][2], x1.z, sacc);
                    sacc = dp4a_us(hi[k][3], x1.w, sacc);
                    const float sf = __fsub_rn(__int_as_float(sacc), 12582912.0f);  // |s| < 2^15
                    acc[k][v] = __fmaf_rn(sf, __fmul_rn(dw[k], dx), acc[k][v]);
                }
            }
        }
    }
#pragma unroll
    for (int k = 0; k < R; k++) {
        const int r = r0 + k;
        if (r >= grp.total_rows) break;  // warp-uniform
        int m = 0;
#pragma unroll
        for (int i = 1; i < GR_MAX_MATS; i++)
            if (i < grp.count && r >= grp.first_row[i]) m = i;
        const int lr = r - grp.first_row[m];
#pragma unroll
        for (int v = 0; v < NV; v++) {
            float t = acc[k][v];
#pragma unroll
            for (int o = 16; o > 0; o >>= 1)
                t = __fadd_rn(t, __shfl_xor_sync(0xffffffffu, t, o));
            if (lane == 0 && v < nv) grp.out[m][(size_t)(v0 + v) * grp.rows[m] + lr] = t;
        }
    }
}

// Quantizes one 32-value block held as 4 consecutive values by each of 8 adjacent lanes,
// exactly as quantize_f32_to_q8_0 / quantize_block_warp (d = max|y| / 127 with NaN dropped,
// id = 1/d from the f32 d, q = clamp(roundf(y * id), -128, 127), NaN -> 0).  Returns this
// lane's 4 q bytes as one word; *dx = the stored f16 scale as f32, *qsum = sum of the 32 q.
// All 32 lanes of the warp must call it.
__device__ __forceinline__ uint32_t quantize_block_8lanes(float4 y, float* dx, int* qsum) {
    float a = fmaxf(fmaxf(fabsf(y.x), fabsf(y.y)), fmaxf(fabsf(y.z), fabsf(y.w)));
    a = fmaxf(a, __shfl_xor_sync(0xffffffffu, a, 1));
    a = fmaxf(a, __shfl_xor_sync(0xffffffffu, a, 2));
    a = fmaxf(a, __shfl_xor_sync(0xffffffffu, a, 4));
    const float d = __fdiv_rn(a, 127.0f);
    const float id = (d != 0.0f) ? __fdiv_rn(1.0f, d) : 0.0f;
    const float v[4] = {y.x, y.y, y.z, y.w};
    uint32_t word = 0;
    int s = 0;
#pragma unroll
    for (int i = 0; i < 4; i++) {
        float q = roundf(__fmul_rn(v[i], id));
        if (q != q) q = 0.0f;
        q = fminf(fmaxf(q, -128.0f), 127.0f);
        const int qi = (int)q;
        s += qi;
        word |= ((uint32_t)qi & 0xFFu) << (8 * i);
    }
    s += __shfl_xor_sync(0xffffffffu, s, 1);
    s += __shfl_xor_sync(0xffffffffu, s, 2);
    s += __shfl_xor_sync(0xffffffffu, s, 4);
    *qsum = s;
    *dx = __half2float(__float2half_rn(d));
    return word;
}

struct GrPrologue {
    const float* a;
    const float* b;
    const float* w;
    float* a_out;
    float eps;
};

// Stages one vector's activations in shared memory from the residual stream (PRO =
// GEMV_PRO_NORM, batch 1, cols <= 32 * GR_NORM_F4 * GR_THREADS / 8): thread t holds float4
// f = t + k * GR_THREADS (k < GR_NORM_F4) of x + delta and of the norm weight in registers, so
// x, delta and w come in one L2 round trip; 8 adjacent lanes hold one Q8_0 block.  Every
// thread runs all GR_NORM_F4 rounds, so every warp takes every shuffle.
constexpr int GR_NORM_F4 = 4;

__device__ __forceinline__ void stage_norm(const GrPrologue& pro, int v0, int nb,
                                           uint32_t* xw32, int2* aux, float* red) {
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int n4 = nb * 8;  // float4 per vector
    const float4* a4 = reinterpret_cast<const float4*>(pro.a) + (size_t)v0 * n4;
    const float4* b4 = pro.b ? reinterpret_cast<const float4*>(pro.b) + (size_t)v0 * n4 : nullptr;
    const float4* w4 = reinterpret_cast<const float4*>(pro.w);
    float4* o4 = (pro.a_out && blockIdx.x == 0)
                     ? reinterpret_cast<float4*>(pro.a_out) + (size_t)v0 * n4
                     : nullptr;
    const float4 zero = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
    float4 xv[GR_NORM_F4], dv[GR_NORM_F4], wv[GR_NORM_F4];
#pragma unroll
    for (int k = 0; k < GR_NORM_F4; k++) {
        const int f = tid + k * GR_THREADS;
        xv[k] = f < n4 ? a4[f] : zero;
        dv[k] = (b4 && f < n4) ? b4[f] : zero;
        wv[k] = f < n4 ? w4[f] : zero;
    }
    float ss = 0.0f;
#pragma unroll
    for (int k = 0; k < GR_NORM_F4; k++) {
        const int f = tid + k * GR_THREADS;
        float4 x = xv[k];
        if (b4)
            x = make_float4(__fadd_rn(x.x, dv[k].x), __fadd_rn(x.y, dv[k].y),
                            __fadd_rn(x.z, dv[k].z), __fadd_rn(x.w, dv[k].w));
        xv[k] = x;
        if (o4 && f < n4) o4[f] = x;
        ss = __fmaf_rn(x.x, x.x, ss);
        ss = __fmaf_rn(x.y, x.y, ss);
        ss = __fmaf_rn(x.z, x.z, ss);
        ss = __fmaf_rn(x.w, x.w, ss);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    if (lane == 0) red[warp] = ss;
    __syncthreads();
    float t = 0.0f;
#pragma unroll
    for (int w = 0; w < GR_WARPS; w++) t += red[w];
    const float mean = __fdiv_rn(t, (float)(n4 * 4));
    const float scale = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(mean, pro.eps)));
#pragma unroll
    for (int k = 0; k < GR_NORM_F4; k++) {
        const int f = tid + k * GR_THREADS;
        const float4 x = xv[k], g = wv[k];
        const float4 y = make_float4(__fmul_rn(__fmul_rn(x.x, scale), g.x),
                                     __fmul_rn(__fmul_rn(x.y, scale), g.y),
                                     __fmul_rn(__fmul_rn(x.z, scale), g.z),
                                     __fmul_rn(__fmul_rn(x.w, scale), g.w));
        float dx;
        int qsum;
        const uint32_t word = quantize_block_8lanes(y, &dx, &qsum);
        if (f < n4) {
            const int b = f >> 3;
            xw32[b * 8 + (f & 7)] = word;
            if ((f & 7) == 0) aux[b] = make_int2(__float_as_int(dx), GR_BIAS - 8 * qsum);
        }
    }
}

template <int BPL, int NV, int R, int PRO>
__global__ void __launch_bounds__(GR_THREADS)
    gemv_fast_kernel(const __grid_constant__ GrGroup grp, const uint8_t* __restrict__ xq8,
                     const GrPrologue pro, int nb, int batch, int static_weights) {
    __shared__ float red[GR_MAX_NV * GR_WARPS];
    pdl_launch_dependents();
    extern __shared__ __align__(16) uint8_t smem_raw[];
    uint4* xw = reinterpret_cast<uint4*>(smem_raw);                          // [NV][nb][2]
    int2* aux = reinterpret_cast<int2*>(smem_raw + (size_t)NV * nb * 32);     // [NV][nb]
    const int tid = threadIdx.x, lane = tid & 31;
    const int v0 = blockIdx.y * NV;
    const int nv = min(NV, batch - v0);
    // warp w's iteration i covers rows (w + i * warps) * R .. + R - 1
    const int stride = gridDim.x * GR_WARPS * R;
    int r = (blockIdx.x * GR_WARPS + (tid >> 5)) * R;

    RowRegs<BPL> cur[R] = {};
    if (static_weights)
#pragma unroll
        for (int k = 0; k < R; k++)
            if (r + k < grp.total_rows) load_row<BPL>(grp, r + k, nb, lane, cur[k]);
    pdl_wait_prerequisites();
    if (!static_weights)
#pragma unroll
        for (int k = 0; k < R; k++)
            if (r + k < grp.total_rows) load_row<BPL>(grp, r + k, nb, lane, cur[k]);

    // ---- activations: per block 8 aligned words, d_x, -8 * sum(x) + bias ----
    if (PRO == GEMV_PRO_NORM)
        stage_norm(pro, v0, nb, reinterpret_cast<uint32_t*>(xw), aux, red);
    else
    for (int vb = tid; vb < NV * nb; vb += GR_THREADS) {
        uint32_t w[8];
        uint16_t dbits = 0;
        if (vb < nv * nb) {
            const uint16_t* blk =
                reinterpret_cast<const uint16_t*>(xq8 + ((size_t)v0 * nb + vb) * 34);
            dbits = __ldg(blk);
#pragma unroll
            for (int i = 0; i < 8; i++)
                w[i] = (uint32_t)__ldg(blk + 1 + 2 * i) | ((uint32_t)__ldg(blk + 2 + 2 * i) << 16);
        } else {
#pragma unroll
            for (int i = 0; i < 8; i++) w[i] = 0;
        }
        int sum = 0;
#pragma unroll
        for (int i = 0; i < 8; i++) sum = __dp4a((int)w[i], 0x01010101, sum);
        xw[2 * vb] = make_uint4(w[0], w[1], w[2], w[3]);
        xw[2 * vb + 1] = make_uint4(w[4], w[5], w[6], w[7]);
        aux[vb] = make_int2(__float_as_int(f16_bits_to_f32(dbits)), GR_BIAS - 8 * sum);
    }
    __syncthreads();

    for (; r < grp.total_rows; r += stride) {
        RowRegs<BPL> nxt[R] = {};
#pragma unroll
        for (int k = 0; k < R; k++)
            if (r + stride + k < grp.total_rows)
                load_row<BPL>(grp, r + stride + k, nb, lane, nxt[k]);
        rows_dot<BPL, NV, R>(grp, cur, r, nb, lane, v0, nv, xw, aux);
#pragma unroll
        for (int k = 0; k < R; k++) cur[k] = nxt[k];
    }
}

// Resident CTAs per SM of one instantiation (cached per device).
template <int BPL, int NV, int R, int PRO>
int fast_occupancy(sulimo_ctx* ctx, int* blocks) {
    static DeviceBits done;
    static std::atomic<int> occ[64];
    const int dev = ctx->device & 63;
    if (!done.test(dev)) {
        int st = check_cuda(cudaFuncSetAttribute(gemv_fast_kernel<BPL, NV, R, PRO>,
                                                 cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                 (int)GR_ACT_LIMIT),
                            "gemv_fast smem attribute");
        if (st) return st;
        int b = 0;
        st = check_cuda(cudaOccupancyMaxActiveBlocksPerMultiprocessor(
                            &b, gemv_fast_kernel<BPL, NV, R, PRO>, GR_THREADS, GR_ACT_LIMIT),
                        "gemv_fast occupancy");
        if (st) return st;
        occ[dev].store(b < 1 ? 1 : b, std::memory_order_relaxed);
        done.set(dev);
    }
    *blocks = occ[dev].load(std::memory_order_relaxed);
    return SULIMO_OK;
}

struct FastArgs {
    const GrGroup* grp;
    const uint8_t* xq8;
    GrPrologue pro;
    int nb, batch, nv, sw;
};

template <int BPL, int NV, int R, int PRO>
int launch_fast(sulimo_ctx* ctx, const FastArgs& a) {
    const int vec_groups = (a.batch + NV - 1) / NV;
    if (vec_groups > 65535) return set_error(SULIMO_EINVAL, "gemv batch too large");
    const size_t smem = (size_t)NV * a.nb * 40;
    int occ = 1;
    int st = fast_occupancy<BPL, NV, R, PRO>(ctx, &occ);
    if (st) return st;
    // R rows per warp when the rows fit one resident wave, else a resident grid that loops
    size_t ctas = ((size_t)a.grp->total_rows + GR_WARPS * R - 1) / (GR_WARPS * R);
    const size_t wave = (size_t)ctx->num_sms * occ;
    if (ctas > wave) ctas = wave;
    dim3 grid((unsigned)ctas, (unsigned)vec_groups);
    (void)launch_pdl(gemv_fast_kernel<BPL, NV, R, PRO>, grid, dim3(GR_THREADS), smem,
                     ctx->stream, *a.grp, a.xq8, a.pro, a.nb, a.batch, a.sw);
    ctx->launches++;
    return check_cuda(cudaGetLastError(), "gemv_fast launch");
}

// Two rows per warp iteration (both loaded before the wait) for short rows when one row per
// warp would need more than one resident wave.
template <int BPL, int PRO>
int launch_fast_nv(sulimo_ctx* ctx, const FastArgs& a) {
    if constexpr (BPL <= 4) {
        if (a.nv == 1) {
            int occ = 1;
            int st = fast_occupancy<BPL, 1, 1, PRO>(ctx, &occ);
            if (st) return st;
            if ((size_t)a.grp->total_rows > (size_t)ctx->num_sms * occ * GR_WARPS)
                return launch_fast<BPL, 1, 2, PRO>(ctx, a);
        }
    }
    if constexpr (PRO == GEMV_PRO_NORM) {
        return launch_fast<BPL, 1, 1, PRO>(ctx, a);  // batch 1 only (gemv_fast_fused_ok)
    } else if constexpr (BPL <= 4) {
        // several vectors: two rows per warp share each staged activation load (the rows'
        // re-reads of the vectors, not the weights, bound the batched matvec)
        switch (a.nv) {
            case 8: return launch_fast<BPL, 8, 2, PRO>(ctx, a);
            case 4: return launch_fast<BPL, 4, 2, PRO>(ctx, a);
            case 2: return launch_fast<BPL, 2, 2, PRO>(ctx, a);
            default: return launch_fast<BPL, 1, 1, PRO>(ctx, a);
        }
    } else {
        switch (a.nv) {
            case 8: return launch_fast<BPL, 8, 1, PRO>(ctx, a);
            case 4: return launch_fast<BPL, 4, 1, PRO>(ctx, a);
            case 2: return launch_fast<BPL, 2, 1, PRO>(ctx, a);
            default: return launch_fast<BPL, 1, 1, PRO>(ctx, a);
        }
    }
}

template <int PRO>
int launch_fast_bpl(sulimo_ctx* ctx, const FastArgs& a, int bpl) {
    switch (bpl) {
        case 1: return launch_fast_nv<1, PRO>(ctx, a);
        case 2: return launch_fast_nv<2, PRO>(ctx, a);
        case 3: return launch_fast_nv<3, PRO>(ctx, a);
        case 4: return launch_fast_nv<4, PRO>(ctx, a);
        case 5: return launch_fast_nv<5, PRO>(ctx, a);
        case 6: return launch_fast_nv<6, PRO>(ctx, a);
        case 7: return launch_fast_nv<7, PRO>(ctx, a);
        case 8: return launch_fast_nv<8, PRO>(ctx, a);
        default: return launch_fast_nv<9, PRO>(ctx, a);
    }
}

// Layout conditions of the fast form; *nv_out = vectors per weight pass.
bool fast_applies(const GemvMatSrc* src, int count, int cols, int batch, int* nv_out) {
    const int nb = cols / 32;
    const int bpl = (nb + 31) / 32;
    bool ok = count >= 1 && count <= GR_MAX_MATS && cols > 0 && cols % 32 == 0 && bpl >= 1 &&
              bpl <= GR_MAX_BPL && batch >= 1;
    long total = 0;
    for (int i = 0; ok && i < count; i++) {
        ok = src[i].quants && src[i].scales && src[i].out &&
             ((uintptr_t)src[i].quants % 16) == 0 && ((uintptr_t)src[i].scales % 2) == 0 &&
             src[i].rows > 0;
        total += src[i].rows;
    }
    if (total > 0x7fffffffL) ok = false;
    int nv = GR_MAX_NV;
    while (nv > 1 && (nv > batch || (size_t)nv * nb * 40 > GR_ACT_LIMIT)) nv >>= 1;
    if ((size_t)nv * nb * 40 > GR_ACT_LIMIT) ok = false;
    *nv_out = nv;
    return ok;
}

void fill_group(GrGroup& grp, const GemvMatSrc* src, int count) {
    int row = 0;
    for (int i = 0; i < GR_MAX_MATS; i++) {
        const int k = i < count ? i : 0;
        grp.scales[i] = reinterpret_cast<const uint16_t*>(src[k].scales);
        grp.quants[i] = reinterpret_cast<const uint8_t*>(src[k].quants);
        grp.out[i] = src[k].out;
        grp.rows[i] = src[k].rows;
        grp.first_row[i] = row;
        if (i < count) row += src[i].rows;
    }
    grp.count = count;
    grp.total_rows = row;
}

}  // namespace

// The staging buffer of the batched form, grown outside stream capture only (a capture that
// finds it too small takes the lane-tree form instead).
static bool ensure_q8_stage(sulimo_ctx* ctx, size_t bytes) {
    if (bytes <= ctx->q8_stage_bytes) return true;
    cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
    if (cudaStreamIsCapturing(ctx->stream, &cs) != cudaSuccess || cs != cudaStreamCaptureStatusNone)
        return false;
    if (cudaStreamSynchronize(ctx->stream) != cudaSuccess) return false;
    if (ctx->q8_stage) cudaFree(ctx->q8_stage);
    ctx->q8_stage = nullptr;
    ctx->q8_stage_bytes = 0;
    if (cudaMalloc(&ctx->q8_stage, bytes) != cudaSuccess) {
        ctx->q8_stage = nullptr;
        (void)cudaGetLastError();
        return false;
    }
    ctx->q8_stage_bytes = bytes;
    return true;
}

int launch_gemv_fast_group(sulimo_ctx* ctx, const GemvMatSrc* src, int count, const void* x_q8,
                           int cols, int batch, bool static_weights) {
    // several sequences: restage the Q8_0 blocks, then the tensor-core form
    if (batch >= GEMV_MMA_MIN_BATCH && gemv_mma_applies(src, count, cols, batch, ctx->num_sms) &&
        ensure_q8_stage(ctx, q8_staged_bytes(batch, cols))) {
        const Q8Out xs = q8_staged_view(ctx->q8_stage, batch, cols);
        const int st = launch_q8_stage(ctx, x_q8, batch, cols, xs);
        return st ? st : launch_gemv_mma_group(ctx, src, count, xs, cols, batch, static_weights);
    }
    int nv = 1;
    if (!fast_applies(src, count, cols, batch, &nv)) {
        // the exact kernel satisfies the fast form's contract
        bool handled = false;
        int st = launch_gemv_group(ctx, src, count, x_q8, cols, batch, &handled, static_weights);
        for (int i = 0; i < count && !handled && !st; i++)
            st = launch_gemv_q4_0_q8_0(ctx, src[i].scales, src[i].quants, x_q8, src[i].rows, cols,
                                       batch, src[i].out);
        return st;
    }
    GrGroup grp;
    fill_group(grp, src, count);
    FastArgs a = {&grp, reinterpret_cast<const uint8_t*>(x_q8), {}, cols / 32, batch, nv,
                  static_weights ? 1 : 0};
    return launch_fast_bpl<GEMV_PRO_Q8>(ctx, a, (cols / 32 + 31) / 32);
}

bool gemv_fast_fused_ok(const GemvMatSrc* src, int count, int cols, int batch,
                        const GemvPrologue& pro) {
    int nv = 1;
    if (!fast_applies(src, count, cols, batch, &nv)) return false;
    auto al = [](const void* p) { return ((uintptr_t)p % 16) == 0; };
    return pro.mode == GEMV_PRO_NORM && batch == 1 && cols / 4 <= GR_NORM_F4 * GR_THREADS &&
           pro.a && pro.w && al(pro.a) && al(pro.b) && al(pro.w) && al(pro.a_out);
}

int launch_gemv_fast_fused(sulimo_ctx* ctx, const GemvMatSrc* src, int count,
                           const GemvPrologue& pro, int cols, int batch, bool static_weights) {
    int nv = 1;
    if (!gemv_fast_fused_ok(src, count, cols, batch, pro) ||
        !fast_applies(src, count, cols, batch, &nv))
        return set_error(SULIMO_EINVAL, "fused matvec prologue does not apply to this shape");
    GrGroup grp;
    fill_group(grp, src, count);
    FastArgs a = {&grp, nullptr, {pro.a, pro.b, pro.w, pro.a_out, pro.eps}, cols / 32, batch, nv,
                  static_weights ? 1 : 0};
    return launch_fast_bpl<GEMV_PRO_NORM>(ctx, a, (cols / 32 + 31) / 32);
}

}  // namespace sulimo
