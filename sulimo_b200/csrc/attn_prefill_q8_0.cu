// attn_prefill_q8_0.cu — causal GQA prefill attention over the Q8_0 KV ring: the reference's
// causal_gqa_attention_prefill (kernels/prefill.cl:120-237), enqueued by
// enqueue_attention_prefill from execute_prefill_ubatch (crates/sulimo-ocl/src/prefill.rs:337-566).
//
// Token n of the ubatch sits at position start_pos + n and attends to positions
// 0 .. start_pos + n (ring slot p % capacity), query head h to kv head h / (H / Hkv).
//
// This file: the mma.sync form (rings or buffers outside the tcgen05 form's layout conditions);
// the tcgen05 form is attn_prefill_tc.cu.
// Flash-attention form on tensor cores (mma.sync m16n8k16, f16 in, f32 accumulate): one CTA
// per (64-token tile, query head), 4 warps x 16 tokens.  Keys come in chunks of 64: the chunk's
// Q8_0 integers are staged in shared memory as f16 (exact: |q| <= 128) -- K as [key][dim], V
// transposed as [dim][key] -- with the block scales as f32.  Scores: for each 32-dimension
// block b, S_b = Q_b K_b^T on integers, then S += d_k(key, b) * S_b in f32 (the Q8_0 scale is
// applied exactly as the reference's (float)q * d, not folded into an f16 operand).  Online
// softmax in f32 with the causal mask; P V per 32-dimension output block uses P scaled by
// d_v(key, b) (f16 operand).  The reference accumulates the output in f16 in global memory
// (prefill.cl:233); here it stays f32 in registers and is written once as f16.
#include <stdlib.h>
#include <string.h>

#include "sulimo_common.cuh"
#include "sulimo_internal.h"

namespace sulimo {
namespace {

constexpr int PF_TOK = 64;      // query tokens per CTA (16 per warp)
constexpr int PF_KEYS = 64;     // keys per chunk
constexpr int PF_THREADS = 128;

__device__ __forceinline__ uint32_t pack_f16x2(float lo, float hi) {
    __half2 h = __floats2half2_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&h);
}

// D += A (16x16, row) * B (16x8, col), f16 in, f32 accumulate.
__device__ __forceinline__ void mma16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0,
                                         uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, "
        "{%8, %9}, {%0, %1, %2, %3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

template <int HD>
struct PfSmem {
    __half k[PF_KEYS][HD + 8];   // [key][dim] (+8: bank skew)
    __half vt[HD][PF_KEYS + 8];  // [dim][key]
    float kd[PF_KEYS][HD / 32];
    float vd[PF_KEYS][HD / 32];
};

template <int HD>
__global__ void __launch_bounds__(PF_THREADS)
    attn_prefill_kernel(const float* __restrict__ q, const uint8_t* __restrict__ k_ring,
                        const uint8_t* __restrict__ v_ring, size_t start_pos, size_t capacity,
                        int n_tok, int H, int Hkv, float sm_scale, __half* __restrict__ out) {
    pdl_launch_dependents();
    pdl_wait_prerequisites();
    constexpr int NB = HD / 32;
    __shared__ __align__(16) PfSmem<HD> sm;
    const int tile = blockIdx.x, h = blockIdx.y;
    const int kvh = h / (H / Hkv);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int g = lane >> 2, t = lane & 3;
    const int tok0 = tile * PF_TOK + warp * 16;  // this warp's first token
    const size_t bpp = (size_t)Hkv * NB * 34;    // ring bytes per position
    const size_t head_off = (size_t)kvh * NB * 34;

    // Q fragments (f16) of the warp's 16 tokens: A[row][k] = q[tok0+row][h][k]
    uint32_t qa[HD / 16][4];
    {
        const int r0 = min(tok0 + g, n_tok - 1), r1 = min(tok0 + g + 8, n_tok - 1);
        const float* q0 = q + ((size_t)r0 * H + h) * HD;
        const float* q1 = q + ((size_t)r1 * H + h) * HD;
#pragma unroll
        for (int ks = 0; ks < HD / 16; ks++) {
            const int c = ks * 16 + 2 * t;
            qa[ks][0] = pack_f16x2(q0[c], q0[c + 1]);
            qa[ks][1] = pack_f16x2(q1[c], q1[c + 1]);
            qa[ks][2] = pack_f16x2(q0[c + 8], q0[c + 9]);
            qa[ks][3] = pack_f16x2(q1[c + 8], q1[c + 9]);
        }
    }
    const long pos_r0 = (long)(start_pos + tok0 + g), pos_r1 = pos_r0 + 8;

    float o[HD / 8][4];
#pragma unroll
    for (int i = 0; i < HD / 8; i++) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.0f;
    float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.0f, l1 = 0.0f;

    const long last_tok = min((long)n_tok - 1, (long)tile * PF_TOK + PF_TOK - 1);
    const long key_end = (long)start_pos + last_tok + 1;  // keys [0, key_end) for this CTA
    for (long c0 = 0; c0 < key_end; c0 += PF_KEYS) {
        __syncthreads();  // the previous chunk is consumed
        // stage K and V: one (key, block) per thread per step
        for (int it = threadIdx.x; it < PF_KEYS * NB; it += PF_THREADS) {
            const int kk = it / NB, b = it - kk * NB;
            const long p = c0 + kk;
            if (p < key_end) {
                const size_t off = (size_t)(p % (long)capacity) * bpp + head_off + b * 34;
                const uint16_t* kb = reinterpret_cast<const uint16_t*>(k_ring + off);
                const uint16_t* vb = reinterpret_cast<const uint16_t*>(v_ring + off);
                sm.kd[kk][b] = f16_bits_to_f32(kb[0]);
                sm.vd[kk][b] = f16_bits_to_f32(vb[0]);
#pragma unroll
                for (int i = 0; i < 16; i++) {
                    const uint32_t kw = kb[1 + i], vw = vb[1 + i];
                    const int d = b * 32 + 2 * i;
                    sm.k[kk][d] = __int2half_rn((int)(int8_t)(kw & 0xFF));
                    sm.k[kk][d + 1] = __int2half_rn((int)(int8_t)(kw >> 8));
                    sm.vt[d][kk] = __int2half_rn((int)(int8_t)(vw & 0xFF));
                    sm.vt[d + 1][kk] = __int2half_rn((int)(int8_t)(vw >> 8));
                }
            } else {
                sm.kd[kk][b] = 0.0f;
                sm.vd[kk][b] = 0.0f;
#pragma unroll
                for (int i = 0; i < 32; i++) {
                    sm.k[kk][b * 32 + i] = __float2half(0.0f);
                    sm.vt[b * 32 + i][kk] = __float2half(0.0f);
                }
            }
        }
        __syncthreads();
        // warp-uniform skip (mma.sync is warp-collective): no row of this warp sees the chunk
        if (tok0 >= n_tok || c0 > (long)start_pos + tok0 + 15) continue;

        // ---- scores S[16][64]: per 8-key tile nt, sum over dimension blocks of d_k * (Q_b K_b) ----
        float s[PF_KEYS / 8][4];
#pragma unroll
        for (int nt = 0; nt < PF_KEYS / 8; nt++) {
            s[nt][0] = s[nt][1] = s[nt][2] = s[nt][3] = 0.0f;
            const int key = nt * 8 + g;  // B column owned for the fragment load
#pragma unroll
            for (int b = 0; b < NB; b++) {
                float part[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll
                for (int kq = 0; kq < 2; kq++) {
                    const int ks = b * 2 + kq;
                    const int d = ks * 16 + 2 * t;
                    const uint32_t b0 = *reinterpret_cast<const uint32_t*>(&sm.k[key][d]);
                    const uint32_t b1 = *reinterpret_cast<const uint32_t*>(&sm.k[key][d + 8]);
                    mma16816(part, qa[ks], b0, b1);
                }
                // accumulator columns 2t, 2t+1 of the tile = keys nt*8 + 2t, +1
                const float dk0 = sm.kd[nt * 8 + 2 * t][b], dk1 = sm.kd[nt * 8 + 2 * t + 1][b];
                s[nt][0] = __fmaf_rn(part[0], dk0, s[nt][0]);
                s[nt][1] = __fmaf_rn(part[1], dk1, s[nt][1]);
                s[nt][2] = __fmaf_rn(part[2], dk0, s[nt][2]);
                s[nt][3] = __fmaf_rn(part[3], dk1, s[nt][3]);
            }
        }
        // scale, causal mask, chunk row max
        float cm0 = -INFINITY, cm1 = -INFINITY;
#pragma unroll
        for (int nt = 0; nt < PF_KEYS / 8; nt++) {
            const long kp = c0 + nt * 8 + 2 * t;
            s[nt][0] = (kp <= pos_r0) ? s[nt][0] * sm_scale : -INFINITY;
            s[nt][1] = (kp + 1 <= pos_r0) ? s[nt][1] * sm_scale : -INFINITY;
            s[nt][2] = (kp <= pos_r1) ? s[nt][2] * sm_scale : -INFINITY;
            s[nt][3] = (kp + 1 <= pos_r1) ? s[nt][3] * sm_scale : -INFINITY;
            cm0 = fmaxf(cm0, fmaxf(s[nt][0], s[nt][1]));
            cm1 = fmaxf(cm1, fmaxf(s[nt][2], s[nt][3]));
        }
#pragma unroll
        for (int off = 1; off <= 2; off <<= 1) {
            cm0 = fmaxf(cm0, __shfl_xor_sync(0xffffffffu, cm0, off));
            cm1 = fmaxf(cm1, __shfl_xor_sync(0xffffffffu, cm1, off));
        }
        const float nm0 = fmaxf(m0, cm0), nm1 = fmaxf(m1, cm1);
        const float r0 = (nm0 == -INFINITY) ? 1.0f : expf(m0 - nm0);
        const float r1 = (nm1 == -INFINITY) ? 1.0f : expf(m1 - nm1);
        m0 = nm0;
        m1 = nm1;
        float ps0 = 0.0f, ps1 = 0.0f;
#pragma unroll
        for (int nt = 0; nt < PF_KEYS / 8; nt++) {
            s[nt][0] = (s[nt][0] == -INFINITY) ? 0.0f : expf(s[nt][0] - m0);
            s[nt][1] = (s[nt][1] == -INFINITY) ? 0.0f : expf(s[nt][1] - m0);
            s[nt][2] = (s[nt][2] == -INFINITY) ? 0.0f : expf(s[nt][2] - m1);
            s[nt][3] = (s[nt][3] == -INFINITY) ? 0.0f : expf(s[nt][3] - m1);
            ps0 += s[nt][0] + s[nt][1];
            ps1 += s[nt][2] + s[nt][3];
        }
#pragma unroll
        for (int off = 1; off <= 2; off <<= 1) {
            ps0 += __shfl_xor_sync(0xffffffffu, ps0, off);
            ps1 += __shfl_xor_sync(0xffffffffu, ps1, off);
        }
        l0 = l0 * r0 + ps0;
        l1 = l1 * r1 + ps1;
#pragma unroll
        for (int i = 0; i < HD / 8; i++) {
            o[i][0] *= r0;
            o[i][1] *= r0;
            o[i][2] *= r1;
            o[i][3] *= r1;
        }
        // ---- O += (P * d_v) V per 32-dimension output block ----
#pragma unroll
        for (int b = 0; b < NB; b++) {
#pragma unroll
            for (int kt = 0; kt < PF_KEYS / 16; kt++) {
                // A = P[16][keys kt*16 .. +16] scaled by d_v(key, b): the S accumulator tiles
                // 2kt and 2kt+1 hold exactly the A fragment layout of m16n8k16
                const int ka = kt * 16 + 2 * t, kb2 = ka + 8;
                const float da0 = sm.vd[ka][b], da1 = sm.vd[ka + 1][b];
                const float db0 = sm.vd[kb2][b], db1 = sm.vd[kb2 + 1][b];
                uint32_t pa[4];
                pa[0] = pack_f16x2(s[2 * kt][0] * da0, s[2 * kt][1] * da1);
                pa[1] = pack_f16x2(s[2 * kt][2] * da0, s[2 * kt][3] * da1);
                pa[2] = pack_f16x2(s[2 * kt + 1][0] * db0, s[2 * kt + 1][1] * db1);
                pa[3] = pack_f16x2(s[2 * kt + 1][2] * db0, s[2 * kt + 1][3] * db1);
#pragma unroll
                for (int nd = 0; nd < 4; nd++) {
                    const int dim = b * 32 + nd * 8 + g;  // B column (output dimension)
                    const uint32_t b0 = *reinterpret_cast<const uint32_t*>(&sm.vt[dim][ka]);
                    const uint32_t b1 = *reinterpret_cast<const uint32_t*>(&sm.vt[dim][kb2]);
                    mma16816(o[b * 4 + nd], pa, b0, b1);
                }
            }
        }
    }
    if (tok0 >= n_tok) return;
    const float inv0 = l0 > 0.0f ? 1.0f / l0 : 0.0f, inv1 = l1 > 0.0f ? 1.0f / l1 : 0.0f;
    const int r0 = tok0 + g, r1 = tok0 + g + 8;
#pragma unroll
    for (int i = 0; i < HD / 8; i++) {
        const int d = i * 8 + 2 * t;
        if (r0 < n_tok)
            *reinterpret_cast<__half2*>(out + ((size_t)r0 * H + h) * HD + d) =
                __floats2half2_rn(o[i][0] * inv0, o[i][1] * inv0);
        if (r1 < n_tok)
            *reinterpret_cast<__half2*>(out + ((size_t)r1 * H + h) * HD + d) =
                __floats2half2_rn(o[i][2] * inv1, o[i][3] * inv1);
    }
}

}  // namespace

// The tcgen05 form (attn_prefill_tc.cu) where its layout conditions hold (16-byte aligned q,
// out and rings, 16-byte multiple slot pitch), else this mma.sync form; SULIMO_PREFILL_ATTN=mma
// selects this form always (a measurement switch).
int launch_attn_prefill(sulimo_ctx* ctx, const float* q, const void* k_ring, const void* v_ring,
                        size_t start_pos, size_t capacity, int n_tok, int H, int Hkv, int hd,
                        void* out) {
    static const bool force_mma = [] {
        const char* e = getenv("SULIMO_PREFILL_ATTN");
        return e && strcmp(e, "mma") == 0;
    }();
    if (!force_mma && attn_prefill_tc_applies(q, k_ring, v_ring, capacity, Hkv, hd, out))
        return launch_attn_prefill_tc(ctx, q, k_ring, v_ring, start_pos, capacity, n_tok, H, Hkv,
                                      hd, out);
    dim3 grid((unsigned)((n_tok + PF_TOK - 1) / PF_TOK), (unsigned)H);
    const float scale = 1.0f / sqrtf((float)hd);
    const uint8_t* k = reinterpret_cast<const uint8_t*>(k_ring);
    const uint8_t* v = reinterpret_cast<const uint8_t*>(v_ring);
    __half* o = reinterpret_cast<__half*>(out);
    switch (hd) {
        case 64:
            (void)launch_pdl(attn_prefill_kernel<64>, grid, dim3(PF_THREADS), 0, ctx->stream, q, k,
                             v, start_pos, capacity, n_tok, H, Hkv, scale, o);
            break;
        case 128:
            (void)launch_pdl(attn_prefill_kernel<128>, grid, dim3(PF_THREADS), 0, ctx->stream, q, k,
                             v, start_pos, capacity, n_tok, H, Hkv, scale, o);
            break;
        default:
            return set_error(SULIMO_EINVAL, "prefill attention supports head_dim 64 and 128");
    }
    ctx->launches++;
    return check_cuda(cudaGetLastError(), "attn_prefill launch");
}

}  // namespace sulimo
