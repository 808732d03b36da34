// forward.cu — one decode position through a Llama / Qwen2 / Gemma 2-architecture model on the
// GPU: the reference's forward_token (crates/sulimo-engine/src/forward_pass.rs:190-417) for a
// batch of independent sequences that sit at the same position; and the prefill ubatch
// (execute_prefill_ubatch, crates/sulimo-ocl/src/prefill.rs:337-566) for Llama / Qwen2.
//
// Per layer, at one sequence (8 launches on the context's stream, no host synchronisation, each a
// programmatic dependent of the previous one):
//   GEMV q,k,v         one fast-mode launch for the three matrices; its prologue adds the
//                      previous FFN output to the residual, RMSNorms it (apply_rmsnorm
//                      :493-507) and quantizes it to Q8_0 (quantize_f32_to_q8_0), recomputed by
//                      every CTA from L2 while its first weight tiles stream in
//   qkv_rope_store     + biases (add_bias :452-465), RoPE Norm/Neox per head
//                      (rope_head_scalar, scalar.rs:92-130), K/V quantized into ring slot
//                      pos % capacity (KvCache::store_key/store_value, kv_cache.rs:93-110)
//   attention          causal GQA decode over the Q8_0 ring, context pos+1
//                      (causal_gqa_decode_scalar_ext, scalar.rs:287-359): split-K kernel
//                      + merge kernel, the merge writing the o projection's Q8_0 input -- 2
//                      launches
//   GEMV o             o = Wo . a
//   GEMV gate,up       one launch; prologue: x += o, RMSNorm (ffn_norm), Q8_0
//   swiglu_q8          silu(gate)*up -> Q8_0 (swiglu_scalar, scalar.rs:161-170)
//   GEMV down
// then the vocab GEMV with the output norm in its prologue (logits, fp32).  With several
// sequences the norm + quantize is a separate add_rmsnorm_q8 launch before each fused GEMV
// (recomputing it per CTA for every sequence costs more than the launch).  The GEMVs run the
// fast mode (gemv_fast_q4_0_q8_0.cu): exact integer block sums, one fp32 FMA per block and a
// fixed lane tree, equal to the AVX2 kernel to fp32 rounding; they dominate the step (the weight
// stream).  RMSNorm sums squares as a tree (the reference sums eight AVX2 lanes sequentially),
// and RoPE / SiLU use CUDA's powf / sinf / cosf / expf, so the activations agree with the
// reference to float rounding, not bit for bit.
// Gemma 2 (arch SULIMO_ARCH_GEMMA2): the embedding rows are scaled by sqrt(embd), every norm is
// weighted by (1 + w), the attention and FFN outputs are RMS-normalized by the layer's post norms
// before their residual adds (inside add_rmsnorm_q8, which always runs as its own launch for
// this architecture), GeGLU replaces SwiGLU and the logits are soft-capped by one more launch.
#include "sulimo_common.cuh"
#include "sulimo_internal.h"

namespace sulimo {
namespace {

constexpr int GLUE_THREADS = 256;
constexpr int NORM_THREADS = 1024;  // one CTA per sequence: the whole vector in one pass

__device__ __forceinline__ float block_sum(float v, float* red) {
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (lane == 0) red[warp] = v;
    __syncthreads();
    float s = 0.0f;
    if (threadIdx.x < 32) {
        s = threadIdx.x < (int)(blockDim.x >> 5) ? red[threadIdx.x] : 0.0f;
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) s += __shfl_xor_sync(0xffffffffu, s, off);
        if (threadIdx.x == 0) red[32] = s;
    }
    __syncthreads();
    return red[32];
}

// One CTA per sequence.  x[seq][E] (+= delta[seq][E] when delta is given, written back), then
// y = (x * 1/sqrt(mean(x^2) + eps)) * w, quantized to Q8_0 (E/32 blocks) as q8 names (row seq).
// F16_OUT: y as f16 [seq][E] into y16 (the prefill GEMMs' activations) instead.
// post_w (Gemma 2's post_attn_norm / post_ffn_norm, forward_pass.rs:330-336, 379-385): delta is
// RMS-normalized with these weights before it is added.  gemma: every norm weight enters as
// (1 + w) (rmsnorm_gemma, avx2.rs:236-268).
template <bool F16_OUT>
__global__ void __launch_bounds__(NORM_THREADS)
    add_rmsnorm_q8_kernel(float* __restrict__ x, const float* __restrict__ delta,
                          const float* __restrict__ w, int E, float eps, const Q8Out q8,
                          __half* __restrict__ y16, const float* __restrict__ post_w, int gemma) {
    pdl_launch_dependents();
    pdl_wait_prerequisites();
    extern __shared__ float sx[];  // E floats + 33 reduction slots
    float* red = sx + E;
    const int seq = blockIdx.x;
    float* xs = x + (size_t)seq * E;
    const float* ds = delta ? delta + (size_t)seq * E : nullptr;
    auto weight = [&](const float* wv, int i) { return gemma ? __fadd_rn(1.0f, wv[i]) : wv[i]; };
    float dscale = 1.0f;
    if (ds && post_w) {
        float sd = 0.0f;
        for (int i = threadIdx.x; i < E; i += blockDim.x) sd = __fmaf_rn(ds[i], ds[i], sd);
        const float dsum = block_sum(sd, red);
        dscale = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(dsum, (float)E), eps)));
        __syncthreads();  // red is reused below
    }
    float ss = 0.0f;
    for (int i = threadIdx.x; i < E; i += blockDim.x) {
        float v = xs[i];
        if (ds) {
            const float d = post_w ? __fmul_rn(__fmul_rn(ds[i], dscale), weight(post_w, i)) : ds[i];
            v = __fadd_rn(v, d);
            xs[i] = v;
        }
        sx[i] = v;
        ss = __fmaf_rn(v, v, ss);
    }
    const float sum_sq = block_sum(ss, red);
    const float mean = __fdiv_rn(sum_sq, (float)E);
    const float scale = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(mean, eps)));
    if (F16_OUT) {
        __half* ys = y16 + (size_t)seq * E;
        for (int i = threadIdx.x; i < E; i += blockDim.x)
            ys[i] = __float2half_rn(__fmul_rn(__fmul_rn(sx[i], scale), weight(w, i)));
        return;
    }
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    for (int b = warp; b < E / 32; b += blockDim.x >> 5) {
        const int i = b * 32 + lane;
        const float y = __fmul_rn(__fmul_rn(sx[i], scale), weight(w, i));
        q8_store_block(q8, y, (size_t)seq, b, lane);
    }
}

// The ordered sum p[0] + p[1] + ... of `splits` float4 partials `stride` floats apart, every
// load of a batch of eight issued before the first add.
__device__ __forceinline__ float4 sum_splits4(const float* p, size_t stride, int splits) {
    float4 acc = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
    for (int z0 = 0; z0 < splits; z0 += 8) {
        float4 v[8];
#pragma unroll
        for (int j = 0; j < 8; j++)
            if (z0 + j < splits)
                v[j] = __ldcg(reinterpret_cast<const float4*>(p + (size_t)(z0 + j) * stride));
#pragma unroll
        for (int j = 0; j < 8; j++) {
            if (z0 + j >= splits) break;
            if (z0 + j == 0) {
                acc = v[j];
            } else {
                acc.x += v[j].x;
                acc.y += v[j].y;
                acc.z += v[j].z;
                acc.w += v[j].w;
            }
        }
    }
    return acc;
}

// A prefill ubatch's residual step after a split-K projection (o or down): x += the ordered
// sum of the projection's fp32 partials (split z of token row t at part + z * split_stride +
// t * E), then RMSNorm(x) * w as f16 — the split-K reduce and add_rmsnorm_q8_kernel<true> in
// one pass.  One CTA per token, four consecutive values per thread (E a multiple of 4): the
// block has E / 4 threads (at most 1024), so every partial of the row is requested at once.
__global__ void __launch_bounds__(1024)
    reduce_add_rmsnorm_f16_kernel(float* __restrict__ x, const float* __restrict__ part,
                                  size_t split_stride, int splits, int E,
                                  const float* __restrict__ w, float eps,
                                  __half* __restrict__ y16) {
    pdl_launch_dependents();
    pdl_wait_prerequisites();
    extern __shared__ float sx[];  // E floats + 33 reduction slots
    float* red = sx + E;
    const int t = blockIdx.x;
    float* xs = x + (size_t)t * E;
    const float* ps = part + (size_t)t * E;
    float ss = 0.0f;
    for (int i = threadIdx.x * 4; i < E; i += blockDim.x * 4) {
        const float4 d = sum_splits4(ps + i, split_stride, splits);
        float4 v = *reinterpret_cast<const float4*>(xs + i);
        v.x = __fadd_rn(v.x, d.x);
        v.y = __fadd_rn(v.y, d.y);
        v.z = __fadd_rn(v.z, d.z);
        v.w = __fadd_rn(v.w, d.w);
        *reinterpret_cast<float4*>(xs + i) = v;
        *reinterpret_cast<float4*>(sx + i) = v;
        ss = __fmaf_rn(v.x, v.x, ss);
        ss = __fmaf_rn(v.y, v.y, ss);
        ss = __fmaf_rn(v.z, v.z, ss);
        ss = __fmaf_rn(v.w, v.w, ss);
    }
    const float sum_sq = block_sum(ss, red);
    const float mean = __fdiv_rn(sum_sq, (float)E);
    const float scale = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(mean, eps)));
    __half* ys = y16 + (size_t)t * E;
    for (int i = threadIdx.x * 4; i < E; i += blockDim.x * 4) {
        const float4 v = *reinterpret_cast<const float4*>(sx + i);
        const __half2 lo = __floats2half2_rn(__fmul_rn(__fmul_rn(v.x, scale), w[i]),
                                             __fmul_rn(__fmul_rn(v.y, scale), w[i + 1]));
        const __half2 hi = __floats2half2_rn(__fmul_rn(__fmul_rn(v.z, scale), w[i + 2]),
                                             __fmul_rn(__fmul_rn(v.w, scale), w[i + 3]));
        *reinterpret_cast<uint2*>(ys + i) = make_uint2(*reinterpret_cast<const uint32_t*>(&lo),
                                                       *reinterpret_cast<const uint32_t*>(&hi));
    }
}

// x[i] *= s (Gemma 2's embedding scale sqrt(embd), forward_pass.rs:210-214)
__global__ void __launch_bounds__(256) scale_kernel(float* __restrict__ x, size_t n, float s) {
    pdl_launch_dependents();
    pdl_wait_prerequisites();
    const size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) x[i] = __fmul_rn(x[i], s);
}

// v = tanh(v * inv_cap) * cap (logit_softcap_scalar, scalar.rs:63-71), in place
__global__ void __launch_bounds__(256)
    logit_softcap_kernel(float* __restrict__ v, size_t n, float inv_cap, float cap) {
    pdl_launch_dependents();
    pdl_wait_prerequisites();
    const size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) v[i] = __fmul_rn(tanhf(__fmul_rn(v[i], inv_cap)), cap);
}

// RoPE of one head in place (rope_head_scalar): pair (2i, 2i+1) in Norm mode (0), (i, i+half)
// in Neox mode (1); theta = pos / base^(2i/rope_dim).
__device__ __forceinline__ void rope_pair(float* v, int i, int half, int mode, float c, float s) {
    const int a = mode == 0 ? 2 * i : i, b = mode == 0 ? 2 * i + 1 : i + half;
    const float v0 = v[a], v1 = v[b];
    v[a] = __fsub_rn(__fmul_rn(v0, c), __fmul_rn(v1, s));
    v[b] = __fadd_rn(__fmul_rn(v0, s), __fmul_rn(v1, c));
}

// One CTA per (head, sequence) over the q heads, then the k heads, then the v heads: bias add,
// RoPE (q and k; angles pos / base^(2i/rope_dim) per pair), then q written back as f32 for the
// attention and k / v quantized into the sequence's rings at slot pos % capacity (kv head h at
// block h*hd/32 of the slot).
__global__ void __launch_bounds__(128)
    qkv_rope_store_kernel(float* __restrict__ q, const float* __restrict__ k,
                          const float* __restrict__ v, const float* __restrict__ bq,
                          const float* __restrict__ bk, const float* __restrict__ bv, int H,
                          int Hkv, int hd, int rope_dim, int mode, float base, size_t pos0,
                          size_t pos_step, uint8_t* __restrict__ k_ring,
                          uint8_t* __restrict__ v_ring, size_t capacity, size_t seq_stride) {
    pdl_launch_dependents();
    pdl_wait_prerequisites();
    __shared__ float sv[256];
    // blockIdx.y: a sequence of a decode batch (pos_step 0, own ring) or a token of a prefill
    // ubatch (pos_step 1, one ring)
    const int head = blockIdx.x, seq = blockIdx.y;
    const size_t pos = pos0 + (size_t)seq * pos_step;
    const int kind = head < H ? 0 : (head < H + Hkv ? 1 : 2);  // q, k, v
    const int hh = kind == 0 ? head : (kind == 1 ? head - H : head - H - Hkv);
    const int dim = kind == 0 ? H * hd : Hkv * hd;
    const float* src = kind == 0 ? q : (kind == 1 ? k : v);
    const float* bias = kind == 0 ? bq : (kind == 1 ? bk : bv);
    const float* vec = src + (size_t)seq * dim + (size_t)hh * hd;
    for (int i = threadIdx.x; i < hd; i += blockDim.x) {
        const float x = vec[i];
        sv[i] = bias ? __fadd_rn(x, bias[hh * hd + i]) : x;
    }
    __syncthreads();
    if (kind < 2) {
        const int half = rope_dim / 2;
        for (int i = threadIdx.x; i < half; i += blockDim.x) {
            const float freq =
                __fdiv_rn(1.0f, powf(base, __fdiv_rn((float)(2 * i), (float)rope_dim)));
            const float theta = __fmul_rn((float)pos, freq);
            rope_pair(sv, i, half, mode, cosf(theta), sinf(theta));
        }
        __syncthreads();
    }
    if (kind == 0) {
        float* dst = q + (size_t)seq * dim + (size_t)hh * hd;
        for (int i = threadIdx.x; i < hd; i += blockDim.x) dst[i] = sv[i];
        return;
    }
    const size_t bpp = (size_t)Hkv * hd / 32;
    uint8_t* ring = (kind == 1 ? k_ring : v_ring) + (size_t)seq * seq_stride +
                    (pos % capacity) * bpp * 34 + (size_t)hh * (hd / 32) * 34;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    for (int b = warp; b < hd / 32; b += blockDim.x >> 5)
        quantize_block_warp(sv[b * 32 + lane], ring + b * 34, lane);
}

// A prefill ubatch's q / k / v from the stacked GEMM: its fp32 split-K partials
// [splits][n][qd + 2 kvd] summed in split order, then per token what qkv_rope_store_kernel does
// (bias, RoPE of the q and k heads, q written as f32, k and v quantized into the ring at slot
// pos % capacity).  One CTA per token: the row in shared memory, the angles of each rotary
// frequency computed once and used by every head; (qd + 2 kvd) / 4 threads (at most 1024), so
// every partial of the row is requested at once.
__global__ void __launch_bounds__(1024)
    qkv_reduce_rope_store_kernel(const float* __restrict__ part, int splits, int n,
                                 const float* __restrict__ bq, const float* __restrict__ bk,
                                 const float* __restrict__ bv, int H, int Hkv, int hd,
                                 int rope_dim, int mode, float base, size_t pos0,
                                 float* __restrict__ q, uint8_t* __restrict__ k_ring,
                                 uint8_t* __restrict__ v_ring, size_t capacity) {
    pdl_launch_dependents();
    pdl_wait_prerequisites();
    extern __shared__ float qkv_row[];  // [qd + 2 kvd], then cos and sin [rope_dim / 2] each
    const int qd = H * hd, kvd = Hkv * hd, mt = qd + 2 * kvd, half = rope_dim / 2;
    const int t = blockIdx.x;
    const size_t pos = pos0 + (size_t)t;
    float* cs = qkv_row + mt;
    float* sn = cs + half;
    const size_t nm = (size_t)n * mt;
    const float* src = part + (size_t)t * mt;
    for (int j = threadIdx.x * 4; j < mt; j += blockDim.x * 4) {
        float4 acc = sum_splits4(src + j, nm, splits);
        // qd and kvd are multiples of 4: a group of four lies in one of q, k, v
        const float* b = j < qd ? (bq ? bq + j : nullptr)
                                : (j < qd + kvd ? (bk ? bk + (j - qd) : nullptr)
                                                : (bv ? bv + (j - qd - kvd) : nullptr));
        if (b) {
            acc.x = __fadd_rn(acc.x, b[0]);
            acc.y = __fadd_rn(acc.y, b[1]);
            acc.z = __fadd_rn(acc.z, b[2]);
            acc.w = __fadd_rn(acc.w, b[3]);
        }
        *reinterpret_cast<float4*>(qkv_row + j) = acc;
    }
    for (int i = threadIdx.x; i < half; i += blockDim.x) {
        const float freq =
            __fdiv_rn(1.0f, powf(base, __fdiv_rn((float)(2 * i), (float)rope_dim)));
        const float theta = __fmul_rn((float)pos, freq);
        cs[i] = cosf(theta);
        sn[i] = sinf(theta);
    }
    __syncthreads();
    // the q heads then the k heads lie back to back: head hh at hh * hd
    for (int w = threadIdx.x; w < (H + Hkv) * half; w += blockDim.x) {
        const int hh = w / half, i = w % half;
        rope_pair(qkv_row + hh * hd, i, half, mode, cs[i], sn[i]);
    }
    __syncthreads();
    float* qdst = q + (size_t)t * qd;
    for (int j = threadIdx.x * 4; j < qd; j += blockDim.x * 4)
        *reinterpret_cast<float4*>(qdst + j) = *reinterpret_cast<const float4*>(qkv_row + j);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int kb = kvd / 32;  // Q8_0 blocks of one tensor per slot
    const size_t slot = (pos % capacity) * (size_t)kb * 34;
    for (int b = warp; b < 2 * kb; b += blockDim.x >> 5) {
        const bool isv = b >= kb;
        const int bb = isv ? b - kb : b;
        quantize_block_warp(qkv_row[qd + (isv ? kvd : 0) + bb * 32 + lane],
                            (isv ? v_ring : k_ring) + slot + (size_t)bb * 34, lane);
    }
}

// silu(gate) * up -> f16 (the prefill down-projection GEMM's activations), 4 elements per
// thread: 16-byte loads and an 8-byte store (n4 = n / 4; the buffers are 16-byte aligned).
__device__ __forceinline__ float silu_mul(float g, float u) {
    return __fmul_rn(__fdiv_rn(g, __fadd_rn(1.0f, expf(-g))), u);
}

__global__ void __launch_bounds__(GLUE_THREADS)
    swiglu_f16_kernel(const float4* __restrict__ gate, const float4* __restrict__ up, size_t n4,
                      uint2* __restrict__ out) {
    pdl_launch_dependents();
    pdl_wait_prerequisites();
    const size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n4) return;
    const float4 g = gate[i], u = up[i];
    const __half2 lo = __floats2half2_rn(silu_mul(g.x, u.x), silu_mul(g.y, u.y));
    const __half2 hi = __floats2half2_rn(silu_mul(g.z, u.z), silu_mul(g.w, u.w));
    out[i] = make_uint2(*reinterpret_cast<const uint32_t*>(&lo),
                        *reinterpret_cast<const uint32_t*>(&hi));
}

// The token list of repack_context (crates/sulimo-engine/src/scheduler.rs:316-326): the first
// sys_len tokens, then the last recent_len.
__global__ void __launch_bounds__(GLUE_THREADS)
    gather_context_kernel(const int32_t* __restrict__ past, size_t n_past, size_t sys_len,
                          size_t recent_len, int32_t* __restrict__ out) {
    pdl_launch_dependents();
    pdl_wait_prerequisites();
    const size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= sys_len + recent_len) return;
    out[i] = i < sys_len ? past[i] : past[n_past - recent_len + (i - sys_len)];
}

// f16 [n4 * 4] -> f32: a prefill ubatch's caller-written f16 embeddings into the fp32 residual.
__global__ void __launch_bounds__(GLUE_THREADS)
    widen_f16_kernel(const uint2* __restrict__ in, size_t n4, float4* __restrict__ out) {
    pdl_launch_dependents();
    pdl_wait_prerequisites();
    const size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n4) return;
    const uint2 v = in[i];
    const float2 lo = __half22float2(*reinterpret_cast<const __half2*>(&v.x));
    const float2 hi = __half22float2(*reinterpret_cast<const __half2*>(&v.y));
    out[i] = make_float4(lo.x, lo.y, hi.x, hi.y);
}

// silu(gate) * up (swiglu_scalar) or, for Gemma 2, gelu(gate) * up with the tanh form of
// geglu_scalar (scalar.rs:77-89) -> Q8_0 (rows of F = q8.K values): one warp per 32-value block,
// all sequences' blocks in one grid.
__global__ void __launch_bounds__(GLUE_THREADS)
    swiglu_q8_kernel(const float* __restrict__ gate, const float* __restrict__ up, size_t nblocks,
                     const Q8Out q8, int geglu) {
    pdl_launch_dependents();
    pdl_wait_prerequisites();
    const int lane = threadIdx.x & 31;
    size_t b = (size_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    if (b >= nblocks) return;
    const float g = gate[b * 32 + lane];
    float act;
    if (geglu) {
        const float cube = __fmul_rn(__fmul_rn(g, g), g);
        const float inner = __fmul_rn(0.7978846f, __fadd_rn(g, __fmul_rn(0.044715f, cube)));
        act = __fmul_rn(__fmul_rn(0.5f, g), __fadd_rn(1.0f, tanhf(inner)));
    } else {
        act = __fdiv_rn(g, __fadd_rn(1.0f, expf(-g)));
    }
    const size_t nb = (size_t)(q8.K / 32);
    q8_store_block(q8, __fmul_rn(act, up[b * 32 + lane]), b / nb, (int)(b % nb), lane);
}

// First index of the maximum of each row (greedy sampling); NaN never wins.  ARGMAX_CTAS CTAs
// per row each scan a column range and publish their (max, first index); the last CTA of a
// row to finish (a per-row counter) folds the partials in range order, writes the index and
// resets the counter for the next launch.
constexpr int ARGMAX_CTAS = 32;

__device__ __forceinline__ void argmax_merge(float& best, int& idx, float v, int i) {
    if (v > best || (v == best && i < idx)) {
        best = v;
        idx = i;
    }
}

__global__ void __launch_bounds__(GLUE_THREADS)
    argmax_rows_kernel(const float* __restrict__ x, int cols, float* __restrict__ part_v,
                       int* __restrict__ part_i, unsigned* __restrict__ counters,
                       int32_t* __restrict__ out) {
    pdl_launch_dependents();
    pdl_wait_prerequisites();
    __shared__ float bv[GLUE_THREADS / 32];
    __shared__ int bi[GLUE_THREADS / 32];
    __shared__ bool last;
    const int row = blockIdx.y, c = blockIdx.x;
    const int per = (cols + ARGMAX_CTAS - 1) / ARGMAX_CTAS;
    const int c0 = c * per, c1 = min(cols, c0 + per);
    const float* r = x + (size_t)row * cols;
    float best = -INFINITY;
    int idx = 0x7fffffff;
    for (int i = c0 + threadIdx.x; i < c1; i += blockDim.x) argmax_merge(best, idx, r[i], i);
#pragma unroll
    for (int off = 16; off > 0; off >>= 1)
        argmax_merge(best, idx, __shfl_xor_sync(0xffffffffu, best, off),
                     __shfl_xor_sync(0xffffffffu, idx, off));
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (lane == 0) {
        bv[warp] = best;
        bi[warp] = idx;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        for (int w = 1; w < GLUE_THREADS / 32; w++) argmax_merge(best, idx, bv[w], bi[w]);
        part_v[row * ARGMAX_CTAS + c] = best;
        part_i[row * ARGMAX_CTAS + c] = idx;
        __threadfence();
        last = atomicAdd(&counters[row], 1u) == ARGMAX_CTAS - 1;
    }
    __syncthreads();
    if (last && threadIdx.x == 0) {
        __threadfence();
        float b = -INFINITY;
        int k = 0x7fffffff;
        for (int w = 0; w < ARGMAX_CTAS; w++)
            argmax_merge(b, k, __ldcg(part_v + row * ARGMAX_CTAS + w),
                         __ldcg(part_i + row * ARGMAX_CTAS + w));
        out[row] = k == 0x7fffffff ? 0 : k;
        counters[row] = 0u;
    }
}

struct Scratch {
    float *x, *q, *k, *v, *att, *o, *g, *u;
    uint8_t* q8;
    float* x2;   // the residual stream's second buffer (fused norms write x + delta here)
    void* q8s;   // staged Q8_0 activations for the batched tensor-core matvec
};

size_t align256(size_t b) { return (b + 255) / 256 * 256; }

// Carves the caller's scratch (the reference's ScratchBuffers, forward_pass.rs:150-186, plus the
// staged activation form of the batched matvec).
size_t scratch_layout(const sulimo_model_desc* m, int batch, uint8_t* base, Scratch* s) {
    const size_t E = m->embd, F = m->ffn, qd = (size_t)m->head_count * m->head_dim;
    const size_t kvd = (size_t)m->head_count_kv * m->head_dim;
    size_t q8n = E > qd ? E : qd;
    if (F > q8n) q8n = F;
    const size_t sizes[10] = {E * 4, qd * 4, kvd * 4, kvd * 4, qd * 4, (E > F ? E : F) * 4,
                              F * 4, F * 4, q8n / 32 * 34, E * 4};
    size_t off = 0;
    uint8_t* p[11];
    for (int i = 0; i < 10; i++) {
        p[i] = base ? base + off : nullptr;
        off += align256(sizes[i] * (size_t)batch);
    }
    p[10] = base ? base + off : nullptr;
    off += align256(q8_staged_bytes(batch, (int)q8n));
    if (s) {
        s->x = reinterpret_cast<float*>(p[0]);
        s->q = reinterpret_cast<float*>(p[1]);
        s->k = reinterpret_cast<float*>(p[2]);
        s->v = reinterpret_cast<float*>(p[3]);
        s->att = reinterpret_cast<float*>(p[4]);
        s->o = reinterpret_cast<float*>(p[5]);
        s->g = reinterpret_cast<float*>(p[6]);
        s->u = reinterpret_cast<float*>(p[7]);
        s->q8 = p[8];
        s->x2 = reinterpret_cast<float*>(p[9]);
        s->q8s = p[10];
    }
    return off;
}

// The RMSNorm kernels keep the whole vector in shared memory (up to 227 KB per CTA).
int ensure_norm_attr(sulimo_ctx* ctx) {
    static DeviceBits done;
    if (done.test(ctx->device)) return SULIMO_OK;
    int st = check_cuda(cudaFuncSetAttribute(add_rmsnorm_q8_kernel<false>,
                                             cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             227 * 1024),
                        "rmsnorm smem attribute");
    if (!st)
        st = check_cuda(cudaFuncSetAttribute(add_rmsnorm_q8_kernel<true>,
                                             cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             227 * 1024),
                        "rmsnorm smem attribute");
    if (!st)
        st = check_cuda(cudaFuncSetAttribute(reduce_add_rmsnorm_f16_kernel,
                                             cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             227 * 1024),
                        "rmsnorm smem attribute");
    if (!st) done.set(ctx->device);
    return st;
}

// Threads of a one-row-per-CTA kernel over `width` floats, four per thread: a multiple of 32,
// at most 1024.
unsigned row_threads(int width) {
    const int t = (width / 4 + 31) / 32 * 32;
    return (unsigned)(t < 32 ? 32 : (t > 1024 ? 1024 : t));
}

// Prefill scratch: x, q, k, v, o, gate, up (f32 [n][dim]) and one f16 activation buffer
// [n][max(embd, q dim, ffn)] shared by the norm, attention and SwiGLU outputs.
struct PrefillScratch {
    float *x, *q, *k, *v, *o, *g, *u;
    __half* h;
};

size_t prefill_layout(const sulimo_model_desc* m, int n, uint8_t* base, PrefillScratch* s) {
    const size_t E = m->embd, F = m->ffn, qd = (size_t)m->head_count * m->head_dim;
    const size_t kvd = (size_t)m->head_count_kv * m->head_dim;
    size_t hn = E > qd ? E : qd;
    if (F > hn) hn = F;
    const size_t sizes[8] = {E * 4, qd * 4, kvd * 4, kvd * 4, E * 4, F * 4, F * 4, hn * 2};
    uint8_t* p[8];
    size_t off = 0;
    for (int i = 0; i < 8; i++) {
        p[i] = base ? base + off : nullptr;
        off += align256(sizes[i] * (size_t)n);
    }
    if (s) {
        s->x = reinterpret_cast<float*>(p[0]);
        s->q = reinterpret_cast<float*>(p[1]);
        s->k = reinterpret_cast<float*>(p[2]);
        s->v = reinterpret_cast<float*>(p[3]);
        s->o = reinterpret_cast<float*>(p[4]);
        s->g = reinterpret_cast<float*>(p[5]);
        s->u = reinterpret_cast<float*>(p[6]);
        s->h = reinterpret_cast<__half*>(p[7]);
    }
    return off;
}

}  // namespace

size_t prefill_scratch_bytes(const sulimo_model_desc* m, int n) {
    return prefill_layout(m, n, nullptr, nullptr);
}

// One prefill ubatch of n tokens at positions start_pos .. start_pos+n-1 of one sequence
// (execute_prefill_ubatch, crates/sulimo-ocl/src/prefill.rs:337-566): per layer residual +
// RMSNorm -> f16, q/k/v projections, biases + RoPE + K/V ring store for every token, causal
// prefill attention (f16 out), o projection, residual + RMSNorm, gate/up projections with
// SwiGLU (f16), down projection; then the last token's residual, final norm and the vocab
// projection (enqueue_logits_final, prefill.rs:300-330) into logits[vocab].  Where the CTA-pair
// GEMM takes the shapes, q/k/v are one stacked GEMM whose split-K partials the RoPE / ring-store
// kernel sums, the o and down partials are summed by the residual + RMSNorm kernel that follows
// them, and gate/up run as one gated GEMM that writes silu(gate)*up; otherwise each projection
// is its own GEMM with its own reduce.  The reference's GPU ubatch skips the QKV biases and keeps
// activations in f16; this one adds the biases (as forward_token does) and keeps the residual
// stream in fp32.
int launch_prefill_ubatch(sulimo_ctx* ctx, const sulimo_model_desc* m, const int32_t* tokens,
                          const void* x_f16, int n, size_t start_pos, float* logits,
                          void* scratch) {
    PrefillScratch s;
    prefill_layout(m, n, reinterpret_cast<uint8_t*>(scratch), &s);
    const int E = m->embd, F = m->ffn, H = m->head_count, Hkv = m->head_count_kv,
              hd = m->head_dim;
    const int qd = H * hd, kvd = Hkv * hd;
    const size_t norm_smem = (size_t)(E + 33) * sizeof(float);
    __half* h16 = reinterpret_cast<__half*>(s.h);
    const Q8Out no_q8 = {nullptr, nullptr, nullptr, 0};
    int st;
    if ((st = ensure_norm_attr(ctx))) return st;
    if (tokens) {
        if ((st = launch_dequant_rows(ctx, m->tok_scales, m->tok_quants, E, tokens, n, s.x,
                                      DEQUANT_F16_WIDE)))
            return st;
    } else {
        const size_t nh4 = (size_t)n * E / 4;  // E is a multiple of 32
        (void)launch_pdl(widen_f16_kernel,
                         dim3((unsigned)((nh4 + GLUE_THREADS - 1) / GLUE_THREADS)),
                         dim3(GLUE_THREADS), 0, ctx->stream, reinterpret_cast<const uint2*>(x_f16),
                         nh4, reinterpret_cast<float4*>(s.x));
        ctx->launches++;
        if ((st = check_cuda(cudaGetLastError(), "widen_f16 launch"))) return st;
    }
    auto gemm = [&](const void* sc, const void* qu, const void* x, float* out, int rows, int k) {
        return launch_gemm_q4_0_f16(ctx, sc, qu, x, out, rows, k, n, SULIMO_OUT_F32, k, 0);
    };
    // q, k and v as one stacked GEMM (split-K partials summed by the RoPE / ring-store kernel)
    // where the shapes allow; three GEMMs and qkv_rope_store_kernel otherwise
    const size_t qkv_smem = (size_t)(qd + 2 * kvd + m->rope_dim) * sizeof(float);
    bool stacked_qkv = qkv_smem <= 48 * 1024;
    if (stacked_qkv) {
        const GemmSeg probe[3] = {{m->layers[0].wq_scales, m->layers[0].wq_quants, qd},
                                  {m->layers[0].wk_scales, m->layers[0].wk_quants, kvd},
                                  {m->layers[0].wv_scales, m->layers[0].wv_quants, kvd}};
        stacked_qkv = gemm_stacked_applies(probe, 3, E, n);
    }
    // the o and down projections as split-K partials summed by the residual + RMSNorm kernel
    // that follows each, where the pair GEMM takes their shapes
    const GemmSeg o_shape{nullptr, nullptr, E};
    const bool fused_o = E % 4 == 0 && gemm_stacked_applies(&o_shape, 1, qd, n);
    const bool fused_d = E % 4 == 0 && gemm_stacked_applies(&o_shape, 1, F, n);
    // gate and up as one gated pair GEMM writing silu(gate) * up as f16 where it applies
    const bool gated = gemm_gated_applies(F, E, n);
    // the residual update still to apply: a projection's dense output, or its partials
    const float* pending = nullptr;
    const float* pend_part = nullptr;
    int pend_splits = 0;
    auto residual_norm = [&](float* x, const float* dense, const float* part, int splits,
                             const void* w, int rows) -> int {
        if (part)
            (void)launch_pdl(reduce_add_rmsnorm_f16_kernel, dim3(rows), dim3(row_threads(E)),
                             norm_smem,
                             ctx->stream, x, part, (size_t)n * E, splits, E,
                             reinterpret_cast<const float*>(w), m->eps, h16);
        else
            (void)launch_pdl(add_rmsnorm_q8_kernel<true>, dim3(rows), dim3(NORM_THREADS),
                             norm_smem, ctx->stream, x, dense, reinterpret_cast<const float*>(w),
                             E, m->eps, no_q8, h16, (const float*)nullptr, 0);
        ctx->launches++;
        return check_cuda(cudaGetLastError(), "residual norm launch");
    };
    for (int l = 0; l < m->n_layers; l++) {
        const sulimo_layer_desc& L = m->layers[l];
        if ((st = residual_norm(s.x, pending, pend_part, pend_splits, L.attn_norm, n))) return st;
        if (stacked_qkv) {
            const GemmSeg qkv[3] = {{L.wq_scales, L.wq_quants, qd},
                                    {L.wk_scales, L.wk_quants, kvd},
                                    {L.wv_scales, L.wv_quants, kvd}};
            const float* part = nullptr;
            int splits = 0;
            if ((st = launch_gemm_pair_stacked(ctx, qkv, 3, s.h, E, n, &part, &splits)))
                return st;
            (void)launch_pdl(qkv_reduce_rope_store_kernel, dim3(n),
                             dim3(row_threads(qd + 2 * kvd)), qkv_smem,
                             ctx->stream, part, splits, n, reinterpret_cast<const float*>(L.bq),
                             reinterpret_cast<const float*>(L.bk),
                             reinterpret_cast<const float*>(L.bv), H, Hkv, hd, m->rope_dim,
                             m->rope_mode, m->rope_base, start_pos, s.q,
                             reinterpret_cast<uint8_t*>(L.k_ring),
                             reinterpret_cast<uint8_t*>(L.v_ring), m->kv_capacity);
        } else {
            if ((st = gemm(L.wq_scales, L.wq_quants, s.h, s.q, qd, E)) ||
                (st = gemm(L.wk_scales, L.wk_quants, s.h, s.k, kvd, E)) ||
                (st = gemm(L.wv_scales, L.wv_quants, s.h, s.v, kvd, E)))
                return st;
            (void)launch_pdl(qkv_rope_store_kernel, dim3(H + 2 * Hkv, n), dim3(128), 0,
                             ctx->stream, s.q, (const float*)s.k, (const float*)s.v,
                             reinterpret_cast<const float*>(L.bq),
                             reinterpret_cast<const float*>(L.bk),
                             reinterpret_cast<const float*>(L.bv), H, Hkv, hd, m->rope_dim,
                             m->rope_mode, m->rope_base, start_pos, (size_t)1,
                             reinterpret_cast<uint8_t*>(L.k_ring),
                             reinterpret_cast<uint8_t*>(L.v_ring), m->kv_capacity, (size_t)0);
        }
        ctx->launches++;
        if ((st = check_cuda(cudaGetLastError(), "qkv_rope_store launch"))) return st;
        if ((st = launch_attn_prefill(ctx, s.q, L.k_ring, L.v_ring, start_pos, m->kv_capacity, n,
                                      H, Hkv, hd, s.h)))
            return st;
        if (fused_o) {
            const GemmSeg wo{L.wo_scales, L.wo_quants, E};
            const float* part = nullptr;
            int splits = 0;
            if ((st = launch_gemm_pair_stacked(ctx, &wo, 1, s.h, qd, n, &part, &splits)) ||
                (st = residual_norm(s.x, nullptr, part, splits, L.ffn_norm, n)))
                return st;
        } else if ((st = gemm(L.wo_scales, L.wo_quants, s.h, s.o, E, qd)) ||
                   (st = residual_norm(s.x, s.o, nullptr, 0, L.ffn_norm, n))) {
            return st;
        }
        if (gated) {
            // f16 [n][F] into s.g: other CTAs may still be reading the activations in s.h
            if ((st = launch_gemm_pair_gated(ctx, GemmSeg{L.wg_scales, L.wg_quants, F},
                                             GemmSeg{L.wu_scales, L.wu_quants, F}, s.h, E, n,
                                             s.g)))
                return st;
        } else {
            if ((st = gemm(L.wg_scales, L.wg_quants, s.h, s.g, F, E)) ||
                (st = gemm(L.wu_scales, L.wu_quants, s.h, s.u, F, E)))
                return st;
            const size_t nf4 = (size_t)n * F / 4;  // F is a multiple of 32
            (void)launch_pdl(swiglu_f16_kernel,
                             dim3((unsigned)((nf4 + GLUE_THREADS - 1) / GLUE_THREADS)),
                             dim3(GLUE_THREADS), 0, ctx->stream,
                             reinterpret_cast<const float4*>(s.g),
                             reinterpret_cast<const float4*>(s.u), nf4,
                             reinterpret_cast<uint2*>(s.h));
            ctx->launches++;
            if ((st = check_cuda(cudaGetLastError(), "swiglu_f16 launch"))) return st;
        }
        const void* ffn_act = gated ? static_cast<const void*>(s.g) : static_cast<const void*>(s.h);
        if (fused_d) {
            const GemmSeg wd{L.wd_scales, L.wd_quants, E};
            if ((st = launch_gemm_pair_stacked(ctx, &wd, 1, ffn_act, F, n, &pend_part,
                                               &pend_splits)))
                return st;
            pending = nullptr;
        } else {
            if ((st = gemm(L.wd_scales, L.wd_quants, ffn_act, s.o, E, F))) return st;
            pending = s.o;
            pend_part = nullptr;
        }
    }
    // the last token only: residual, final norm, vocab projection (fp32 logits)
    const size_t last = (size_t)(n - 1) * E;
    if ((st = residual_norm(s.x + last, pending ? pending + last : nullptr,
                            pend_part ? pend_part + last : nullptr, pend_splits, m->out_norm, 1)))
        return st;
    return launch_gemm_q4_0_f16(ctx, m->out_scales, m->out_quants, s.h, logits, m->vocab, E, 1,
                                SULIMO_OUT_F32, E, 0);
}

void repack_context_plan(size_t n_past, size_t capacity, size_t* sys_len, size_t* recent_len) {
    size_t s = capacity / 8;
    s = s < 4 ? 4 : (s > 64 ? 64 : s);
    if (s > n_past) s = n_past;
    size_t r = capacity / 2;
    if (r > n_past - s) r = n_past - s;
    *sys_len = s;
    *recent_len = r;
}

// repack_context + the re-prefill from position 0 that follows it (engine.rs:226-239), with the
// token list gathered on the device: ubatches of at most `ubatch` tokens of new_tokens (no host
// round trip), the last one's logits in `logits`.
int launch_repack_context(sulimo_ctx* ctx, const sulimo_model_desc* m, const int32_t* past,
                          size_t n_past, int32_t* new_tokens, int ubatch, float* logits,
                          void* scratch, size_t* new_pos) {
    size_t sys_len, recent_len;
    repack_context_plan(n_past, m->kv_capacity, &sys_len, &recent_len);
    const size_t n = sys_len + recent_len;
    *new_pos = n;
    if (n == 0) return SULIMO_OK;
    (void)launch_pdl(gather_context_kernel,
                     dim3((unsigned)((n + GLUE_THREADS - 1) / GLUE_THREADS)), dim3(GLUE_THREADS),
                     0, ctx->stream, past, n_past, sys_len, recent_len, new_tokens);
    ctx->launches++;
    int st = check_cuda(cudaGetLastError(), "gather_context launch");
    for (size_t p0 = 0; !st && p0 < n; p0 += (size_t)ubatch) {
        const int cnt = (int)(n - p0 < (size_t)ubatch ? n - p0 : (size_t)ubatch);
        st = launch_prefill_ubatch(ctx, m, new_tokens + p0, nullptr, cnt, p0, logits, scratch);
    }
    return st;
}

size_t forward_scratch_bytes(const sulimo_model_desc* m, int batch) {
    return scratch_layout(m, batch, nullptr, nullptr);
}

int launch_argmax_rows(sulimo_ctx* ctx, const float* x, int rows, int cols, int32_t* out) {
    // per-row partials + counters in a context-owned buffer (grown outside graph capture by a
    // first call; counters start and end at zero)
    const size_t need = (size_t)rows * (ARGMAX_CTAS * 8 + 4);
    if (need > ctx->argmax_bytes) {
        int st = check_cuda(cudaStreamSynchronize(ctx->stream), "argmax scratch sync");
        if (st) return st;
        if (ctx->argmax_scratch) cudaFree(ctx->argmax_scratch);
        ctx->argmax_scratch = nullptr;
        ctx->argmax_bytes = 0;
        if ((st = check_cuda(cudaMalloc(&ctx->argmax_scratch, need), "argmax scratch"))) return st;
        if ((st = check_cuda(cudaMemset(ctx->argmax_scratch, 0, need), "argmax scratch"))) return st;
        ctx->argmax_bytes = need;
    }
    uint8_t* base = reinterpret_cast<uint8_t*>(ctx->argmax_scratch);
    float* pv = reinterpret_cast<float*>(base);
    int* pi = reinterpret_cast<int*>(base + (size_t)rows * ARGMAX_CTAS * 4);
    unsigned* cnt = reinterpret_cast<unsigned*>(base + (size_t)rows * ARGMAX_CTAS * 8);
    (void)launch_pdl(argmax_rows_kernel, dim3(ARGMAX_CTAS, rows), dim3(GLUE_THREADS), 0,
                     ctx->stream, x, cols, pv, pi, cnt, out);
    ctx->launches++;
    return check_cuda(cudaGetLastError(), "argmax_rows launch");
}

// The Q8_0 form a decode step's producer writes for the matvec over g: the staged form when the
// batched tensor-core matvec takes it, else the block array.
static Q8Out step_q8_form(sulimo_ctx* ctx, const Scratch& s, const GemvMatSrc* g, int count,
                          int K, int batch) {
    if (batch >= GEMV_MMA_MIN_BATCH && ((uintptr_t)s.q8s % 16) == 0 &&
        gemv_mma_applies(g, count, K, batch, ctx->num_sms))
        return q8_staged_view(s.q8s, batch, K);
    const Q8Out o = {s.q8, nullptr, nullptr, K};
    return o;
}

// The fast-mode matvec over a decode step's static weights, from the form the producer wrote.
static int step_gemv(sulimo_ctx* ctx, const GemvMatSrc* g, int count, const Q8Out& x, int K,
                     int batch) {
    if (x.codes) return launch_gemv_mma_group(ctx, g, count, x, K, batch, true);
    return launch_gemv_fast_group(ctx, g, count, x.aos, K, batch, true);
}

// Residual add + RMSNorm + Q8_0 feeding `count` matrices.  For one sequence the norm is
// folded into the matvec's prologue (each CTA recomputes it from L2 while its weights stream
// in; v = x + delta goes to the other residual buffer when keep_x, which becomes x).  With more
// sequences that redundant per-CTA work costs more than the launch it saves (measured on
// config 4: batch 1 1.48 -> 1.40 ms per step, batch 8 5.19 -> 6.41 ms), so the norm kernel
// updates x in place and writes the activations, then the matvec runs.
// Gemma 2 (post_w: the delta's post norm; gemma: (1 + w) norm weights) always takes the
// separate norm kernel.
static int norm_and_gemv(sulimo_ctx* ctx, const Scratch& s, float*& x, float*& x_other,
                         const float* delta, const float* w, float eps, int E, int batch,
                         const GemvMatSrc* g, int count, bool keep_x,
                         const float* post_w = nullptr, int gemma = 0) {
    const GemvPrologue pro = {GEMV_PRO_NORM, x, delta, w, keep_x ? x_other : nullptr, eps};
    if (batch == 1 && !gemma && !post_w && gemv_fast_fused_ok(g, count, E, batch, pro)) {
        const int st = launch_gemv_fast_fused(ctx, g, count, pro, E, batch, true);
        if (!st && keep_x) {
            float* t = x;
            x = x_other;
            x_other = t;
        }
        return st;
    }
    const Q8Out form = step_q8_form(ctx, s, g, count, E, batch);
    (void)launch_pdl(add_rmsnorm_q8_kernel<false>, dim3(batch), dim3(NORM_THREADS),
                     (size_t)(E + 33) * sizeof(float), ctx->stream, x, delta, w, E, eps, form,
                     (__half*)nullptr, post_w, gemma);
    ctx->launches++;
    int st = check_cuda(cudaGetLastError(), "add_rmsnorm_q8 launch");
    return st ? st : step_gemv(ctx, g, count, form, E, batch);
}

// SwiGLU + Q8_0 feeding the down projection.  Folding it into the matvec's prologue, as the
// norm is, was measured slower at every batch size (config 4 batch 1: 1.48 -> 1.61 ms per
// step): every CTA of the down projection (hundreds) would recompute all F activations with
// expf, so this one small kernel runs instead.
static int swiglu_and_gemv(sulimo_ctx* ctx, const Scratch& s, const float* gate, const float* up,
                           int F, int batch, const GemvMatSrc& g, int geglu) {
    const size_t nblk = (size_t)batch * F / 32;
    const Q8Out form = step_q8_form(ctx, s, &g, 1, F, batch);
    (void)launch_pdl(swiglu_q8_kernel, dim3((unsigned)((nblk + 7) / 8)), dim3(GLUE_THREADS), 0,
                     ctx->stream, gate, up, nblk, form, geglu);
    ctx->launches++;
    int st = check_cuda(cudaGetLastError(), "swiglu_q8 launch");
    return st ? st : step_gemv(ctx, &g, 1, form, F, batch);
}

int launch_forward_token(sulimo_ctx* ctx, const sulimo_model_desc* m, const int32_t* tokens,
                         int batch, size_t pos, float* logits, void* scratch) {
    Scratch s;
    scratch_layout(m, batch, reinterpret_cast<uint8_t*>(scratch), &s);
    const int E = m->embd, F = m->ffn, H = m->head_count, Hkv = m->head_count_kv,
              hd = m->head_dim;
    const int qd = H * hd, kvd = Hkv * hd;
    const size_t ctx_len = pos + 1;
    int st;
    if ((st = ensure_norm_attr(ctx))) return st;
    // attention workspace for this geometry (grown outside any graph capture by a first call)
    int splits = 0;
    const sulimo_layer_desc& L0 = m->layers[0];
    const size_t pbytes = attn_decode_partial_bytes(ctx_len, m->kv_capacity, H, Hkv, hd, batch,
                                                    ctx->num_sms, m->kv_seq_stride, L0.k_ring,
                                                    L0.v_ring, &splits);
    if ((st = ensure_workspace(ctx, pbytes))) return st;

    // x = token_embd[token] (lookup_token_embedding, forward_pass.rs:419-450: exact f32 dequant)
    if ((st = launch_dequant_rows(ctx, m->tok_scales, m->tok_quants, E, tokens, batch, s.x,
                                  SULIMO_OUT_F32)))
        return st;
    const int gemma = m->arch == SULIMO_ARCH_GEMMA2;
    if (gemma) {  // x *= sqrt(embd) (forward_pass.rs:210-214)
        const size_t n = (size_t)batch * E;
        (void)launch_pdl(scale_kernel, dim3((unsigned)((n + 255) / 256)), dim3(256), 0,
                         ctx->stream, s.x, n, sqrtf((float)E));
        ctx->launches++;
        if ((st = check_cuda(cudaGetLastError(), "scale launch"))) return st;
    }
    float* x = s.x;        // the residual stream
    float* x_other = s.x2;
    const float* pending = nullptr;       // the previous layer's FFN output, added to x next
    const float* pending_post = nullptr;  // its post-FFN norm (Gemma 2) or null
    for (int l = 0; l < m->n_layers; l++) {
        const sulimo_layer_desc& L = m->layers[l];
        {  // attention norm, then q, k, v in one launch
            const GemvMatSrc g[3] = {{L.wq_scales, L.wq_quants, s.q, qd},
                                     {L.wk_scales, L.wk_quants, s.k, kvd},
                                     {L.wv_scales, L.wv_quants, s.v, kvd}};
            if ((st = norm_and_gemv(ctx, s, x, x_other, pending,
                                    reinterpret_cast<const float*>(L.attn_norm), m->eps, E, batch,
                                    g, 3, true, pending_post, gemma)))
                return st;
        }
        (void)launch_pdl(qkv_rope_store_kernel, dim3(H + 2 * Hkv, batch), dim3(128), 0,
                         ctx->stream, s.q, (const float*)s.k, (const float*)s.v,
                         reinterpret_cast<const float*>(L.bq), reinterpret_cast<const float*>(L.bk),
                         reinterpret_cast<const float*>(L.bv), H, Hkv, hd, m->rope_dim,
                         m->rope_mode, m->rope_base, pos, (size_t)0,
                         reinterpret_cast<uint8_t*>(L.k_ring),
                         reinterpret_cast<uint8_t*>(L.v_ring), m->kv_capacity, m->kv_seq_stride);
        ctx->launches++;
        if ((st = check_cuda(cudaGetLastError(), "qkv_rope_store launch"))) return st;
        // attention, its output quantized to Q8_0 in the merge kernel (the o projection's input)
        // every ring slot but the newest (written by qkv_rope_store) is static during the step
        const GemvMatSrc go = {L.wo_scales, L.wo_quants, s.o, E};
        const Q8Out att_form = step_q8_form(ctx, s, &go, 1, qd, batch);
        if ((st = launch_attn_decode(ctx, s.q, L.k_ring, L.v_ring, m->kv_seq_stride,
                                     m->kv_capacity, ctx_len, H, Hkv, hd, batch, m->attn_softcap,
                                     nullptr, reinterpret_cast<float*>(ctx->workspace),
                                     ctx->workspace_bytes, &att_form, pos)) ||
            (st = step_gemv(ctx, &go, 1, att_form, qd, batch)))
            return st;
        {  // FFN norm (x += o), then gate and up in one launch
            const GemvMatSrc g[2] = {{L.wg_scales, L.wg_quants, s.g, F},
                                     {L.wu_scales, L.wu_quants, s.u, F}};
            if ((st = norm_and_gemv(ctx, s, x, x_other, s.o,
                                    reinterpret_cast<const float*>(L.ffn_norm), m->eps, E, batch,
                                    g, 2, true, reinterpret_cast<const float*>(L.post_attn_norm),
                                    gemma)))
                return st;
        }
        const GemvMatSrc gd = {L.wd_scales, L.wd_quants, s.o, E};
        if ((st = swiglu_and_gemv(ctx, s, s.g, s.u, F, batch, gd, gemma))) return st;
        pending = s.o;
        pending_post = reinterpret_cast<const float*>(L.post_ffn_norm);
    }
    // output norm and the vocab projection (the residual is not needed afterwards)
    const GemvMatSrc gl = {m->out_scales, m->out_quants, logits, m->vocab};
    if ((st = norm_and_gemv(ctx, s, x, x_other, pending, m->out_norm, m->eps, E, batch, &gl, 1,
                            false, pending_post, gemma)))
        return st;
    if (m->final_softcap > 0.0f) {  // logit_softcap_scalar (forward_pass.rs:411-414)
        const size_t n = (size_t)batch * m->vocab;
        (void)launch_pdl(logit_softcap_kernel, dim3((unsigned)((n + 255) / 256)), dim3(256), 0,
                         ctx->stream, logits, n, 1.0f / m->final_softcap, m->final_softcap);
        ctx->launches++;
        st = check_cuda(cudaGetLastError(), "logit_softcap launch");
    }
    return st;
}

}  // namespace sulimo
