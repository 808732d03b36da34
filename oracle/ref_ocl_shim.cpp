/*
 * ref_ocl_shim.cpp — runs the reference's own OpenCL C kernels on the host CPU.
 *
 * TEST INFRASTRUCTURE ONLY.  The library this file builds (oracle/_ref/libsulimo_ref_ocl.so)
 * pins the C restatement in sulimo_oracle.c to values produced by the reference's code; it is
 * used by tests/ and by the fixture script tests/golden/make_ref_ocl_golden.py.  The product
 * (libsulimo_cuda.so, the sulimo_b200 package) never links or calls it.
 *
 * The reference's two kernel files, kernels/gemm_q4_0.cl and kernels/prefill.cl, are compiled
 * UNCHANGED: they are #included from the reference checkout (the build recipe passes that
 * directory with -I; oracle/ref_build.py).  This file supplies what an OpenCL C compiler would:
 *   - the kernel and address-space qualifiers (`__kernel`, `__global`), which mean nothing on
 *     the host;
 *   - `half` as _Float16 (IEEE binary16; float -> half conversions round to nearest even, the
 *     OpenCL default for explicit conversions; half arithmetic is correctly rounded, because a
 *     float intermediate of one operation followed by one rounding to half is innocuous:
 *     24 >= 2*11 + 2 significand bits), and the `h` suffix of half literals (`0.0h`);
 *   - get_global_id() from a per-thread ND-range index;
 *   - the float overloads of the math builtins (sqrt, pow, cos, sin, exp, fabs, round -> glibc
 *     sqrtf, powf, cosf, sinf, expf, fabsf, roundf).
 * Each ND-range is executed as loops over its global ids, spread over host threads along the
 * first dimension; every work-item of these kernels writes only its own outputs, so the order
 * of work-items does not change any result.
 *
 * Built with -ffp-contract=off and without fast-math, so each kernel's arithmetic runs in its
 * source order with one rounding per operation.  (The reference compiles the kernels for its
 * device with -cl-mad-enable -cl-fast-relaxed-math, crates/sulimo-ocl/src/program.rs:23, under
 * which a device compiler may contract or reassociate; this shim gives the source-order result,
 * which is also what the reference's CPU oracle gemm_q4_0_f16_scalar_reference computes,
 * crates/sulimo-ocl/src/gemm.rs:106-147.)
 *
 * ref_execute_prefill_ubatch restates the host side of execute_prefill_ubatch
 * (crates/sulimo-ocl/src/prefill.rs:337-566): the same kernels, in the same order, over the same
 * scratch buffers, with the same arguments.
 */
#include <cmath>
#include <cstddef>
#include <cstdint>
#include <cstring>
#include <thread>
#include <vector>

#include "sulimo_oracle.h"

using std::cos;
using std::exp;
using std::fabs;
using std::pow;
using std::round;
using std::sin;
using std::sqrt;

namespace refocl {

typedef _Float16 half;
typedef unsigned char uchar;

#define __kernel static
#define __global

// OpenCL C half literal suffix (`0.0h`).
constexpr half operator""h(long double v) { return (half)v; }

static thread_local size_t g_gid[3];
static inline size_t get_global_id(unsigned int dim) { return dim < 3 ? g_gid[dim] : 0; }

#include "gemm_q4_0.cl"
#include "prefill.cl"

#undef __kernel
#undef __global

// Runs body() for every global id (i, j) of a [g0, g1] ND-range; the first dimension is split
// into contiguous chunks over `threads` host threads.
template <class F>
static void nd_range(size_t g0, size_t g1, int threads, F body) {
    if (g0 == 0 || g1 == 0) return;
    if (threads < 1) threads = 1;
    if ((size_t)threads > g0) threads = (int)g0;
    auto run = [&](size_t lo, size_t hi) {
        for (size_t i = lo; i < hi; i++)
            for (size_t j = 0; j < g1; j++) {
                g_gid[0] = i;
                g_gid[1] = j;
                g_gid[2] = 0;
                body();
            }
    };
    if (threads == 1) {
        run(0, g0);
        return;
    }
    std::vector<std::thread> pool;
    const size_t chunk = (g0 + threads - 1) / threads;
    for (int t = 0; t < threads; t++) {
        const size_t lo = (size_t)t * chunk;
        const size_t hi = lo + chunk < g0 ? lo + chunk : g0;
        if (lo >= hi) break;
        pool.emplace_back(run, lo, hi);
    }
    for (auto& th : pool) th.join();
}

static inline half* H(uint16_t* p) { return reinterpret_cast<half*>(p); }
static inline const half* H(const uint16_t* p) { return reinterpret_cast<const half*>(p); }
static inline const half* H(const uint8_t* p) { return reinterpret_cast<const half*>(p); }

}  // namespace refocl

using namespace refocl;

extern "C" {

/* gemm_q4_0_f16_portable (kernels/gemm_q4_0.cl:13-58), ND-range [M, N] as in
 * enqueue_gemm_q4_0_f16 (crates/sulimo-ocl/src/prefill.rs:69-105). */
void ref_gemm_q4_0_f16_portable(const uint16_t* scales, const uint8_t* quants, const uint16_t* x,
                                uint16_t* out, int M, int K, int N, int threads) {
    nd_range((size_t)M, (size_t)N, threads,
             [&] { gemm_q4_0_f16_portable(H(scales), quants, H(x), H(out), M, K, N); });
}

/* rmsnorm_f16_f32w (kernels/prefill.cl:4-29), ND-range [N]. */
void ref_rmsnorm_f16_f32w(const uint16_t* x, const float* w, uint16_t* out, int D, float eps,
                          int N) {
    nd_range((size_t)N, 1, 1, [&] { rmsnorm_f16_f32w(H(x), w, H(out), D, eps, N); });
}

/* rope_f16 (kernels/prefill.cl:32-68), ND-range [N, head_count]; mode 0 = Norm, else Neox. */
void ref_rope_f16(uint16_t* vec, int head_count, int head_dim, int rope_dim, float freq_base,
                  int mode, int start_pos, int N) {
    nd_range((size_t)N, (size_t)head_count, 1, [&] {
        rope_f16(H(vec), head_count, head_dim, rope_dim, freq_base, mode, start_pos, N);
    });
}

/* kv_store_q8_0 (kernels/prefill.cl:72-116), ND-range [N, blocks_per_pos]. */
void ref_kv_store_q8_0(const uint16_t* act, uint8_t* kv, int start_pos, int capacity,
                       int blocks_per_pos, int N) {
    nd_range((size_t)N, (size_t)blocks_per_pos, 1, [&] {
        kv_store_q8_0(H(act), kv, start_pos, capacity, blocks_per_pos, N);
    });
}

/* causal_gqa_attention_prefill (kernels/prefill.cl:120-237), ND-range [N, head_count]. */
void ref_causal_gqa_attention_prefill(const uint16_t* q, const uint8_t* k_cache,
                                      const uint8_t* v_cache, uint16_t* out, int start_pos,
                                      int capacity, int head_count, int head_count_kv,
                                      int head_dim, int N, int threads) {
    nd_range((size_t)N, (size_t)head_count, threads, [&] {
        causal_gqa_attention_prefill(H(q), k_cache, v_cache, H(out), start_pos, capacity,
                                     head_count, head_count_kv, head_dim, N);
    });
}

/* silu_mul_f16 (kernels/prefill.cl:240-253), ND-range [total]. */
void ref_silu_mul_f16(const uint16_t* gate, const uint16_t* up, uint16_t* out, int total) {
    nd_range((size_t)total, 1, 1, [&] { silu_mul_f16(H(gate), H(up), H(out), total); });
}

/* add_f16 (kernels/prefill.cl:256-266), ND-range [total]. */
void ref_add_f16(uint16_t* a, const uint16_t* b, int total) {
    nd_range((size_t)total, 1, 1, [&] { add_f16(H(a), H(b), total); });
}

/* logits_f16_output (kernels/prefill.cl:269-308), ND-range [M]. */
void ref_logits_f16_output(const uint16_t* x_all, const uint16_t* scales, const uint8_t* quants,
                           float* logits, int M, int K, int token_idx, int threads) {
    nd_range((size_t)M, 1, threads, [&] {
        logits_f16_output(H(x_all), H(scales), quants, logits, M, K, token_idx);
    });
}

/* execute_prefill_ubatch (crates/sulimo-ocl/src/prefill.rs:337-566) over the kernels above.
 * x: scratch.x, [n][embd] f16, holding the ubatch's token embeddings on entry (the engine fills
 * it with lookup_token_embedding_f16, crates/sulimo-engine/src/engine.rs:249-256) and the
 * residual stream on return.  Writes K/V ring slots (start_pos + t) % kv_capacity of every
 * layer and the last token's fp32 logits[vocab].  Scales are f16 arrays (the SoA `scales`). */
int ref_execute_prefill_ubatch(const oracle_model* m, uint16_t* x, size_t start_pos, size_t n,
                               float* logits, int threads) {
    if (!m || !x || !logits || n == 0) return -1;
    const int embd = m->embd, ffn = m->ffn, hc = m->head_count, hkv = m->head_count_kv,
              hd = m->head_dim;
    const int N = (int)n, sp = (int)start_pos, cap = (int)m->kv_capacity;
    const int rope_mode = m->rope_mode;  // 0 = Norm (Llama), 1 = Neox
    const int bpp = hkv * hd / 32;
    std::vector<uint16_t> h((size_t)n * embd), q((size_t)n * hc * hd), k((size_t)n * hkv * hd),
        v((size_t)n * hkv * hd), attn((size_t)n * hc * hd), gate((size_t)n * ffn),
        up((size_t)n * ffn), sw((size_t)n * ffn), down((size_t)n * embd);
    auto S = [](const uint8_t* p) { return reinterpret_cast<const uint16_t*>(p); };
    for (int l = 0; l < m->n_layers; l++) {
        const oracle_layer& L = m->layers[l];
        ref_rmsnorm_f16_f32w(x, L.attn_norm, h.data(), embd, m->eps, N);
        ref_gemm_q4_0_f16_portable(S(L.wq_s), L.wq_q, h.data(), q.data(), hc * hd, embd, N,
                                   threads);
        ref_gemm_q4_0_f16_portable(S(L.wk_s), L.wk_q, h.data(), k.data(), hkv * hd, embd, N,
                                   threads);
        ref_gemm_q4_0_f16_portable(S(L.wv_s), L.wv_q, h.data(), v.data(), hkv * hd, embd, N,
                                   threads);
        ref_rope_f16(q.data(), hc, hd, m->rope_dim, m->rope_base, rope_mode, sp, N);
        ref_rope_f16(k.data(), hkv, hd, m->rope_dim, m->rope_base, rope_mode, sp, N);
        ref_kv_store_q8_0(k.data(), L.k_ring, sp, cap, bpp, N);
        ref_kv_store_q8_0(v.data(), L.v_ring, sp, cap, bpp, N);
        ref_causal_gqa_attention_prefill(q.data(), L.k_ring, L.v_ring, attn.data(), sp, cap, hc,
                                         hkv, hd, N, threads);
        ref_gemm_q4_0_f16_portable(S(L.wo_s), L.wo_q, attn.data(), h.data(), embd, embd, N,
                                   threads);
        ref_add_f16(x, h.data(), N * embd);
        ref_rmsnorm_f16_f32w(x, L.ffn_norm, h.data(), embd, m->eps, N);
        ref_gemm_q4_0_f16_portable(S(L.wg_s), L.wg_q, h.data(), gate.data(), ffn, embd, N,
                                   threads);
        ref_gemm_q4_0_f16_portable(S(L.wu_s), L.wu_q, h.data(), up.data(), ffn, embd, N,
                                   threads);
        ref_silu_mul_f16(gate.data(), up.data(), sw.data(), N * ffn);
        ref_gemm_q4_0_f16_portable(S(L.wd_s), L.wd_q, sw.data(), down.data(), embd, ffn, N,
                                   threads);
        ref_add_f16(x, down.data(), N * embd);
    }
    ref_rmsnorm_f16_f32w(x, m->out_norm, h.data(), embd, m->eps, N);
    ref_logits_f16_output(h.data(), S(m->out_s), m->out_q, logits, m->vocab, embd, N - 1,
                          threads);
    return 0;
}

}  // extern "C"
