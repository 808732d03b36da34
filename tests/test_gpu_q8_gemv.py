"""GPU parity: Q8_0 quantize / KV-ring store / Q4_0 dequant / decode GEMV, all bit- or
byte-exact against the oracle.  Every call goes through the C ABI (libsulimo_cuda.so)."""
import os

import numpy as np
import pytest

import oracle.ffi as O
import sulimo_b200 as sb
from gpu_util import dev, empty, host
from helpers import make_q4_0

pytestmark = pytest.mark.gpu
GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def gpu_quantize(ctx, x):
    import torch
    src = dev(x.astype(np.float32))
    dst = empty(x.size // 32 * 34, torch.uint8)
    sb.quantize_f32_to_q8_0(ctx, src, dst)
    ctx.finish()
    return host(dst)


# ---- quantize_f32_to_q8_0 (kv_cache.rs:162-192) -------------------------------------------

@pytest.mark.parametrize("n", [32, 1536, 8960, 32 * 4097])
def test_quantize_byte_exact_random(ctx, n):
    x = np.random.default_rng(n).standard_normal(n).astype(np.float32) * 3
    assert np.array_equal(gpu_quantize(ctx, x), O.quantize_f32_to_q8_0(x))


def test_quantize_byte_exact_edge_values(ctx):
    x = np.zeros(32 * 8, np.float32)
    x[32:64] = 1e-40
    x[64:96] = np.linspace(-1e4, 1e4, 32)
    x[96:128] = -7.0
    x[128] = np.nan
    x[129:160] = 2.0
    x[160:192] = np.float32(3.4e38)
    x[192:224] = np.arange(32) * 0.5 - 8.0  # exact ties of x*id
    x[224:256] = 1e-30
    assert np.array_equal(gpu_quantize(ctx, x), O.quantize_f32_to_q8_0(x))


def test_quantize_golden_roundtrip(ctx):
    g = np.load(os.path.join(GOLDEN, "q8_roundtrip.npz"))
    assert np.array_equal(gpu_quantize(ctx, g["src"]), g["q8"])


def test_quantize_rejects_bad_length(ctx):
    import torch
    src = empty(33, torch.float32)
    dst = empty(64, torch.uint8)
    with pytest.raises(sb.SulimoError) as e:
        sb.quantize_f32_to_q8_0(ctx, src, dst, 33)
    assert e.value.kind == "InvalidArgument"


# ---- kv_store_q8_0 (prefill.cl:72-116) / KvCache::store_key (kv_cache.rs:93-110) -----------

def test_kv_store_reference_case_f16(ctx):
    """crates/sulimo-ocl/tests/test_prefill.rs:57-192: 16 tokens x 8 blocks, start_pos 5,
    capacity 64 — byte-exact (the reference test allows one quant step)."""
    import torch
    n, bpp, cap, start = 16, 8, 64, 5
    i = np.arange(n * bpp * 32, dtype=np.float32)
    act = (np.sin(i * np.float32(0.17)) * 5 + ((np.arange(i.size) % 7) - 3)).astype(np.float16)
    kv = torch.zeros(cap * bpp * 34, dtype=torch.uint8, device="cuda")
    sb.kv_store_q8_0(ctx, dev(act), kv, start, cap, bpp, n)
    ctx.finish()
    ref = np.zeros(cap * bpp * 34, np.uint8)
    O.kv_store_q8_0(act.view(np.uint16), ref, start, cap, bpp, n)
    assert np.array_equal(host(kv), ref)


def test_kv_store_wraps_ring_f32(ctx):
    import torch
    n, bpp, cap, start = 37, 4, 16, 10   # wraps twice; later tokens overwrite earlier slots
    act = np.random.default_rng(1).standard_normal((n, bpp * 32)).astype(np.float32)
    kv = torch.zeros(cap * bpp * 34, dtype=torch.uint8, device="cuda")
    # the ring is written token by token, as a decode loop does (one store per position)
    for t in range(n):
        sb.kv_store_q8_0(ctx, dev(act[t]), kv, start + t, cap, bpp, 1)
    ctx.finish()
    ref = np.zeros(cap * bpp * 34, np.uint8)
    for t in range(n):
        O.kv_store_f32(act[t], ref, start + t, cap, bpp)
    assert np.array_equal(host(kv), ref)


# ---- dequantize_q4_0_soa (repack.rs:107-131) and f16 embedding (scheduler.rs:329-357) -------

@pytest.mark.parametrize("out_dtype", [sb.OUT_F32, sb.OUT_F16])
def test_dequant_rows_bit_exact(ctx, out_dtype):
    import torch
    rows, cols = 300, 1536
    ws, wq = make_q4_0(rows, cols, seed=11)
    ids = np.array([0, 7, 299, 150, 7], np.int32)
    out = empty(len(ids) * cols, torch.float32 if out_dtype == sb.OUT_F32 else torch.float16)
    sb.dequantize_q4_0_rows(ctx, dev(ws), dev(wq), cols, dev(ids), out, out_dtype)
    ctx.finish()
    nb = cols // 32
    for c, r in enumerate(ids):
        if out_dtype == sb.OUT_F32:
            ref = O.dequantize_q4_0_soa(ws[r * nb:(r + 1) * nb], wq[r * nb * 16:(r + 1) * nb * 16], nb)
            got = host(out)[c * cols:(c + 1) * cols]
            assert np.array_equal(got.view(np.uint32), ref.view(np.uint32))
        else:
            ref = O.lookup_token_embedding_f16(ws, wq, cols, int(r))
            got = host(out)[c * cols:(c + 1) * cols].view(np.uint16)
            assert np.array_equal(got, ref)


# ---- integer block sums and the decode GEMV (avx2.rs:113-189) -------------------------------

def test_block_sums_config1_bit_exact(ctx):
    import torch
    rows, cols = 8960, 1536
    ws, wq = make_q4_0(rows, cols, seed=0)
    x = np.random.default_rng(100).standard_normal(cols).astype(np.float32)
    xq8 = O.quantize_f32_to_q8_0(x)
    out = empty(rows * cols // 32, torch.int32)
    sb.block_sums_q4_0_q8_0(ctx, dev(wq), dev(xq8), rows, cols, out)
    ctx.finish()
    assert np.array_equal(host(out), O.block_sums_q4_0_q8_0(ws, wq, xq8, rows, cols))


def run_gemv(ctx, ws, wq, xq8, rows, cols, batch):
    import torch
    out = empty(batch * rows, torch.float32)
    sb.dispatch_matvec_q4_0_q8_0(ctx, dev(ws), dev(wq), dev(xq8), rows, cols, out, batch)
    ctx.finish()
    return host(out)


def test_gemv_config1_bit_exact(ctx):
    """benchmark config 1: 8960 x 1536 Q4_0 x Q8_0, batch 1, seed 0 — bit-identical to the
    AVX2 kernel (and the integer block sums equal, test above)."""
    rows, cols = 8960, 1536
    ws, wq = make_q4_0(rows, cols, seed=0)
    x = np.random.default_rng(0).standard_normal(cols).astype(np.float32)
    xq8 = O.quantize_f32_to_q8_0(x)
    got = run_gemv(ctx, ws, wq, xq8, rows, cols, 1)
    ref = O.matvec_q4_0_q8_0_avx2(ws, wq, xq8, rows, cols, threads=8)
    assert np.array_equal(got.view(np.uint32), ref.view(np.uint32))


def test_gemv_golden_sample(ctx):
    g = np.load(os.path.join(GOLDEN, "config1_sample.npz"))
    got = run_gemv(ctx, g["ws"], g["wq"], g["xq8"], 8, 1536, 1)
    assert np.array_equal(got.view(np.uint32), g["out_avx2"].view(np.uint32))


def test_gemv_reference_avx2_case(ctx):
    g = np.load(os.path.join(GOLDEN, "avx2_test.npz"))
    got = run_gemv(ctx, g["ws"], g["wq"], g["xq8"], 1, 256, 1)
    assert got.view(np.uint32)[0] == g["dot_avx2"].view(np.uint32)[0]


@pytest.mark.parametrize("rows,cols,batch", [
    (1, 32, 1), (17, 64, 1), (300, 8960, 1), (8192, 3072, 2), (100, 96, 3), (33, 2080, 1),
    (1536, 8960, 1), (256, 3072, 8), (1000, 2048, 5), (512, 3072, 32), (65, 256, 9),
])
def test_gemv_shapes_bit_exact(ctx, rows, cols, batch):
    ws, wq = make_q4_0(rows, cols, seed=rows + cols)
    x = np.random.default_rng(batch).standard_normal((batch, cols)).astype(np.float32)
    xq8 = np.concatenate([O.quantize_f32_to_q8_0(x[b]) for b in range(batch)])
    got = run_gemv(ctx, ws, wq, xq8, rows, cols, batch).reshape(batch, rows)
    for b in range(batch):
        ref = O.matvec_q4_0_q8_0_avx2(ws, wq, xq8[b * cols // 32 * 34:(b + 1) * cols // 32 * 34],
                                      rows, cols, threads=8)
        assert np.array_equal(got[b].view(np.uint32), ref.view(np.uint32)), f"batch {b}"


def test_gemv_unaligned_scales_take_the_general_kernel(ctx):
    """Scales that are only 2-byte aligned cannot be streamed with TMA; the general kernel
    must give the same bits."""
    import torch
    rows, cols = 700, 1536
    ws, wq = make_q4_0(rows, cols, seed=21)
    x = np.random.default_rng(22).standard_normal(cols).astype(np.float32)
    xq8 = O.quantize_f32_to_q8_0(x)
    big = dev(np.concatenate([np.zeros(1, np.uint16), ws]))      # scales start 2 bytes in
    out = empty(rows, torch.float32)
    sb.dispatch_matvec_q4_0_q8_0(ctx, big.data_ptr() + 2, dev(wq), dev(xq8), rows, cols, out)
    ctx.finish()
    ref = O.matvec_q4_0_q8_0_avx2(ws, wq, xq8, rows, cols, threads=8)
    assert np.array_equal(host(out).view(np.uint32), ref.view(np.uint32))


def test_gemv_rejects_bad_cols(ctx):
    import torch
    t = empty(64, torch.uint8)
    with pytest.raises(sb.SulimoError):
        sb.dispatch_matvec_q4_0_q8_0(ctx, t, t, t, 1, 48, empty(1, torch.float32))


@pytest.mark.parametrize("rows,cols,batch", [(8960, 1536, 1), (3072, 8192, 1), (300, 2048, 4)])
def test_gemv_static_weights_bit_exact(ctx, rows, cols, batch):
    """The static-weights entry (weight tiles fetched before the launch's dependency wait) gives
    the same bits, also when launched right behind another matvec writing its activations'
    neighbour buffer."""
    import torch
    ws, wq = make_q4_0(rows, cols, seed=rows + 3)
    x = np.random.default_rng(batch + 5).standard_normal((batch, cols)).astype(np.float32)
    xq8 = np.concatenate([O.quantize_f32_to_q8_0(x[b]) for b in range(batch)])
    out = empty(batch * rows, torch.float32)
    dws, dwq, dx = dev(ws), dev(wq), dev(xq8)
    for _ in range(2):
        sb.dispatch_matvec_q4_0_q8_0(ctx, dws, dwq, dx, rows, cols, out, batch, True)
    ctx.finish()
    got = host(out).reshape(batch, rows)
    for b in range(batch):
        ref = O.matvec_q4_0_q8_0_avx2(ws, wq, xq8[b * cols // 32 * 34:(b + 1) * cols // 32 * 34],
                                      rows, cols, threads=8)
        assert np.array_equal(got[b].view(np.uint32), ref.view(np.uint32))


# ---- fast mode (sulimo_cuda_gemv_q4_0_q8_0_fast): exact block sums, fixed fp32 partial tree ----

@pytest.mark.parametrize("rows,cols,batch", [(8960, 1536, 1), (3072, 8192, 1), (1000, 3072, 3),
                                             (16, 256, 1), (257, 2048, 8), (300, 96, 2)])
def test_gemv_fast_matches_avx2_within_rounding(ctx, rows, cols, batch):
    """Fast mode vs the AVX2 oracle: the same exact integer block sums, fp32 additions grouped
    differently, so per-row errors stay at fp32 rounding of the row's terms (rel-L2 <= 1e-5,
    far inside the 2e-3 fast-mode bound); repeated calls, with and without the static-weights
    prefetch, give the same bits.  Ragged shapes: rows not a multiple of the 8 rows of a CTA,
    K blocks not a multiple of the 32 lanes (cols 96, 1536, 2048)."""
    import torch
    ws, wq = make_q4_0(rows, cols, seed=rows * 7 + cols)
    x = np.random.default_rng(batch + 11).standard_normal((batch, cols)).astype(np.float32)
    xq8 = np.concatenate([O.quantize_f32_to_q8_0(x[b]) for b in range(batch)])
    dws, dwq, dx = dev(ws), dev(wq), dev(xq8)
    outs = []
    for static in (False, True):
        out = empty(batch * rows, torch.float32)
        sb.matvec_q4_0_q8_0_fast(ctx, dws, dwq, dx, rows, cols, out, batch, static)
        ctx.finish()
        outs.append(host(out).reshape(batch, rows))
    assert np.array_equal(outs[0].view(np.uint32), outs[1].view(np.uint32))
    nbx = cols // 32 * 34
    for b in range(batch):
        ref = O.matvec_q4_0_q8_0_avx2(ws, wq, xq8[b * nbx:(b + 1) * nbx], rows, cols, threads=8)
        got = outs[0][b]
        rel = np.linalg.norm(got.astype(np.float64) - ref) / np.linalg.norm(ref.astype(np.float64))
        assert rel <= 1e-5, rel


# ---- fast mode, several sequences: the tensor-core form (gemv_mma_q4_0_q8_0.cu) ----------------

@pytest.mark.parametrize("rows,cols,batch", [(3072, 3072, 8), (8192, 3072, 32), (3072, 8192, 32),
                                             (1000, 2048, 13), (16, 256, 2), (257, 512, 17),
                                             (20000, 3072, 8), (5120, 3072, 40)])
def test_gemv_fast_batched_tensor_core_form(ctx, rows, cols, batch):
    """From 2 sequences (K a multiple of 256) the fast entry restages the Q8_0 blocks and runs the
    tensor-core matvec: exact integer block sums (mma m16n8k32), fp32 accumulation in block order.
    Each sequence against the AVX2 oracle at rel-L2 <= 1e-5; static / non-static and repeated
    calls bit-identical.  Shapes: config 4's q/o (8 sequences), gate/up and down (32: one and
    four 8-sequence groups per CTA), a vocabulary-sized matrix, ragged rows (not a multiple of
    the 16-row tiles), ragged batches (13, 17, 40: partial 8-sequence tiles and groups), and
    activations with all-zero and saturated blocks."""
    import torch
    ws, wq = make_q4_0(rows, cols, seed=rows + 3 * cols + batch)
    rng = np.random.default_rng(batch * 31 + rows)
    x = rng.standard_normal((batch, cols)).astype(np.float32)
    x[0, :64] = 0.0                      # two all-zero blocks (d = 0)
    x[-1, 32:64] = 1e4 * np.sign(x[-1, 32:64])   # a saturated block (codes +-127)
    xq8 = np.concatenate([O.quantize_f32_to_q8_0(x[b]) for b in range(batch)])
    dws, dwq, dx = dev(ws), dev(wq), dev(xq8)
    outs = []
    for static in (False, True, True):
        out = empty(batch * rows, torch.float32)
        out.fill_(float("nan"))
        sb.matvec_q4_0_q8_0_fast(ctx, dws, dwq, dx, rows, cols, out, batch, static)
        ctx.finish()
        outs.append(host(out).reshape(batch, rows))
    for o in outs[1:]:
        assert np.array_equal(outs[0].view(np.uint32), o.view(np.uint32))
    nbx = cols // 32 * 34
    for b in range(batch):
        ref = O.matvec_q4_0_q8_0_avx2(ws, wq, xq8[b * nbx:(b + 1) * nbx], rows, cols, threads=8)
        got = outs[0][b]
        assert np.isfinite(got).all(), b
        rel = np.linalg.norm(got.astype(np.float64) - ref) / np.linalg.norm(ref.astype(np.float64))
        assert rel <= 1e-5, (b, rel)
