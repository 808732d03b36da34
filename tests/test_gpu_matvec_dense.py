"""GPU parity of the F32 / F16 branches of apply_matvec (crates/sulimo-engine/src/forward_pass.rs:
509-527 -> dispatch_matvec_f32 / dispatch_matvec_f16, crates/sulimo-cpu/src/avx2.rs:72-104):
bit-identical to the AVX2 kernels (avx2.rs:259-331) restated in the oracle, for column counts
with and without a tail past the last full 8-lane chunk, one to five activation vectors, and the
router itself (Q4_0 / F32 / F16, unknown types refused)."""
import ctypes as C

import numpy as np
import pytest

import oracle.ffi as O
import sulimo_b200 as sb
from gpu_util import dev, empty, host
from helpers import make_q4_0

pytestmark = pytest.mark.gpu


def bits(a):
    return np.asarray(a, np.float32).view(np.uint32)


@pytest.mark.parametrize("kind", ["f32", "f16"])
@pytest.mark.parametrize("rows,cols,batch", [(1000, 1536, 1), (257, 3072, 3), (33, 1537, 5),
                                             (64, 7, 2), (4096, 256, 4)])
def test_dense_matvec_bit_exact(ctx, kind, rows, cols, batch):
    import torch
    rng = np.random.default_rng(rows + cols)
    w = (rng.standard_normal((rows, cols)) * 0.05).astype(np.float32)
    if kind == "f16":
        w = w.astype(np.float16).view(np.uint16)
    x = rng.standard_normal((batch, cols)).astype(np.float32)
    out = empty(batch * rows, torch.float32)
    fn = sb.dispatch_matvec_f32 if kind == "f32" else sb.dispatch_matvec_f16
    fn(ctx, dev(w), dev(x), rows, cols, out, batch=batch)
    ctx.finish()
    got = host(out).reshape(batch, rows)
    for b in range(batch):
        ref = O.matvec_dense(w, x[b], rows, cols, kind)
        assert np.array_equal(bits(got[b]), bits(ref)), b


def test_apply_matvec_routes_by_type(ctx):
    import torch
    rng = np.random.default_rng(3)
    rows, cols = 300, 512
    ws, wq = make_q4_0(rows, cols, seed=4)
    xf = rng.standard_normal(cols).astype(np.float32)
    xq8 = O.quantize_f32_to_q8_0(xf)
    out = empty(rows, torch.float32)
    sb.apply_matvec(ctx, sb.GGML_Q4_0, dev(ws), dev(wq), dev(xq8), None, rows, cols, out)
    ctx.finish()
    assert np.array_equal(bits(host(out)), bits(O.matvec_q4_0_q8_0_avx2(ws, wq, xq8, rows, cols)))
    w16 = (rng.standard_normal((rows, cols)) * 0.1).astype(np.float16).view(np.uint16)
    sb.apply_matvec(ctx, sb.GGML_F16, dev(w16), None, None, dev(xf), rows, cols, out)
    ctx.finish()
    assert np.array_equal(bits(host(out)), bits(O.matvec_dense(w16, xf, rows, cols, "f16")))
    with pytest.raises(sb.SulimoError) as e:
        sb.apply_matvec(ctx, 8, dev(w16), None, None, dev(xf), rows, cols, out)  # Q8_0 weights
    assert e.value.kind == "InvalidArgument"
