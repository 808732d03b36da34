"""GPU test of sulimo_cuda_attn_decode_q8_0_noalloc, the decode-attention entry point that
allocates nothing.

It is for callers that must not allocate device memory: a decode loop held to a no-allocation
rule per token, or a host that plans all device memory up front.  Instead of the context
workspace (grown with cudaMalloc on demand) it keeps its partial results in a fixed array inside
the library.  This file checks, through the C ABI:
  - two calls in a row (different shapes, so the second call runs over the first call's
    leftovers in the shared array) against the oracle's causal_gqa_decode_scalar_ext restatement
    (crates/sulimo-cpu/src/scalar.rs:287-359) and against the regular entry point, within the
    attention tolerance;
  - on a fresh context, that the entry point leaves the context's own workspace at zero bytes
    and that the device's free memory does not change across a call;
  - that a problem larger than the array is refused with an error.
It is named to be collected last.
"""
import ctypes as C

import numpy as np
import pytest

import oracle.ffi as O
from gpu_util import dev, empty, host
from helpers import rel_l2
from sulimo_b200 import capi

pytestmark = pytest.mark.gpu
TOL = 2e-3
SCRATCH_FLOATS = 1 << 19


def ring(rng, cap, kv_heads, head_dim, batch):
    """Random Q8_0 rings (valid f16 scales, int8 quants) for `batch` sequences."""
    nblk = batch * cap * kv_heads * head_dim // 32
    blocks = rng.integers(-127, 128, size=(nblk, 34), dtype=np.int16).astype(np.int8).view(np.uint8)
    scales = (rng.uniform(0.002, 0.03, nblk)).astype(np.float16).view(np.uint8).reshape(nblk, 2)
    blocks[:, :2] = scales
    return blocks.reshape(-1)


def attend(ctx, fn, q, kr, vr, cap, ctx_len, H, Hkv, hd, batch):
    import torch
    out = empty(batch * H * hd, torch.float32)
    stride = kr.numel() // batch   # bytes between the sequences' rings
    capi.call(fn, ctx.handle, q.data_ptr(), kr.data_ptr(), vr.data_ptr(), stride, cap, ctx_len,
              H, Hkv, hd, batch, C.c_float(0.0), out.data_ptr())
    ctx.finish()
    return host(out)


@pytest.mark.parametrize("calls", [[
    # (head_count, kv_heads, head_dim, capacity, context_len, batch)
    (16, 2, 256, 8192, 8192, 1),   # long context: the split count is reduced to fit the array
    (12, 2, 128, 4096, 300, 2),    # then Qwen2.5-1.5B geometry over the same array
]])
def test_noalloc_matches_oracle_and_workspace_entry_point_twice(ctx, calls):
    rng = np.random.default_rng(42)
    for (H, Hkv, hd, cap, ctx_len, batch) in calls:
        kr_h, vr_h = ring(rng, cap, Hkv, hd, batch), ring(rng, cap, Hkv, hd, batch)
        q_h = rng.standard_normal(batch * H * hd).astype(np.float32)
        kr, vr, q = dev(kr_h), dev(vr_h), dev(q_h)
        got = attend(ctx, "sulimo_cuda_attn_decode_q8_0_noalloc", q, kr, vr, cap, ctx_len, H,
                     Hkv, hd, batch)
        ref = attend(ctx, "sulimo_cuda_attn_decode_q8_0", q, kr, vr, cap, ctx_len, H, Hkv, hd,
                     batch)
        assert np.all(np.isfinite(got))
        assert rel_l2(got, ref) <= TOL
        stride = kr_h.size // batch
        for s in range(batch):
            oracle = O.causal_gqa_decode(q_h[s * H * hd:(s + 1) * H * hd],
                                         kr_h[s * stride:(s + 1) * stride],
                                         vr_h[s * stride:(s + 1) * stride], cap, ctx_len, H, Hkv,
                                         hd)
            err = rel_l2(got[s * H * hd:(s + 1) * H * hd], oracle)
            assert err <= TOL, (H, ctx_len, s, err)


def test_noalloc_allocates_nothing_on_a_fresh_context():
    """A fresh context, whose first call is the no-allocation entry point: its workspace stays
    at zero bytes, and (on a second fresh context, after the library's device code is loaded)
    the device's free memory is the same before and after a call."""
    import torch
    import sulimo_b200 as sb
    rng = np.random.default_rng(7)
    H, Hkv, hd, cap, ctx_len, batch = 12, 2, 128, 4096, 1000, 1
    kr, vr = dev(ring(rng, cap, Hkv, hd, batch)), dev(ring(rng, cap, Hkv, hd, batch))
    q = dev(rng.standard_normal(batch * H * hd).astype(np.float32))
    lib = capi.load()
    outs = []
    for fresh in range(2):
        c = sb.CudaContext(0)
        c.set_stream(torch.cuda.current_stream())
        out = empty(batch * H * hd, torch.float32)
        torch.cuda.synchronize()
        free0 = torch.cuda.mem_get_info()[0]
        capi.call("sulimo_cuda_attn_decode_q8_0_noalloc", c.handle, q.data_ptr(), kr.data_ptr(),
                  vr.data_ptr(), kr.numel(), cap, ctx_len, H, Hkv, hd, batch, C.c_float(0.0),
                  out.data_ptr())
        c.finish()
        free1 = torch.cuda.mem_get_info()[0]
        assert lib.sulimo_cuda_ctx_workspace_bytes(c.handle) == 0
        if fresh == 1:
            assert free1 == free0, (free0, free1)
        outs.append(host(out))
        c.close()
    assert np.array_equal(outs[0], outs[1])


def test_noalloc_refuses_problems_beyond_the_fixed_scratch(ctx):
    import torch
    H, Hkv, hd, cap, ctx_len, batch = 24, 8, 128, 4096, 4096, 64
    assert batch * H * (ctx_len // 256) * (hd + 2) > SCRATCH_FLOATS
    t = empty(1024, torch.float32)
    st = capi.load().sulimo_cuda_attn_decode_q8_0_noalloc(
        ctx.handle, t.data_ptr(), t.data_ptr(), t.data_ptr(), 0, cap, ctx_len, H, Hkv, hd, batch,
        C.c_float(0.0), t.data_ptr())
    assert st == capi.EINVAL
    assert b"fixed attention scratch" in capi.load().sulimo_cuda_last_error()
    ctx.finish()  # nothing was launched, the context stays usable
