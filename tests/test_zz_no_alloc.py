"""GPU test of sulimo_cuda_attn_decode_q8_0_noalloc, the decode-attention entry point that
allocates nothing.

It is for callers that must not allocate device memory: a decode loop held to a no-allocation
rule per token, or a host that plans all device memory up front.  Instead of the context
workspace (grown with cudaMalloc on demand) it keeps its partial results in a fixed array inside
the library.  This file checks, through the C ABI, that two calls in a row (different shapes, so
the second call runs over the first call's leftovers in the shared array) give the same results
as the regular entry point within the attention tolerance, and that a problem larger than the
array is refused with an error.  It is named to be collected last.
"""
import ctypes as C

import numpy as np
import pytest

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
def test_noalloc_matches_workspace_entry_point_twice(ctx, calls):
    rng = np.random.default_rng(42)
    for (H, Hkv, hd, cap, ctx_len, batch) in calls:
        kr = dev(ring(rng, cap, Hkv, hd, batch))
        vr = dev(ring(rng, cap, Hkv, hd, batch))
        q = dev(rng.standard_normal(batch * H * hd).astype(np.float32))
        ref = attend(ctx, "sulimo_cuda_attn_decode_q8_0", q, kr, vr, cap, ctx_len, H, Hkv, hd,
                     batch)
        got = attend(ctx, "sulimo_cuda_attn_decode_q8_0_noalloc", q, kr, vr, cap, ctx_len, H,
                     Hkv, hd, batch)
        assert np.all(np.isfinite(got))
        assert rel_l2(got, ref) <= TOL


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
