"""GPU parity of the two load/scheduler-side operations moved onto the device:

- repack_q4_0_aos_to_soa (crates/sulimo-core/src/repack.rs:45-81): GGUF Q4_0 blocks to the SoA
  scales / quants, byte-exact against the oracle's restatement (itself checked against the
  reference's repack test, repack.rs:138-179), for 16-byte and 2-byte aligned sources, ragged
  block counts, and the reference's three errors;
- repack_context + the re-prefill that follows it (crates/sulimo-engine/src/scheduler.rs:316-326,
  engine.rs:226-239): the plan's counts against the reference's arithmetic restated here, the
  device-gathered token list against the host-built one, and the device re-prefill equal bit for
  bit (logits and K/V rings) to prefilling the host-built list with sulimo_cuda_prefill_ubatch.
"""
import ctypes as C

import numpy as np
import pytest

import oracle.ffi as O
import sulimo_b200 as sb
from gpu_util import dev, empty, host
from sulimo_b200 import capi

pytestmark = pytest.mark.gpu


def repack_plan_reference(n_past, capacity):
    """repack_context's counts (scheduler.rs:316-318)."""
    sys_len = min(max(capacity // 8, 4), 64, n_past)
    recent_len = min(capacity // 2, max(n_past - sys_len, 0))
    return sys_len, recent_len


@pytest.mark.parametrize("nblocks,offset", [(1, 0), (255, 0), (4097, 0), (1000, 2), (77, 18)])
def test_repack_q4_0_aos_to_soa_byte_exact(ctx, nblocks, offset):
    import torch
    rng = np.random.default_rng(nblocks)
    aos = rng.integers(0, 256, nblocks * 18, dtype=np.uint8)
    n_ref, sc_ref, qu_ref = O.repack_q4_0_aos_to_soa(aos)
    assert n_ref == nblocks
    buf = torch.zeros(nblocks * 18 + offset + 16, dtype=torch.uint8, device="cuda")
    buf[offset:offset + nblocks * 18] = torch.from_numpy(aos).cuda()
    sc = torch.zeros(nblocks * 2, dtype=torch.uint8, device="cuda")
    qu = torch.zeros(nblocks * 16, dtype=torch.uint8, device="cuda")
    nb = C.c_size_t()
    capi.call("sulimo_cuda_repack_q4_0_aos_to_soa", ctx.handle, buf.data_ptr() + offset,
              nblocks * 18, sc.data_ptr(), sc.numel(), qu.data_ptr(), qu.numel(), C.byref(nb))
    ctx.finish()
    assert nb.value == nblocks
    assert np.array_equal(host(sc), sc_ref) and np.array_equal(host(qu), qu_ref)


def test_repack_q4_0_errors(ctx):
    t = empty(64, __import__("torch").uint8)
    nb = C.c_size_t()
    L = capi.load()
    args = (ctx.handle, t.data_ptr())
    assert L.sulimo_cuda_repack_q4_0_aos_to_soa(*args, 17, t.data_ptr(), 64, t.data_ptr(), 64,
                                                 C.byref(nb)) == capi.EINVAL
    assert b"InvalidAosLength" in L.sulimo_cuda_last_error()
    assert L.sulimo_cuda_repack_q4_0_aos_to_soa(*args, 36, t.data_ptr(), 3, t.data_ptr(), 64,
                                                 C.byref(nb)) == capi.EINVAL
    assert b"ScalesBufferTooSmall" in L.sulimo_cuda_last_error()
    assert L.sulimo_cuda_repack_q4_0_aos_to_soa(*args, 36, t.data_ptr(), 4, t.data_ptr(), 31,
                                                 C.byref(nb)) == capi.EINVAL
    assert b"QuantsBufferTooSmall" in L.sulimo_cuda_last_error()


@pytest.mark.parametrize("n_past,capacity", [(0, 64), (3, 64), (64, 64), (100, 64), (9, 16),
                                             (5000, 4096), (70, 1024)])
def test_repack_context_plan(n_past, capacity):
    s, r = C.c_size_t(), C.c_size_t()
    capi.load().sulimo_cuda_repack_context_plan(n_past, capacity, C.byref(s), C.byref(r))
    assert (s.value, r.value) == repack_plan_reference(n_past, capacity)


def test_repack_context_reprefill_on_device(ctx):
    import torch
    from sulimo_b200.model import DecodeModel
    from sulimo_b200.synthetic import make_model_numpy, to_device
    cfg = dict(n_layers=2, embd=256, ffn=512, head_count=4, head_count_kv=2, head_dim=64,
               vocab=512, rope_dim=64, rope_mode=1, eps=1e-6, rope_base=1e6, attn_softcap=0.0,
               bias=True)
    cap, n_past, ub = 64, 61, 20
    w = to_device(make_model_numpy(cfg, seed=21, kv_capacity=cap))
    past = torch.from_numpy(np.random.default_rng(22).integers(0, 512, n_past).astype(np.int32)).cuda()
    sys_len, recent_len = repack_plan_reference(n_past, cap)
    keep = torch.cat([past[:sys_len], past[n_past - recent_len:]])
    # host-built list, prefilled ubatch by ubatch
    ref_model = DecodeModel(ctx, w, batch=1)
    lg_ref = None
    for p0 in range(0, keep.numel(), ub):
        lg_ref = ref_model.prefill(keep[p0:p0 + ub].contiguous(), p0).clone()
    # the device path
    dm = DecodeModel(ctx, w, batch=1)
    need = capi.load().sulimo_cuda_prefill_scratch_bytes(dm._desc_ptr, ub)
    scratch = torch.empty(need, dtype=torch.uint8, device="cuda")
    new_tokens = torch.empty(n_past, dtype=torch.int32, device="cuda")
    logits = torch.empty(cfg["vocab"], dtype=torch.float32, device="cuda")
    new_pos = C.c_size_t()
    capi.call("sulimo_cuda_repack_context", ctx.handle, dm._desc_ptr, past.data_ptr(), n_past,
              new_tokens.data_ptr(), ub, logits.data_ptr(), scratch.data_ptr(), need,
              C.byref(new_pos))
    ctx.finish()
    assert new_pos.value == sys_len + recent_len
    assert torch.equal(new_tokens[:new_pos.value], keep)
    assert np.array_equal(host(logits).view(np.uint32), host(lg_ref).view(np.uint32))
    for (ka, va), (kb, vb) in zip(dm.rings, ref_model.rings):
        assert torch.equal(ka, kb) and torch.equal(va, vb)
