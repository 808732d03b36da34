"""GPU tests of the host runtime behind the C ABI: buffers (OclBuffer, buffer.rs), the live
buffer counter (active_cl_mem_count), event waits with deadlines (wait_event_zero_spin,
waiter.rs) and the launch counter."""
import ctypes as C

import numpy as np
import pytest

import sulimo_b200 as sb
from sulimo_b200 import capi

pytestmark = pytest.mark.gpu


def test_buffer_roundtrip_and_leak_counter(ctx):
    L = capi.load()
    base = L.sulimo_cuda_live_buffer_count()
    for _ in range(50):   # test_m4_scheduler.rs:287-364 runs 50 cycles and checks for leaks
        data = np.random.default_rng(0).integers(0, 256, 4096 * 3, dtype=np.uint8)
        h = C.c_void_p()
        capi.call("sulimo_cuda_buffer_from_host", ctx.handle, data.ctypes.data, data.size, 1, 0,
                  C.byref(h))
        back = np.zeros_like(data)
        capi.call("sulimo_cuda_buffer_read", h, 0, back.ctypes.data, back.size)
        assert np.array_equal(back, data)
        assert L.sulimo_cuda_buffer_device_ptr(h)
        capi.call("sulimo_cuda_buffer_free", h)
    assert L.sulimo_cuda_live_buffer_count() == base


def test_buffer_arena_alignment_contract(ctx):
    """buffer.rs:49-54: host_ptr 4096-aligned, size % 64 == 0 (checked when strict)."""
    raw = np.zeros(8192 + 4096, np.uint8)
    off = (-raw.ctypes.data) % 4096
    h = C.c_void_p()
    st = capi.load().sulimo_cuda_buffer_from_host(ctx.handle, raw.ctypes.data + off + 1, 64, 1,
                                                  1, C.byref(h))
    assert st == capi.EALIGN
    st = capi.load().sulimo_cuda_buffer_from_host(ctx.handle, raw.ctypes.data + off, 65, 1, 1,
                                                  C.byref(h))
    assert st == capi.EALIGN
    capi.call("sulimo_cuda_buffer_from_host", ctx.handle, raw.ctypes.data + off, 4096, 1, 1,
              C.byref(h))
    with pytest.raises(sb.SulimoError):
        capi.call("sulimo_cuda_buffer_read", h, 4000, raw.ctypes.data, 200)  # out of bounds
    capi.call("sulimo_cuda_buffer_free", h)


def test_event_wait_completes_and_counts_launches(ctx):
    import torch
    n0 = ctx.launch_count
    x = torch.randn(32 * 64, device="cuda")
    q = torch.empty(64 * 34, dtype=torch.uint8, device="cuda")
    sb.quantize_f32_to_q8_0(ctx, x, q)
    ev = C.c_void_p()
    capi.call("sulimo_cuda_event_record", ctx.handle, C.byref(ev))
    capi.call("sulimo_cuda_event_wait", ev, 5_000_000_000)   # with a deadline
    capi.call("sulimo_cuda_event_wait", ev, 0)               # blocking, no deadline
    capi.call("sulimo_cuda_event_free", ev)
    assert ctx.launch_count == n0 + 1


def test_event_wait_deadline_expires_on_pending_work(ctx):
    """A wait whose deadline passes returns Timeout instead of blocking; the pending work is
    torch's bounded sleep kernel (~0.1 s of device clocks) on a side stream."""
    import torch
    s = torch.cuda.Stream()
    c2 = sb.CudaContext(0, stream=s)
    with torch.cuda.stream(s):
        torch.cuda._sleep(200_000_000)
    ev = C.c_void_p()
    capi.call("sulimo_cuda_event_record", c2.handle, C.byref(ev))
    st = capi.load().sulimo_cuda_event_wait(ev, 1_000)        # 1 us deadline
    assert st == capi.ETIMEOUT
    capi.call("sulimo_cuda_event_wait", ev, 0)                # then wait it out
    capi.call("sulimo_cuda_event_free", ev)
    c2.close()
