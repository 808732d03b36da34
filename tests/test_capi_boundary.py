"""CPU tests of the C-ABI boundary: the library loads without a GPU, exports exactly the
symbols include/sulimo_cuda.h declares, and fails cleanly (no abort) when no device exists."""
import ctypes as C
import os
import re

import pytest

import sulimo_b200 as sb
from sulimo_b200 import capi

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "sulimo_cuda.h")


def declared_symbols():
    text = open(HEADER).read()
    return sorted(set(re.findall(r"\b(sulimo_cuda_[a-z0-9_]+)\s*\(", text)))


def test_library_exports_every_declared_symbol():
    L = capi.load()
    syms = declared_symbols()
    assert len(syms) >= 25
    for s in syms:
        assert hasattr(L, s), f"{s} declared in the header but not exported"
    # the ctypes signature table covers the whole header, nothing more
    assert sorted(capi.SIGNATURES) == syms


def test_exported_symbols_are_exactly_the_header():
    import subprocess
    out = subprocess.run(["nm", "-D", "--defined-only", capi.LIB_PATH], capture_output=True,
                         text=True, check=True).stdout
    exported = sorted(l.split()[-1] for l in out.splitlines() if " T " in l)
    assert exported == declared_symbols()


def test_version_string():
    assert b"sm_100a" in capi.load().sulimo_cuda_version()


def test_null_arguments_are_rejected_without_a_device():
    L = capi.load()
    assert L.sulimo_cuda_ctx_create(0, None) == capi.EINVAL
    assert L.sulimo_cuda_ctx_synchronize(None) == capi.EINVAL
    assert L.sulimo_cuda_gemm_q4_0_f16(None, None, None, None, None, 8, 32, 1, 0) == capi.EINVAL
    assert L.sulimo_cuda_buffer_free(None) == capi.OK
    assert L.sulimo_cuda_event_wait(None, 0) == capi.EINVAL
    assert b"null" in L.sulimo_cuda_last_error()
    assert L.sulimo_cuda_live_buffer_count() == 0


def test_context_creation_without_gpu_reports_no_device():
    import torch
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    h = C.c_void_p()
    st = capi.load().sulimo_cuda_ctx_create(0, C.byref(h))
    assert st == capi.ENODEV and not h.value
    with pytest.raises(sb.SulimoError) as e:
        sb.CudaContext(0)
    assert e.value.kind == "DeviceNotFound"


def test_missing_library_fails_loudly(tmp_path, monkeypatch):
    monkeypatch.setattr(capi, "_lib", None)
    with pytest.raises(RuntimeError, match="no CPU fallback"):
        capi.load(str(tmp_path / "absent.so"))
    monkeypatch.setattr(capi, "_lib", None)
