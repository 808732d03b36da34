"""ctypes binding of libsulimo_cuda.so (the C ABI declared in include/sulimo_cuda.h).

This is the Python view of the same boundary a `sulimo-cuda` Rust crate binds: plain pointers,
sizes and int status codes.  Loading fails loudly when the library has not been built; there is
no CPU fallback.
"""
import ctypes as C
import os

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libsulimo_cuda.so")

OK, EINVAL, ENODEV, EOOM, ELAUNCH, ETIMEOUT, ENCCL, EALIGN, EDEVICE = range(9)
OUT_F16, OUT_F32 = 0, 1
GGML_F32, GGML_F16, GGML_Q4_0 = 0, 1, 2
ACT_F16, ACT_F32 = 0, 1

STATUS_NAMES = {
    OK: "Ok", EINVAL: "InvalidArgument", ENODEV: "DeviceNotFound", EOOM: "OutOfMemory",
    ELAUNCH: "Driver", ETIMEOUT: "Timeout", ENCCL: "Nccl", EALIGN: "Alignment",
    EDEVICE: "ExecutionFailed",
}

# name -> (restype, argtypes); the list is the whole exported surface of the header.
_vp, _sz, _i, _u64, _f = C.c_void_p, C.c_size_t, C.c_int, C.c_uint64, C.c_float
SIGNATURES = {
    "sulimo_cuda_last_error": (C.c_char_p, []),
    "sulimo_cuda_version": (C.c_char_p, []),
    "sulimo_cuda_ctx_create": (_i, [_i, C.POINTER(_vp)]),
    "sulimo_cuda_ctx_destroy": (_i, [_vp]),
    "sulimo_cuda_ctx_synchronize": (_i, [_vp]),
    "sulimo_cuda_ctx_set_stream": (_i, [_vp, _vp]),
    "sulimo_cuda_ctx_get_stream": (_vp, [_vp]),
    "sulimo_cuda_ctx_device": (_i, [_vp]),
    "sulimo_cuda_ctx_launch_count": (_u64, [_vp]),
    "sulimo_cuda_ctx_workspace_bytes": (_sz, [_vp]),
    "sulimo_cuda_matvec_f32": (_i, [_vp, _vp, _vp, _i, _i, _i, _vp]),
    "sulimo_cuda_matvec_f16": (_i, [_vp, _vp, _vp, _i, _i, _i, _vp]),
    "sulimo_cuda_apply_matvec": (_i, [_vp, _i, _vp, _vp, _vp, _vp, _i, _i, _i, _vp]),
    "sulimo_cuda_repack_context_plan": (None, [_sz, _sz, C.POINTER(_sz), C.POINTER(_sz)]),
    "sulimo_cuda_repack_context": (_i, [_vp, _vp, _vp, _sz, _vp, _i, _vp, _vp, _sz,
                                        C.POINTER(_sz)]),
    "sulimo_cuda_repack_q4_0_aos_to_soa": (_i, [_vp, _vp, _sz, _vp, _sz, _vp, _sz,
                                                C.POINTER(_sz)]),
    "sulimo_cuda_buffer_from_host": (_i, [_vp, _vp, _sz, _i, _i, C.POINTER(_vp)]),
    "sulimo_cuda_buffer_alloc": (_i, [_vp, _sz, C.POINTER(_vp)]),
    "sulimo_cuda_buffer_write": (_i, [_vp, _sz, _vp, _sz]),
    "sulimo_cuda_buffer_read": (_i, [_vp, _sz, _vp, _sz]),
    "sulimo_cuda_buffer_device_ptr": (_vp, [_vp]),
    "sulimo_cuda_buffer_size": (_sz, [_vp]),
    "sulimo_cuda_buffer_free": (_i, [_vp]),
    "sulimo_cuda_live_buffer_count": (_sz, []),
    "sulimo_cuda_event_record": (_i, [_vp, C.POINTER(_vp)]),
    "sulimo_cuda_event_wait": (_i, [_vp, _u64]),
    "sulimo_cuda_event_free": (_i, [_vp]),
    "sulimo_cuda_gemm_q4_0_f16": (_i, [_vp, _vp, _vp, _vp, _vp, _i, _i, _i, _i]),
    "sulimo_cuda_gemm_q4_0_f16_exact": (_i, [_vp, _vp, _vp, _vp, _vp, _i, _i, _i, _i]),
    "sulimo_cuda_logits_final": (_i, [_vp, _vp, _vp, _vp, _vp, _i, _i, _i]),
    "sulimo_cuda_gemv_q4_0_q8_0": (_i, [_vp, _vp, _vp, _vp, _i, _i, _i, _vp]),
    "sulimo_cuda_gemv_q4_0_q8_0_static": (_i, [_vp, _vp, _vp, _vp, _i, _i, _i, _vp]),
    "sulimo_cuda_gemv_q4_0_q8_0_fast": (_i, [_vp, _vp, _vp, _vp, _i, _i, _i, _vp, _i]),
    "sulimo_cuda_block_sums_q4_0_q8_0": (_i, [_vp, _vp, _vp, _i, _i, _vp]),
    "sulimo_cuda_quantize_q8_0": (_i, [_vp, _vp, _vp, _sz]),
    "sulimo_cuda_kv_store_q8_0": (_i, [_vp, _vp, _i, _vp, _sz, _sz, _sz, _sz]),
    "sulimo_cuda_dequantize_q4_0_rows": (_i, [_vp, _vp, _vp, _i, _vp, _i, _vp, _i]),
    "sulimo_cuda_unshard_rows": (_i, [_vp, _vp, _vp, _i, _i, _sz, _sz, _i]),
    "sulimo_cuda_ipc_handle": (_i, [_vp, _vp]),
    "sulimo_cuda_ipc_open": (_i, [_vp, _vp, C.POINTER(_vp)]),
    "sulimo_cuda_ipc_close": (_i, [_vp, _vp]),
    "sulimo_cuda_gemm_q4_0_f16_allgather": (_i, [_vp, _vp, _vp, _vp, _i, _i, _i, _i, _i, _vp, _sz,
                                                 _sz, _vp, _vp, _i, _i, C.c_uint,
                                                 C.POINTER(C.c_uint)]),
    "sulimo_cuda_wait_counter": (_i, [_vp, _vp, C.c_uint]),
    "sulimo_cuda_forward_scratch_bytes": (_sz, [_vp, _i]),
    "sulimo_cuda_forward_token": (_i, [_vp, _vp, _vp, _i, _sz, _vp, _vp, _sz]),
    "sulimo_cuda_argmax_rows": (_i, [_vp, _vp, _i, _i, _vp]),
    "sulimo_cuda_prefill_scratch_bytes": (_sz, [_vp, _i]),
    "sulimo_cuda_prefill_ubatch": (_i, [_vp, _vp, _vp, _i, _sz, _vp, _vp, _sz]),
    "sulimo_cuda_prefill_ubatch_x": (_i, [_vp, _vp, _vp, _i, _sz, _vp, _vp, _sz]),
    "sulimo_cuda_attn_prefill_q8_0": (_i, [_vp, _vp, _vp, _vp, _sz, _sz, _i, _i, _i, _i, _vp]),
    "sulimo_cuda_attn_decode_q8_0": (_i, [_vp, _vp, _vp, _vp, _sz, _sz, _sz, _i, _i, _i, _i,
                                          _f, _vp]),
    "sulimo_cuda_attn_decode_q8_0_noalloc": (_i, [_vp, _vp, _vp, _vp, _sz, _sz, _sz, _i, _i, _i,
                                                  _i, _f, _vp]),
}

_lib = None


class SulimoError(RuntimeError):
    """A non-zero status from the C ABI (the OclError of the reference, program.rs:26-40)."""

    def __init__(self, status, fn, message):
        self.status = status
        self.kind = STATUS_NAMES.get(status, str(status))
        super().__init__(f"{fn}: {self.kind} ({status}): {message}")


def load(path=None):
    """Loads the library (once).  Raises if it is missing: the product has no fallback."""
    global _lib
    if _lib is not None:
        return _lib
    p = path or LIB_PATH
    if not os.path.exists(p):
        raise RuntimeError(
            f"{p} is missing: build it with `python -m sulimo_b200.build` (no CPU fallback)")
    L = C.CDLL(p)
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(L, name)
        fn.restype = res
        fn.argtypes = args
    _lib = L
    return L


def check(status, fn_name):
    if status != OK:
        msg = load().sulimo_cuda_last_error()
        raise SulimoError(status, fn_name, msg.decode() if msg else "")
    return status


def call(name, *args):
    """Calls an int-returning entry point and raises SulimoError on a non-zero status."""
    return check(getattr(load(), name)(*args), name)
