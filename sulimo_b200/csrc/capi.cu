// capi.cu — the extern "C" boundary of libsulimo_cuda: context, buffers, events, argument
// checks and dispatch to the sm_100a kernels.  Mirrors the host runtime of the reference's
// sulimo-ocl crate (program.rs, buffer.rs, waiter.rs, gemm.rs, prefill.rs) with CUDA objects.
#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>
#include <string.h>
#include <time.h>

#include <atomic>
#include <mutex>
#include <string>

#include "sulimo_internal.h"

namespace {
thread_local std::string g_last_error;
std::atomic<size_t> g_live_buffers{0};
}  // namespace

struct sulimo_buf {
    sulimo_ctx* ctx = nullptr;
    void* dev = nullptr;
    size_t size = 0;
    int read_only = 0;
};

struct sulimo_event {
    cudaEvent_t ev = nullptr;
    sulimo_ctx* ctx = nullptr;
};

namespace sulimo {

int set_error(int status, const std::string& msg) {
    g_last_error = msg;
    return status;
}

int check_cuda(cudaError_t e, const char* what) {
    if (e == cudaSuccess) return SULIMO_OK;
    int st = (e == cudaErrorMemoryAllocation) ? SULIMO_EOOM : SULIMO_ELAUNCH;
    return set_error(st, std::string(what) + ": " + cudaGetErrorString(e));
}

int ensure_workspace(sulimo_ctx* ctx, size_t bytes) {
    if (bytes <= ctx->workspace_bytes) return SULIMO_OK;
    // Growing frees the old block, which in-flight work may still read: drain first.
    cudaError_t e = cudaStreamSynchronize(ctx->stream);
    if (e != cudaSuccess) return check_cuda(e, "workspace sync");
    if (ctx->workspace) cudaFree(ctx->workspace);
    ctx->workspace = nullptr;
    ctx->workspace_bytes = 0;
    size_t want = bytes < (size_t)(1 << 20) ? (size_t)(1 << 20) : bytes;
    e = cudaMalloc(&ctx->workspace, want);
    if (e != cudaSuccess) return check_cuda(e, "workspace cudaMalloc");
    ctx->workspace_bytes = want;
    return SULIMO_OK;
}

EncodeTiledFn get_encode_tiled() {
    static EncodeTiledFn fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
                cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiledFn>(p);
    });
    return fn;
}

int encode_tensor_map(CUtensorMap* map, CUtensorMapDataType dt, const void* base, int rank,
                      const uint64_t* dims, const uint64_t* strides, const uint32_t* box,
                      CUtensorMapSwizzle swz) {
    EncodeTiledFn enc = get_encode_tiled();
    if (!enc) return set_error(SULIMO_ENODEV, "cuTensorMapEncodeTiled unavailable");
    if (rank < 1 || rank > 3) return set_error(SULIMO_EINVAL, "tensor map rank must be 1..3");
    cuuint64_t d[3], st[2];
    cuuint32_t bx[3], estr[3] = {1, 1, 1};
    for (int i = 0; i < rank; i++) {
        d[i] = dims[i];
        bx[i] = box[i];
    }
    for (int i = 0; i + 1 < rank; i++) st[i] = strides[i];
    CUresult r = enc(map, dt, (cuuint32_t)rank, const_cast<void*>(base), d, st, bx, estr,
                     CU_TENSOR_MAP_INTERLEAVE_NONE, swz, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                     CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS)
        return set_error(SULIMO_ELAUNCH, "cuTensorMapEncodeTiled failed: " + std::to_string((int)r));
    return SULIMO_OK;
}

}  // namespace sulimo

using sulimo::set_error;

// After a kernel recorded a device error (a bounded wait ran out) clear the error word so the
// context stays usable.
static void clear_device_state(sulimo_ctx* ctx) { cudaMemset(ctx->d_error, 0, sizeof(int)); }

static int check_ctx(sulimo_ctx* ctx) {
    if (!ctx) return set_error(SULIMO_EINVAL, "null context");
    return SULIMO_OK;
}

static int bind_device(sulimo_ctx* ctx) {
    cudaError_t e = cudaSetDevice(ctx->device);
    return sulimo::check_cuda(e, "cudaSetDevice");
}

static bool aligned(const void* p, size_t a) { return ((uintptr_t)p % a) == 0; }

extern "C" {

const char* sulimo_cuda_last_error(void) { return g_last_error.c_str(); }

const char* sulimo_cuda_version(void) { return "sulimo_cuda 0.1.0 sm_100a"; }

// ---- context ------------------------------------------------------------------------------

int sulimo_cuda_ctx_create(int device, sulimo_ctx** out) {
    if (!out) return set_error(SULIMO_EINVAL, "out is null");
    *out = nullptr;
    int n = 0;
    if (cudaGetDeviceCount(&n) != cudaSuccess || n == 0)
        return set_error(SULIMO_ENODEV, "no CUDA device");
    if (device < 0 || device >= n) return set_error(SULIMO_ENODEV, "device index out of range");
    cudaDeviceProp prop;
    if (cudaGetDeviceProperties(&prop, device) != cudaSuccess)
        return set_error(SULIMO_ENODEV, "cudaGetDeviceProperties failed");
    if (prop.major != 10)
        return set_error(SULIMO_ENODEV, std::string("device is not sm_100 class: ") + prop.name);
    if (cudaSetDevice(device) != cudaSuccess) return set_error(SULIMO_ENODEV, "cudaSetDevice");
    sulimo_ctx* ctx = new sulimo_ctx();
    ctx->device = device;
    ctx->num_sms = prop.multiProcessorCount;
    cudaError_t e = cudaStreamCreateWithFlags(&ctx->own_stream, cudaStreamNonBlocking);
    if (e != cudaSuccess) {
        delete ctx;
        return sulimo::check_cuda(e, "cudaStreamCreate");
    }
    ctx->stream = ctx->own_stream;
    e = cudaMalloc(&ctx->d_error, sizeof(int));
    if (e == cudaSuccess) e = cudaMemset(ctx->d_error, 0, sizeof(int));
    if (e == cudaSuccess)
        e = cudaMalloc(&ctx->attn_counters, sulimo::ATTN_COUNTERS * sizeof(unsigned));
    if (e == cudaSuccess)
        e = cudaMemset(ctx->attn_counters, 0, sulimo::ATTN_COUNTERS * sizeof(unsigned));
    if (e != cudaSuccess) {
        if (ctx->d_error) cudaFree(ctx->d_error);
        if (ctx->attn_counters) cudaFree(ctx->attn_counters);
        cudaStreamDestroy(ctx->own_stream);
        delete ctx;
        return sulimo::check_cuda(e, "error word / attention counters");
    }
    if (!sulimo::get_encode_tiled()) {
        cudaFree(ctx->d_error);
        cudaFree(ctx->attn_counters);
        cudaStreamDestroy(ctx->own_stream);
        delete ctx;
        return set_error(SULIMO_ENODEV, "cuTensorMapEncodeTiled unavailable");
    }
    *out = ctx;
    return SULIMO_OK;
}

int sulimo_cuda_ctx_destroy(sulimo_ctx* ctx) {
    if (!ctx) return SULIMO_OK;
    cudaSetDevice(ctx->device);
    cudaStreamSynchronize(ctx->stream);
    if (ctx->workspace) cudaFree(ctx->workspace);
    if (ctx->d_error) cudaFree(ctx->d_error);
    if (ctx->argmax_scratch) cudaFree(ctx->argmax_scratch);
    if (ctx->attn_counters) cudaFree(ctx->attn_counters);
    if (ctx->q8_stage) cudaFree(ctx->q8_stage);
    if (ctx->own_stream) cudaStreamDestroy(ctx->own_stream);
    delete ctx;
    return SULIMO_OK;
}

int sulimo_cuda_ctx_synchronize(sulimo_ctx* ctx) {
    int st = check_ctx(ctx);
    if (st) return st;
    if ((st = bind_device(ctx))) return st;
    cudaError_t e = cudaStreamSynchronize(ctx->stream);
    if (e != cudaSuccess) return sulimo::check_cuda(e, "cudaStreamSynchronize");
    int flag = 0;
    e = cudaMemcpy(&flag, ctx->d_error, sizeof(int), cudaMemcpyDeviceToHost);
    if (e != cudaSuccess) return sulimo::check_cuda(e, "read error word");
    if (flag != 0) {
        clear_device_state(ctx);
        return set_error(SULIMO_EDEVICE, std::string("device-side error code ") +
                                             std::to_string(flag) +
                                             (flag == 1 ? " (bounded wait ran out)" : ""));
    }
    return SULIMO_OK;
}

int sulimo_cuda_ctx_set_stream(sulimo_ctx* ctx, void* cuda_stream) {
    int st = check_ctx(ctx);
    if (st) return st;
    ctx->stream = (cudaStream_t)cuda_stream;  // NULL is the legacy default stream
    return SULIMO_OK;
}

void* sulimo_cuda_ctx_get_stream(sulimo_ctx* ctx) { return ctx ? (void*)ctx->stream : nullptr; }

int sulimo_cuda_ctx_device(sulimo_ctx* ctx) { return ctx ? ctx->device : -1; }

uint64_t sulimo_cuda_ctx_launch_count(sulimo_ctx* ctx) { return ctx ? ctx->launches.load() : 0; }

size_t sulimo_cuda_ctx_workspace_bytes(sulimo_ctx* ctx) {
    return ctx ? ctx->workspace_bytes + ctx->argmax_bytes : 0;
}

// ---- buffers ------------------------------------------------------------------------------

int sulimo_cuda_buffer_alloc(sulimo_ctx* ctx, size_t size, sulimo_buf** out) {
    int st = check_ctx(ctx);
    if (st) return st;
    if (!out) return set_error(SULIMO_EINVAL, "out is null");
    *out = nullptr;
    if ((st = bind_device(ctx))) return st;
    sulimo_buf* b = new sulimo_buf();
    b->ctx = ctx;
    b->size = size;
    if (size) {
        cudaError_t e = cudaMalloc(&b->dev, size);
        if (e != cudaSuccess) {
            delete b;
            return sulimo::check_cuda(e, "buffer cudaMalloc");
        }
    }
    g_live_buffers.fetch_add(1);
    *out = b;
    return SULIMO_OK;
}

int sulimo_cuda_buffer_from_host(sulimo_ctx* ctx, const void* host_ptr, size_t size,
                                 int read_only, int strict_arena, sulimo_buf** out) {
    if (!out) return set_error(SULIMO_EINVAL, "out is null");
    *out = nullptr;
    if (size && !host_ptr) return set_error(SULIMO_EINVAL, "host_ptr is null");
    if (strict_arena && (!aligned(host_ptr, 4096) || size % 64 != 0))
        return set_error(SULIMO_EALIGN,
                         "host_ptr must be 4096-byte aligned and size a multiple of 64");
    sulimo_buf* b = nullptr;
    int st = sulimo_cuda_buffer_alloc(ctx, size, &b);
    if (st) return st;
    b->read_only = read_only;
    if (size) {
        cudaError_t e = cudaMemcpy(b->dev, host_ptr, size, cudaMemcpyHostToDevice);
        if (e != cudaSuccess) {
            sulimo_cuda_buffer_free(b);
            return sulimo::check_cuda(e, "buffer upload");
        }
    }
    *out = b;
    return SULIMO_OK;
}

int sulimo_cuda_buffer_write(sulimo_buf* buf, size_t offset, const void* host_src, size_t n) {
    if (!buf) return set_error(SULIMO_EINVAL, "null buffer");
    if (offset > buf->size || n > buf->size - offset)
        return set_error(SULIMO_EINVAL, "write out of buffer bounds");
    if (n == 0) return SULIMO_OK;
    int st = bind_device(buf->ctx);
    if (st) return st;
    cudaError_t e = cudaMemcpyAsync((char*)buf->dev + offset, host_src, n, cudaMemcpyHostToDevice,
                                    buf->ctx->stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(buf->ctx->stream);
    return sulimo::check_cuda(e, "buffer write");
}

int sulimo_cuda_buffer_read(sulimo_buf* buf, size_t offset, void* host_dst, size_t n) {
    if (!buf) return set_error(SULIMO_EINVAL, "null buffer");
    if (offset > buf->size || n > buf->size - offset)
        return set_error(SULIMO_EINVAL, "read out of buffer bounds");
    if (n == 0) return SULIMO_OK;
    int st = bind_device(buf->ctx);
    if (st) return st;
    cudaError_t e = cudaMemcpyAsync(host_dst, (const char*)buf->dev + offset, n,
                                    cudaMemcpyDeviceToHost, buf->ctx->stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(buf->ctx->stream);
    return sulimo::check_cuda(e, "buffer read");
}

void* sulimo_cuda_buffer_device_ptr(sulimo_buf* buf) { return buf ? buf->dev : nullptr; }

size_t sulimo_cuda_buffer_size(sulimo_buf* buf) { return buf ? buf->size : 0; }

int sulimo_cuda_buffer_free(sulimo_buf* buf) {
    if (!buf) return SULIMO_OK;
    if (buf->dev) {
        cudaSetDevice(buf->ctx->device);
        cudaFree(buf->dev);
    }
    delete buf;
    g_live_buffers.fetch_sub(1);
    return SULIMO_OK;
}

size_t sulimo_cuda_live_buffer_count(void) { return g_live_buffers.load(); }

// ---- events -------------------------------------------------------------------------------

int sulimo_cuda_event_record(sulimo_ctx* ctx, sulimo_event** out) {
    int st = check_ctx(ctx);
    if (st) return st;
    if (!out) return set_error(SULIMO_EINVAL, "out is null");
    *out = nullptr;
    if ((st = bind_device(ctx))) return st;
    sulimo_event* ev = new sulimo_event();
    ev->ctx = ctx;
    cudaError_t e = cudaEventCreateWithFlags(&ev->ev, cudaEventBlockingSync | cudaEventDisableTiming);
    if (e == cudaSuccess) e = cudaEventRecord(ev->ev, ctx->stream);
    if (e != cudaSuccess) {
        if (ev->ev) cudaEventDestroy(ev->ev);
        delete ev;
        return sulimo::check_cuda(e, "event record");
    }
    *out = ev;
    return SULIMO_OK;
}

int sulimo_cuda_event_wait(sulimo_event* ev, uint64_t timeout_ns) {
    if (!ev) return set_error(SULIMO_EINVAL, "null event");
    int st = bind_device(ev->ctx);
    if (st) return st;
    if (timeout_ns == 0) {
        cudaError_t e = cudaEventSynchronize(ev->ev);  // blocking sync: the thread sleeps
        if (e != cudaSuccess) return sulimo::check_cuda(e, "cudaEventSynchronize");
    } else {
        struct timespec t0, t1;
        clock_gettime(CLOCK_MONOTONIC, &t0);
        uint64_t sleep_ns = 2000;
        while (true) {
            cudaError_t e = cudaEventQuery(ev->ev);
            if (e == cudaSuccess) break;
            if (e != cudaErrorNotReady) return sulimo::check_cuda(e, "cudaEventQuery");
            clock_gettime(CLOCK_MONOTONIC, &t1);
            uint64_t el = (uint64_t)(t1.tv_sec - t0.tv_sec) * 1000000000ull +
                          (uint64_t)(t1.tv_nsec - t0.tv_nsec);
            if (el >= timeout_ns) return set_error(SULIMO_ETIMEOUT, "event wait deadline passed");
            struct timespec ts = {0, (long)sleep_ns};
            nanosleep(&ts, nullptr);
            if (sleep_ns < 200000) sleep_ns *= 2;
        }
    }
    int flag = 0;
    cudaError_t e = cudaMemcpy(&flag, ev->ctx->d_error, sizeof(int), cudaMemcpyDeviceToHost);
    if (e != cudaSuccess) return sulimo::check_cuda(e, "read error word");
    if (flag) {
        clear_device_state(ev->ctx);
        return set_error(SULIMO_EDEVICE, "device-side error code " + std::to_string(flag));
    }
    return SULIMO_OK;
}

int sulimo_cuda_event_free(sulimo_event* ev) {
    if (!ev) return SULIMO_OK;
    if (ev->ev) cudaEventDestroy(ev->ev);
    delete ev;
    return SULIMO_OK;
}

// ---- kernels ------------------------------------------------------------------------------

namespace {

int gemm_entry(sulimo_ctx* ctx, const void* scales, const void* quants, const void* x, void* out,
               int m, int k, int n, int out_dtype, bool exact) {
    int st = check_ctx(ctx);
    if (st) return st;
    if (m <= 0 || k <= 0 || n < 0) return set_error(SULIMO_EINVAL, "m, k must be > 0, n >= 0");
    if (k % 32 != 0) return set_error(SULIMO_EINVAL, "K must be a multiple of 32 (Q4_0 block size)");
    if (m % 8 != 0) return set_error(SULIMO_EINVAL, "M must be a multiple of 8");
    if (out_dtype != SULIMO_OUT_F16 && out_dtype != SULIMO_OUT_F32)
        return set_error(SULIMO_EINVAL, "out_dtype must be SULIMO_OUT_F16 or SULIMO_OUT_F32");
    if (n == 0) return SULIMO_OK;
    if (!scales || !quants || !x || !out) return set_error(SULIMO_EINVAL, "null tensor pointer");
    if (!aligned(x, 16) || !aligned(quants, 16) || !aligned(out, 16) || !aligned(scales, 2))
        return set_error(SULIMO_EALIGN, "x, quants, out must be 16-byte aligned, scales 2-byte");
    if ((st = bind_device(ctx))) return st;
    return sulimo::launch_gemm_q4_0_f16(ctx, scales, quants, x, out, m, k, n, out_dtype, k, 0,
                                        exact);
}

}  // namespace

int sulimo_cuda_gemm_q4_0_f16(sulimo_ctx* ctx, const void* scales, const void* quants,
                              const void* x, void* out, int m, int k, int n, int out_dtype) {
    return gemm_entry(ctx, scales, quants, x, out, m, k, n, out_dtype, false);
}

int sulimo_cuda_gemm_q4_0_f16_exact(sulimo_ctx* ctx, const void* scales, const void* quants,
                                    const void* x, void* out, int m, int k, int n,
                                    int out_dtype) {
    return gemm_entry(ctx, scales, quants, x, out, m, k, n, out_dtype, true);
}

int sulimo_cuda_logits_final(sulimo_ctx* ctx, const void* x_all, const void* scales,
                             const void* quants, float* logits, int vocab, int embd,
                             int token_idx) {
    int st = check_ctx(ctx);
    if (st) return st;
    if (vocab <= 0 || embd <= 0 || token_idx < 0)
        return set_error(SULIMO_EINVAL, "vocab, embd must be > 0 and token_idx >= 0");
    if (embd % 32 != 0) return set_error(SULIMO_EINVAL, "embd must be a multiple of 32");
    if (vocab % 8 != 0) return set_error(SULIMO_EINVAL, "vocab must be a multiple of 8");
    if (!x_all || !scales || !quants || !logits) return set_error(SULIMO_EINVAL, "null pointer");
    if (!aligned(x_all, 16) || !aligned(quants, 16) || !aligned(logits, 16))
        return set_error(SULIMO_EALIGN, "x_all, quants, logits must be 16-byte aligned");
    if ((st = bind_device(ctx))) return st;
    return sulimo::launch_gemm_q4_0_f16(ctx, scales, quants, x_all, logits, vocab, embd, 1,
                                        SULIMO_OUT_F32, embd, token_idx);
}

int sulimo_cuda_gemv_q4_0_q8_0(sulimo_ctx* ctx, const void* w_scales, const void* w_quants,
                               const void* x_q8, int rows, int cols, int batch, float* out) {
    int st = check_ctx(ctx);
    if (st) return st;
    if (rows < 0 || cols <= 0 || batch < 0) return set_error(SULIMO_EINVAL, "bad shape");
    if (cols % 32 != 0) return set_error(SULIMO_EINVAL, "cols must be a multiple of 32");
    if (rows == 0 || batch == 0) return SULIMO_OK;
    if (!w_scales || !w_quants || !x_q8 || !out) return set_error(SULIMO_EINVAL, "null pointer");
    if (!aligned(w_quants, 16) || !aligned(w_scales, 2) || !aligned(x_q8, 2) || !aligned(out, 4))
        return set_error(SULIMO_EALIGN, "w_quants must be 16-byte aligned, scales/x_q8 2-byte");
    if ((st = bind_device(ctx))) return st;
    return sulimo::launch_gemv_q4_0_q8_0(ctx, w_scales, w_quants, x_q8, rows, cols, batch, out);
}

static int matvec_dense(sulimo_ctx* ctx, int wtype, const void* w, const float* x, int rows,
                        int cols, int batch, float* out) {
    int st = check_ctx(ctx);
    if (st) return st;
    if (rows < 0 || cols <= 0 || batch < 0) return set_error(SULIMO_EINVAL, "bad shape");
    if ((size_t)rows * 8 > 0x7fffffffu) return set_error(SULIMO_EINVAL, "too many rows");
    if (rows == 0 || batch == 0) return SULIMO_OK;
    if (!w || !x || !out) return set_error(SULIMO_EINVAL, "null pointer");
    if (!aligned(w, wtype == SULIMO_GGML_F32 ? 4 : 2) || !aligned(x, 4) || !aligned(out, 4))
        return set_error(SULIMO_EALIGN, "w, x, out must be aligned to their element size");
    if ((st = bind_device(ctx))) return st;
    return sulimo::launch_matvec_dense(ctx, wtype, w, x, rows, cols, batch, out);
}

int sulimo_cuda_matvec_f32(sulimo_ctx* ctx, const float* w, const float* x, int rows, int cols,
                           int batch, float* out) {
    return matvec_dense(ctx, SULIMO_GGML_F32, w, x, rows, cols, batch, out);
}

int sulimo_cuda_matvec_f16(sulimo_ctx* ctx, const void* w_f16, const float* x, int rows,
                           int cols, int batch, float* out) {
    return matvec_dense(ctx, SULIMO_GGML_F16, w_f16, x, rows, cols, batch, out);
}

int sulimo_cuda_apply_matvec(sulimo_ctx* ctx, int ggml_type, const void* w0, const void* w1,
                             const void* x_q8, const float* x_f32, int rows, int cols, int batch,
                             float* out) {
    switch (ggml_type) {
        case SULIMO_GGML_Q4_0:
            return sulimo_cuda_gemv_q4_0_q8_0(ctx, w0, w1, x_q8, rows, cols, batch, out);
        case SULIMO_GGML_F32:
        case SULIMO_GGML_F16:
            return matvec_dense(ctx, ggml_type, w0, x_f32, rows, cols, batch, out);
        default:
            return set_error(SULIMO_EINVAL, "tensor type must be F32, F16 or Q4_0");
    }
}

int sulimo_cuda_gemv_q4_0_q8_0_static(sulimo_ctx* ctx, const void* w_scales,
                                      const void* w_quants, const void* x_q8, int rows, int cols,
                                      int batch, float* out) {
    int st = check_ctx(ctx);
    if (st) return st;
    if (rows < 0 || cols <= 0 || batch < 0) return set_error(SULIMO_EINVAL, "bad shape");
    if (cols % 32 != 0) return set_error(SULIMO_EINVAL, "cols must be a multiple of 32");
    if (rows == 0 || batch == 0) return SULIMO_OK;
    if (!w_scales || !w_quants || !x_q8 || !out) return set_error(SULIMO_EINVAL, "null pointer");
    if (!aligned(w_quants, 16) || !aligned(w_scales, 2) || !aligned(x_q8, 2) || !aligned(out, 4))
        return set_error(SULIMO_EALIGN, "w_quants must be 16-byte aligned, scales/x_q8 2-byte");
    if ((st = bind_device(ctx))) return st;
    return sulimo::launch_gemv_static(ctx, w_scales, w_quants, x_q8, rows, cols, batch, out);
}

int sulimo_cuda_gemv_q4_0_q8_0_fast(sulimo_ctx* ctx, const void* w_scales, const void* w_quants,
                                    const void* x_q8, int rows, int cols, int batch, float* out,
                                    int static_weights) {
    int st = check_ctx(ctx);
    if (st) return st;
    if (rows < 0 || cols <= 0 || batch < 0) return set_error(SULIMO_EINVAL, "bad shape");
    if (cols % 32 != 0) return set_error(SULIMO_EINVAL, "cols must be a multiple of 32");
    if (rows == 0 || batch == 0) return SULIMO_OK;
    if (!w_scales || !w_quants || !x_q8 || !out) return set_error(SULIMO_EINVAL, "null pointer");
    if (!aligned(w_quants, 16) || !aligned(w_scales, 2) || !aligned(x_q8, 2) || !aligned(out, 4))
        return set_error(SULIMO_EALIGN, "w_quants must be 16-byte aligned, scales/x_q8 2-byte");
    if ((st = bind_device(ctx))) return st;
    const sulimo::GemvMatSrc src = {w_scales, w_quants, out, rows};
    return sulimo::launch_gemv_fast_group(ctx, &src, 1, x_q8, cols, batch, static_weights != 0);
}

int sulimo_cuda_block_sums_q4_0_q8_0(sulimo_ctx* ctx, const void* w_quants, const void* x_q8,
                                     int rows, int cols, int32_t* out) {
    int st = check_ctx(ctx);
    if (st) return st;
    if (rows < 0 || cols <= 0 || cols % 32 != 0) return set_error(SULIMO_EINVAL, "bad shape");
    if (rows == 0) return SULIMO_OK;
    if (!w_quants || !x_q8 || !out) return set_error(SULIMO_EINVAL, "null pointer");
    if (!aligned(w_quants, 16) || !aligned(x_q8, 2))
        return set_error(SULIMO_EALIGN, "w_quants must be 16-byte aligned, x_q8 2-byte");
    if ((st = bind_device(ctx))) return st;
    return sulimo::launch_block_sums(ctx, w_quants, x_q8, rows, cols, out);
}

int sulimo_cuda_quantize_q8_0(sulimo_ctx* ctx, const float* src, void* dst_q8, size_t n) {
    int st = check_ctx(ctx);
    if (st) return st;
    if (n % 32 != 0) return set_error(SULIMO_EINVAL, "n must be a multiple of 32");
    if (n == 0) return SULIMO_OK;
    if (!src || !dst_q8) return set_error(SULIMO_EINVAL, "null pointer");
    if (!aligned(src, 4) || !aligned(dst_q8, 2)) return set_error(SULIMO_EALIGN, "misaligned");
    if ((st = bind_device(ctx))) return st;
    return sulimo::launch_quantize_q8_0(ctx, src, dst_q8, n);
}

int sulimo_cuda_kv_store_q8_0(sulimo_ctx* ctx, const void* act, int act_dtype, void* kv_ring,
                              size_t start_pos, size_t capacity, size_t blocks_per_pos,
                              size_t n) {
    int st = check_ctx(ctx);
    if (st) return st;
    if (act_dtype != SULIMO_ACT_F16 && act_dtype != SULIMO_ACT_F32)
        return set_error(SULIMO_EINVAL, "act_dtype must be SULIMO_ACT_F16 or SULIMO_ACT_F32");
    if (capacity == 0 || blocks_per_pos == 0)
        return set_error(SULIMO_EINVAL, "capacity and blocks_per_pos must be > 0");
    if (n == 0) return SULIMO_OK;
    if (!act || !kv_ring) return set_error(SULIMO_EINVAL, "null pointer");
    if (!aligned(act, act_dtype == SULIMO_ACT_F16 ? 2 : 4) || !aligned(kv_ring, 2))
        return set_error(SULIMO_EALIGN, "misaligned");
    if ((st = bind_device(ctx))) return st;
    return sulimo::launch_kv_store_q8_0(ctx, act, act_dtype, kv_ring, start_pos, capacity,
                                        blocks_per_pos, n);
}

int sulimo_cuda_dequantize_q4_0_rows(sulimo_ctx* ctx, const void* scales, const void* quants,
                                     int cols, const int32_t* row_ids, int count, void* out,
                                     int out_dtype) {
    int st = check_ctx(ctx);
    if (st) return st;
    if (cols <= 0 || cols % 32 != 0 || count < 0)
        return set_error(SULIMO_EINVAL, "cols must be a positive multiple of 32");
    if (out_dtype != SULIMO_OUT_F16 && out_dtype != SULIMO_OUT_F32)
        return set_error(SULIMO_EINVAL, "bad out_dtype");
    if (count == 0) return SULIMO_OK;
    if (!scales || !quants || !row_ids || !out) return set_error(SULIMO_EINVAL, "null pointer");
    if (!aligned(quants, 16) || !aligned(scales, 2)) return set_error(SULIMO_EALIGN, "misaligned");
    if ((st = bind_device(ctx))) return st;
    return sulimo::launch_dequant_rows(ctx, scales, quants, cols, row_ids, count, out, out_dtype);
}

int sulimo_cuda_unshard_rows(sulimo_ctx* ctx, const void* gathered, void* out, int world,
                             int m_tokens, size_t fs, size_t f, int elem_size) {
    int st = check_ctx(ctx);
    if (st) return st;
    if (world < 1 || m_tokens < 0 || (elem_size != 2 && elem_size != 4))
        return set_error(SULIMO_EINVAL, "bad world / m_tokens / elem_size");
    if (fs == 0 || (size_t)(world - 1) * fs >= f || f > (size_t)world * fs)
        return set_error(SULIMO_EINVAL, "shard rows must satisfy (world-1)*fs < F <= world*fs");
    if (m_tokens > 2147483647 || world > 65535)
        return set_error(SULIMO_EINVAL, "too many tokens / shards");
    if (m_tokens == 0) return SULIMO_OK;
    if (!gathered || !out) return set_error(SULIMO_EINVAL, "null pointer");
    if (!aligned(gathered, elem_size) || !aligned(out, elem_size))
        return set_error(SULIMO_EALIGN, "misaligned");
    if ((st = bind_device(ctx))) return st;
    return sulimo::launch_unshard_rows(ctx, gathered, out, world, m_tokens, fs, f, elem_size);
}

static int check_model(const sulimo_model_desc* m) {
    if (!m || !m->layers || m->n_layers <= 0) return set_error(SULIMO_EINVAL, "null model");
    if (m->embd <= 0 || m->embd % 32 || m->ffn <= 0 || m->ffn % 32 || m->vocab <= 0 ||
        m->vocab % 8)
        return set_error(SULIMO_EINVAL, "embd / ffn multiples of 32, vocab a multiple of 8");
    if (m->head_count <= 0 || m->head_count_kv <= 0 || m->head_count % m->head_count_kv ||
        m->head_count / m->head_count_kv > 8)
        return set_error(SULIMO_EINVAL, "head_count a multiple (<= 8x) of head_count_kv");
    if (m->head_dim <= 0 || m->head_dim % 32 || m->head_dim > 256 || m->rope_dim <= 0 ||
        m->rope_dim % 2 || m->rope_dim > m->head_dim || (m->rope_mode != 0 && m->rope_mode != 1))
        return set_error(SULIMO_EINVAL, "bad head_dim / rope_dim / rope_mode");
    if (m->kv_capacity == 0) return set_error(SULIMO_EINVAL, "kv_capacity must be positive");
    if (m->arch != SULIMO_ARCH_DEFAULT && m->arch != SULIMO_ARCH_GEMMA2)
        return set_error(SULIMO_EINVAL, "arch must be SULIMO_ARCH_DEFAULT or SULIMO_ARCH_GEMMA2");
    if (m->embd * 4 + 33 * 4 > 227 * 1024) return set_error(SULIMO_EINVAL, "embd too large");
    if (!m->tok_scales || !m->tok_quants || !m->out_scales || !m->out_quants || !m->out_norm)
        return set_error(SULIMO_EINVAL, "null embedding / output tensor");
    for (int l = 0; l < m->n_layers; l++) {
        const sulimo_layer_desc& L = m->layers[l];
        const void* need[] = {L.attn_norm, L.ffn_norm, L.wq_scales, L.wq_quants, L.wk_scales,
                              L.wk_quants, L.wv_scales, L.wv_quants, L.wo_scales, L.wo_quants,
                              L.wg_scales, L.wg_quants, L.wu_scales, L.wu_quants, L.wd_scales,
                              L.wd_quants, L.k_ring, L.v_ring};
        for (const void* p : need)
            if (!p) return set_error(SULIMO_EINVAL, "null layer tensor");
        if (!aligned(L.k_ring, 2) || !aligned(L.v_ring, 2))
            return set_error(SULIMO_EALIGN, "rings must be 2-byte aligned");
    }
    if (m->kv_seq_stride % 2) return set_error(SULIMO_EALIGN, "kv_seq_stride must be even");
    return SULIMO_OK;
}

size_t sulimo_cuda_forward_scratch_bytes(const sulimo_model_desc* model, int batch) {
    if (check_model(model) || batch <= 0) return 0;
    return sulimo::forward_scratch_bytes(model, batch);
}

int sulimo_cuda_forward_token(sulimo_ctx* ctx, const sulimo_model_desc* model,
                              const int32_t* tokens, int batch, size_t pos, float* logits,
                              void* scratch, size_t scratch_bytes) {
    int st = check_ctx(ctx);
    if (st) return st;
    if ((st = check_model(model))) return st;
    if (batch <= 0 || batch > 65535) return set_error(SULIMO_EINVAL, "batch must be in [1, 65535]");
    if (!tokens || !logits || !scratch) return set_error(SULIMO_EINVAL, "null pointer");
    if (scratch_bytes < sulimo::forward_scratch_bytes(model, batch))
        return set_error(SULIMO_EINVAL, "scratch smaller than sulimo_cuda_forward_scratch_bytes");
    if (!aligned(scratch, 256) || !aligned(logits, 16) || !aligned(tokens, 4))
        return set_error(SULIMO_EALIGN, "scratch 256-byte, logits 16-byte aligned");
    if (pos + 1 > model->kv_capacity)
        return set_error(SULIMO_EINVAL, "context pos+1 exceeds the ring capacity");
    if ((st = bind_device(ctx))) return st;
    return sulimo::launch_forward_token(ctx, model, tokens, batch, pos, logits, scratch);
}

size_t sulimo_cuda_prefill_scratch_bytes(const sulimo_model_desc* model, int n) {
    if (check_model(model) || n <= 0) return 0;
    return sulimo::prefill_scratch_bytes(model, n);
}

static int prefill_ubatch(sulimo_ctx* ctx, const sulimo_model_desc* model, const int32_t* tokens,
                          const void* x_f16, int n, size_t start_pos, float* logits,
                          void* scratch, size_t scratch_bytes) {
    int st = check_ctx(ctx);
    if (st) return st;
    if ((st = check_model(model))) return st;
    if (model->arch != SULIMO_ARCH_DEFAULT)
        return set_error(SULIMO_EINVAL,
                         "the prefill ubatch has no Gemma 2 steps: use forward_token per token");
    if (model->head_dim != 64 && model->head_dim != 128)
        return set_error(SULIMO_EINVAL, "prefill supports head_dim 64 and 128");
    if (n <= 0 || n > 65535) return set_error(SULIMO_EINVAL, "n must be in [1, 65535]");
    if (start_pos + (size_t)n > model->kv_capacity)
        return set_error(SULIMO_EINVAL, "start_pos + n exceeds the ring capacity");
    if ((!tokens && !x_f16) || !logits || !scratch) return set_error(SULIMO_EINVAL, "null pointer");
    if (scratch_bytes < sulimo::prefill_scratch_bytes(model, n))
        return set_error(SULIMO_EINVAL, "scratch smaller than sulimo_cuda_prefill_scratch_bytes");
    if (!aligned(scratch, 256) || !aligned(logits, 16) || !aligned(tokens, 4) ||
        !aligned(x_f16, 8) ||
        !aligned(model->tok_quants, 16) || !aligned(model->out_quants, 16))
        return set_error(SULIMO_EALIGN, "scratch 256-byte, logits / quants 16-byte aligned");
    for (int l = 0; l < model->n_layers; l++) {
        const sulimo_layer_desc& L = model->layers[l];
        const void* q16[] = {L.wq_quants, L.wk_quants, L.wv_quants, L.wo_quants, L.wg_quants,
                             L.wu_quants, L.wd_quants};
        for (const void* p : q16)
            if (!aligned(p, 16)) return set_error(SULIMO_EALIGN, "quants must be 16-byte aligned");
    }
    if ((st = bind_device(ctx))) return st;
    return sulimo::launch_prefill_ubatch(ctx, model, tokens, x_f16, n, start_pos, logits, scratch);
}

int sulimo_cuda_prefill_ubatch(sulimo_ctx* ctx, const sulimo_model_desc* model,
                               const int32_t* tokens, int n, size_t start_pos, float* logits,
                               void* scratch, size_t scratch_bytes) {
    if (!tokens) return set_error(SULIMO_EINVAL, "null pointer");
    return prefill_ubatch(ctx, model, tokens, nullptr, n, start_pos, logits, scratch,
                          scratch_bytes);
}

int sulimo_cuda_prefill_ubatch_x(sulimo_ctx* ctx, const sulimo_model_desc* model,
                                 const void* x_f16, int n, size_t start_pos, float* logits,
                                 void* scratch, size_t scratch_bytes) {
    if (!x_f16) return set_error(SULIMO_EINVAL, "null pointer");
    return prefill_ubatch(ctx, model, nullptr, x_f16, n, start_pos, logits, scratch,
                          scratch_bytes);
}

void sulimo_cuda_repack_context_plan(size_t n_past, size_t capacity, size_t* sys_len,
                                     size_t* recent_len) {
    size_t s = 0, r = 0;
    sulimo::repack_context_plan(n_past, capacity, &s, &r);
    if (sys_len) *sys_len = s;
    if (recent_len) *recent_len = r;
}

int sulimo_cuda_repack_context(sulimo_ctx* ctx, const sulimo_model_desc* model,
                               const int32_t* past_tokens, size_t n_past, int32_t* new_tokens,
                               int ubatch, float* logits, void* scratch, size_t scratch_bytes,
                               size_t* new_pos_out) {
    int st = check_ctx(ctx);
    if (st) return st;
    if ((st = check_model(model))) return st;
    if (model->arch != SULIMO_ARCH_DEFAULT)
        return set_error(SULIMO_EINVAL,
                         "the re-prefill has no Gemma 2 steps: use forward_token per token");
    if (!new_pos_out) return set_error(SULIMO_EINVAL, "null pointer");
    *new_pos_out = 0;
    if (ubatch <= 0 || ubatch > 65535) return set_error(SULIMO_EINVAL, "ubatch must be in [1, 65535]");
    size_t s, r;
    sulimo::repack_context_plan(n_past, model->kv_capacity, &s, &r);
    if (s + r == 0) return SULIMO_OK;
    if (!past_tokens || !new_tokens || !logits || !scratch)
        return set_error(SULIMO_EINVAL, "null pointer");
    const uint8_t* p0 = reinterpret_cast<const uint8_t*>(past_tokens);
    const uint8_t* q0 = reinterpret_cast<const uint8_t*>(new_tokens);
    if (q0 < p0 + n_past * 4 && p0 < q0 + (s + r) * 4)
        return set_error(SULIMO_EINVAL, "past_tokens and new_tokens overlap");
    if (scratch_bytes < sulimo::prefill_scratch_bytes(model, ubatch))
        return set_error(SULIMO_EINVAL, "scratch smaller than sulimo_cuda_prefill_scratch_bytes(ubatch)");
    if (!aligned(past_tokens, 4) || !aligned(new_tokens, 4) || !aligned(logits, 16) ||
        !aligned(scratch, 256))
        return set_error(SULIMO_EALIGN, "tokens 4-byte, logits 16-byte, scratch 256-byte aligned");
    if (model->head_dim != 64 && model->head_dim != 128)
        return set_error(SULIMO_EINVAL, "prefill supports head_dim 64 and 128");
    if ((st = bind_device(ctx))) return st;
    return sulimo::launch_repack_context(ctx, model, past_tokens, n_past, new_tokens, ubatch, logits,
                                         scratch, new_pos_out);
}

int sulimo_cuda_repack_q4_0_aos_to_soa(sulimo_ctx* ctx, const void* src_aos, size_t src_len,
                                       void* dst_scales, size_t scales_len, void* dst_quants,
                                       size_t quants_len, size_t* num_blocks_out) {
    int st = check_ctx(ctx);
    if (st) return st;
    if (!num_blocks_out) return set_error(SULIMO_EINVAL, "null pointer");
    *num_blocks_out = 0;
    if (src_len % 18) return set_error(SULIMO_EINVAL, "InvalidAosLength: src_len % 18 != 0");
    const size_t nb = src_len / 18;
    if (scales_len < nb * 2) return set_error(SULIMO_EINVAL, "ScalesBufferTooSmall");
    if (quants_len < nb * 16) return set_error(SULIMO_EINVAL, "QuantsBufferTooSmall");
    *num_blocks_out = nb;
    if (nb == 0) return SULIMO_OK;
    if (!src_aos || !dst_scales || !dst_quants) return set_error(SULIMO_EINVAL, "null pointer");
    if (!aligned(src_aos, 2) || !aligned(dst_scales, 2) || !aligned(dst_quants, 16))
        return set_error(SULIMO_EALIGN, "src / scales 2-byte, quants 16-byte aligned");
    if ((st = bind_device(ctx))) return st;
    return sulimo::launch_repack_q4_0(ctx, src_aos, nb, dst_scales, dst_quants);
}

int sulimo_cuda_attn_prefill_q8_0(sulimo_ctx* ctx, const float* q, const void* k_ring,
                                  const void* v_ring, size_t start_pos, size_t capacity, int n,
                                  int head_count, int head_count_kv, int head_dim, void* out) {
    int st = check_ctx(ctx);
    if (st) return st;
    if (head_dim != 64 && head_dim != 128)
        return set_error(SULIMO_EINVAL, "head_dim must be 64 or 128");
    if (head_count <= 0 || head_count_kv <= 0 || head_count % head_count_kv)
        return set_error(SULIMO_EINVAL, "head_count must be a positive multiple of head_count_kv");
    if (n < 0 || n > 65535 * 64 || capacity == 0 || head_count > 65535)
        return set_error(SULIMO_EINVAL, "bad n / capacity / head_count");
    if (start_pos + (size_t)n > capacity)
        return set_error(SULIMO_EINVAL, "start_pos + n exceeds the ring capacity");
    if (n == 0) return SULIMO_OK;
    if (!q || !k_ring || !v_ring || !out) return set_error(SULIMO_EINVAL, "null pointer");
    if (!aligned(q, 8) || !aligned(out, 4) || !aligned(k_ring, 2) || !aligned(v_ring, 2))
        return set_error(SULIMO_EALIGN, "misaligned");
    if ((st = bind_device(ctx))) return st;
    return sulimo::launch_attn_prefill(ctx, q, k_ring, v_ring, start_pos, capacity, n, head_count,
                                       head_count_kv, head_dim, out);
}

int sulimo_cuda_argmax_rows(sulimo_ctx* ctx, const float* x, int rows, int cols, int32_t* out) {
    int st = check_ctx(ctx);
    if (st) return st;
    if (rows < 0 || cols <= 0) return set_error(SULIMO_EINVAL, "bad rows / cols");
    if (rows == 0) return SULIMO_OK;
    if (!x || !out) return set_error(SULIMO_EINVAL, "null pointer");
    if ((st = bind_device(ctx))) return st;
    return sulimo::launch_argmax_rows(ctx, x, rows, cols, out);
}

int sulimo_cuda_ipc_handle(sulimo_buf* buf, void* handle_out) {
    if (!buf || !buf->dev || !handle_out) return set_error(SULIMO_EINVAL, "null buffer / handle");
    cudaSetDevice(buf->ctx->device);
    cudaIpcMemHandle_t h;
    cudaError_t e = cudaIpcGetMemHandle(&h, buf->dev);
    if (e != cudaSuccess) return sulimo::check_cuda(e, "cudaIpcGetMemHandle");
    static_assert(sizeof(h) == 64, "IPC handle size");
    memcpy(handle_out, &h, sizeof(h));
    return SULIMO_OK;
}

int sulimo_cuda_ipc_open(sulimo_ctx* ctx, const void* handle, void** dev_ptr_out) {
    int st = check_ctx(ctx);
    if (st) return st;
    if (!handle || !dev_ptr_out) return set_error(SULIMO_EINVAL, "null handle / out");
    if ((st = bind_device(ctx))) return st;
    cudaIpcMemHandle_t h;
    memcpy(&h, handle, sizeof(h));
    return sulimo::check_cuda(cudaIpcOpenMemHandle(dev_ptr_out, h, cudaIpcMemLazyEnablePeerAccess),
                              "cudaIpcOpenMemHandle");
}

int sulimo_cuda_ipc_close(sulimo_ctx* ctx, void* dev_ptr) {
    int st = check_ctx(ctx);
    if (st) return st;
    if ((st = bind_device(ctx))) return st;
    return sulimo::check_cuda(cudaIpcCloseMemHandle(dev_ptr), "cudaIpcCloseMemHandle");
}

int sulimo_cuda_gemm_q4_0_f16_allgather(sulimo_ctx* ctx, const void* scales, const void* quants,
                                        const void* x, int m_local, int m_valid, int k, int n,
                                        int out_dtype, void* const* out_bases, size_t f_total,
                                        size_t col0, unsigned* const* flags,
                                        unsigned* const* release, int world, int rank,
                                        unsigned epoch, unsigned* tiles_out) {
    int st = check_ctx(ctx);
    if (st) return st;
    if (world < 1 || world > 8) return set_error(SULIMO_EINVAL, "world must be in [1, 8]");
    if (rank < 0 || rank >= world) return set_error(SULIMO_EINVAL, "rank must be in [0, world)");
    if (epoch == 0) return set_error(SULIMO_EINVAL, "epoch must be nonzero");
    if (m_local <= 0 || m_local % 8 || m_valid <= 0 || m_valid > m_local || m_valid % 8 ||
        k <= 0 || k % 32 || n <= 0)
        return set_error(SULIMO_EINVAL, "m_local, m_valid multiples of 8; k of 32; n > 0");
    if (out_dtype != SULIMO_OUT_F16 && out_dtype != SULIMO_OUT_F32)
        return set_error(SULIMO_EINVAL, "bad out_dtype");
    if (f_total % 8 || col0 % 8 || col0 + (size_t)m_valid > f_total)
        return set_error(SULIMO_EINVAL, "col0 + m_valid <= f_total, both multiples of 8");
    if (!scales || !quants || !x || !out_bases || !flags || !release || !tiles_out)
        return set_error(SULIMO_EINVAL, "null pointer");
    for (int r = 0; r < world; r++) {
        if (!out_bases[r] || !flags[r] || !release[r])
            return set_error(SULIMO_EINVAL, "null peer pointer");
        if (!aligned(out_bases[r], 16) || !aligned(flags[r], 4) || !aligned(release[r], 4))
            return set_error(SULIMO_EALIGN, "peer outputs 16-byte, counters 4-byte aligned");
    }
    if (!aligned(x, 16) || !aligned(quants, 16) || !aligned(scales, 2))
        return set_error(SULIMO_EALIGN, "x, quants 16-byte aligned, scales 2-byte");
    if ((st = bind_device(ctx))) return st;
    return sulimo::launch_gemm_allgather(ctx, scales, quants, x, m_local, m_valid, k, n, out_dtype,
                                         out_bases, f_total, col0, flags, release, world, rank,
                                         epoch, tiles_out);
}

int sulimo_cuda_wait_counter(sulimo_ctx* ctx, const unsigned* flag, unsigned target) {
    int st = check_ctx(ctx);
    if (st) return st;
    if (!flag || !aligned(flag, 4)) return set_error(SULIMO_EINVAL, "null / misaligned counter");
    if ((st = bind_device(ctx))) return st;
    return sulimo::launch_wait_counter(ctx, flag, target);
}

int sulimo_cuda_attn_decode_q8_0(sulimo_ctx* ctx, const float* q, const void* k_ring,
                                 const void* v_ring, size_t seq_stride_bytes, size_t capacity,
                                 size_t context_len, int head_count, int head_count_kv,
                                 int head_dim, int batch, float softcap, float* out) {
    int st = check_ctx(ctx);
    if (st) return st;
    if (head_count <= 0 || head_count_kv <= 0 || head_count % head_count_kv != 0)
        return set_error(SULIMO_EINVAL, "head_count must be a positive multiple of head_count_kv");
    if (head_dim <= 0 || head_dim % 32 != 0 || head_dim > 256)
        return set_error(SULIMO_EINVAL, "head_dim must be a multiple of 32 in [32, 256]");
    if (head_count / head_count_kv > 8)
        return set_error(SULIMO_EINVAL, "at most 8 query heads per KV head");
    if (batch < 0 || capacity == 0) return set_error(SULIMO_EINVAL, "bad batch / capacity");
    if (batch == 0) return SULIMO_OK;
    if (!q || !k_ring || !v_ring || !out) return set_error(SULIMO_EINVAL, "null pointer");
    if (!aligned(q, 16) || !aligned(out, 16) || !aligned(k_ring, 2) || !aligned(v_ring, 2) ||
        seq_stride_bytes % 2 != 0)
        return set_error(SULIMO_EALIGN, "q/out 16-byte aligned, rings 2-byte aligned");
    if ((st = bind_device(ctx))) return st;
    int splits = 0;
    size_t pbytes = sulimo::attn_decode_partial_bytes(context_len, capacity, head_count,
                                                      head_count_kv, head_dim, batch,
                                                      ctx->num_sms, seq_stride_bytes, k_ring,
                                                      v_ring, &splits);
    if ((st = sulimo::ensure_workspace(ctx, pbytes))) return st;
    return sulimo::launch_attn_decode(ctx, q, k_ring, v_ring, seq_stride_bytes, capacity,
                                      context_len, head_count, head_count_kv, head_dim, batch,
                                      softcap, out, (float*)ctx->workspace, ctx->workspace_bytes);
}

}  // extern "C"
