// runtime.cu - host runtime behind include/mgpu_cuda.h: device / stream context, buffers,
// events, thread-local error state, argument validation and kernel dispatch.
//
// Replaces, for the matmul path, MVLM's src/engine/device.cpp (context + single in-order
// profiling queue, :141-304), src/engine/memory.cpp (buffers and weight images, :28-111),
// src/engine/compute.cpp (GEMM/GEMV dispatch, :28-152, and the patch_embed / vision_proj
// dispatch, :474-510, :621-651) and src/engine/profiler.cpp (event timing, :25-53).
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <string>
#include <vector>

#include "../../include/mgpu_cuda.h"
#include "kernels.h"

struct mgpu_event;

struct mgpu_device {
    int ordinal;
    cudaStream_t own_stream;
    cudaStream_t stream;
    int sm_count;
    size_t l2_bytes;
    int* d_status;
    int event_mode;
    void* workspace;
    size_t workspace_bytes;
    bool capturing;
    int saved_event_mode;
    std::vector<mgpu_event*> event_pool;
};

struct mgpu_buf {
    mgpu_device* dev;
    void* ptr;
    size_t bytes;
    bool owned;
    int type;
    int layout;
    int64_t rows, cols, ld;
};

struct mgpu_graph {
    mgpu_device* dev;
    cudaGraph_t graph;
    cudaGraphExec_t exec;
};

struct mgpu_event {
    mgpu_device* dev;
    cudaEvent_t start;
    cudaEvent_t end;
    bool timed;
};

namespace {

thread_local int t_err = MGPU_OK;
thread_local char t_msg[512] = "";

void set_error(int code, const char* fmt, ...) {
    t_err = code;
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(t_msg, sizeof(t_msg), fmt, ap);
    va_end(ap);
    fprintf(stderr, "mgpu error %d: %s\n", code, t_msg);
}

bool cuda_ok(cudaError_t e, const char* what) {
    if (e == cudaSuccess) return true;
    set_error(e == cudaErrorMemoryAllocation ? MGPU_ERR_OUT_OF_MEMORY : MGPU_ERR_CUDA, "%s: %s", what,
              cudaGetErrorString(e));
    return false;
}

struct DeviceGuard {
    int prev = -1;
    explicit DeviceGuard(int ordinal) {
        cudaGetDevice(&prev);
        if (prev != ordinal) cudaSetDevice(ordinal);
    }
    ~DeviceGuard() {
        int cur = -1;
        cudaGetDevice(&cur);
        if (prev >= 0 && cur != prev) cudaSetDevice(prev);
    }
};

size_t elem_size(int type) {
    switch (type) {
        case MGPU_F32: return 4;
        case MGPU_F16:
        case MGPU_BF16: return 2;
        default: return 0;
    }
}
bool is_float_type(int t) { return t == MGPU_F32 || t == MGPU_F16 || t == MGPU_BF16; }
bool is_quant_type(int t) { return t == MGPU_Q4_0 || t == MGPU_Q8_0; }
size_t quant_row_bytes(int t, int64_t k) { return (size_t)((k + 31) / 32) * (t == MGPU_Q4_0 ? 18 : 34); }

// Scratch arena layout: [0, 64 KB) holds the split-K tickets of gemv_kn and [64 KB, 128 KB)
// those of the split-K GEMM; both must stay zero between launches (the kernels reset them).
// Everything from kScratchOffset on is free for per-call use (split-K partials, im2col
// patches, staged operands), in stream order.
constexpr size_t kGemvTicketBytes = 64 * 1024;
constexpr size_t kGemmTicketOffset = 64 * 1024;
constexpr size_t kGemmTicketBytes = 64 * 1024;
constexpr size_t kScratchOffset = 128 * 1024;

mgpu_k::LaunchCtx ctx_of(const mgpu_device* d) {
    mgpu_k::LaunchCtx c;
    c.stream = d->stream;
    c.sm_count = d->sm_count;
    c.status = d->d_status;
    c.workspace = d->workspace;
    c.workspace_bytes = d->workspace_bytes;
    return c;
}

// Grow the per-device scratch arena (zero-filled).  Synchronises the stream when it grows.
bool ensure_workspace(mgpu_device* d, size_t bytes) {
    if (bytes <= d->workspace_bytes) return true;
    if (d->capturing) {
        set_error(MGPU_ERR_INVALID_ARG, "scratch must grow (%zu bytes) during graph capture: run the dispatch once "
                  "before capturing it", bytes);
        return false;
    }
    size_t want = std::max(bytes, d->workspace_bytes * 2);
    want = (want + 4095) & ~(size_t)4095;
    // The new arena is zeroed and then takes the old one's contents, so that a caller that
    // has already staged data in the arena (e.g. im2col patches before their GEMM) keeps it.
    void* fresh = nullptr;
    if (!cuda_ok(cudaMalloc(&fresh, want), "cudaMalloc(workspace)")) return false;
    if (!cuda_ok(cudaMemsetAsync(fresh, 0, want, d->stream), "cudaMemsetAsync(workspace)") ||
        (d->workspace && !cuda_ok(cudaMemcpyAsync(fresh, d->workspace, d->workspace_bytes, cudaMemcpyDeviceToDevice,
                                                  d->stream), "cudaMemcpyAsync(workspace)")) ||
        !cuda_ok(cudaStreamSynchronize(d->stream), "cudaStreamSynchronize")) {
        cudaFree(fresh);
        return false;
    }
    if (d->workspace) cudaFree(d->workspace);
    d->workspace = fresh;
    d->workspace_bytes = want;
    return true;
}

mgpu_event* event_begin(mgpu_device* d) {
    if (d->event_mode == 0) return nullptr;
    mgpu_event* ev = nullptr;
    if (!d->event_pool.empty()) {
        ev = d->event_pool.back();
        d->event_pool.pop_back();
    } else {
        ev = new mgpu_event();
        ev->dev = d;
        cudaEventCreate(&ev->start);
        cudaEventCreate(&ev->end);
    }
    ev->timed = d->event_mode == 2;
    if (ev->timed) cudaEventRecord(ev->start, d->stream);
    return ev;
}

mgpu_event* event_end(mgpu_device* d, mgpu_event* ev) {
    if (ev) cudaEventRecord(ev->end, d->stream);
    return ev;
}

// Called after the work it reports on has completed (an event or the stream was waited for).
// The read is a device-to-pageable copy, which returns only once it has landed; it does not
// wait for work queued on the device's stream after that point.  Every upload and fill of the
// library, by contrast, goes on the device's stream: the stream is non-blocking, so an
// operation on the legacy default stream (plain cudaMemcpy / cudaMemset) would not be ordered
// with its kernels.
bool check_status(mgpu_device* d) {
    int st = 0;
    if (!cuda_ok(cudaMemcpy(&st, d->d_status, sizeof(int), cudaMemcpyDeviceToHost), "read status")) return false;
    if (st != 0) {
        cudaMemsetAsync(d->d_status, 0, sizeof(int), d->stream);
        set_error(st, "a kernel's bounded wait expired (device status %d); its output is invalid", st);
        return false;
    }
    return true;
}

// Entry points that return a handle clear the thread-local error first, so that a NULL
// return with mgpu_last_error() == MGPU_OK means "no event recorded", never a stale error.
#define API_ENTRY() \
    do {            \
        t_err = MGPU_OK; \
        t_msg[0] = 0;    \
    } while (0)

#define REQUIRE(cond, ...)                               \
    do {                                                 \
        if (!(cond)) {                                   \
            set_error(MGPU_ERR_INVALID_ARG, __VA_ARGS__); \
            return nullptr;                              \
        }                                                \
    } while (0)

int64_t ld_or(const mgpu_buf* b, int64_t dflt) { return b->ld > 0 ? b->ld : dflt; }

// Validate and enqueue one GEMM; false (with the error set) when it cannot run.
bool gemm_checked(mgpu_device* dev, mgpu_buf* A, mgpu_buf* B, mgpu_buf* C, int M, int N, int K, mgpu_buf* bias,
                  const char* who, size_t scratch_base = kScratchOffset, int act = MGPU_ACT_NONE,
                  mgpu_buf* residual = nullptr, mgpu_buf* mul = nullptr) {
#define GREQ(cond, ...)                                  \
    do {                                                 \
        if (!(cond)) {                                   \
            set_error(MGPU_ERR_INVALID_ARG, __VA_ARGS__); \
            return false;                                \
        }                                                \
    } while (0)
    GREQ(dev && A && B && C, "%s: null argument", who);
    GREQ(M > 0 && N > 0 && K > 0, "%s: M=%d N=%d K=%d must be positive", who, M, N, K);
    mgpu_k::GemmOperand a{A->ptr, A->type, MGPU_LAYOUT_KN, ld_or(A, K)};
    mgpu_k::GemmOperand b{B->ptr, B->type, B->layout, 0};
    if (is_quant_type(B->type)) b.ld = ld_or(B, (int64_t)quant_row_bytes(B->type, K));
    else b.ld = ld_or(B, B->layout == MGPU_LAYOUT_NK ? K : N);
    mgpu_k::GemmOperand c{C->ptr, C->type, MGPU_LAYOUT_KN, ld_or(C, N)};
    GREQ(A->type == MGPU_F16 || A->type == MGPU_BF16, "%s: A must be fp16 or bf16", who);
    if (is_quant_type(B->type))
        GREQ(B->bytes >= (size_t)N * b.ld, "%s: B buffer too small", who);
    else if (B->layout == MGPU_LAYOUT_NK)
        GREQ(B->bytes >= ((size_t)(N - 1) * b.ld + K) * 2, "%s: B buffer too small for N=%d K=%d", who, N, K);
    else
        GREQ(B->bytes >= ((size_t)(K - 1) * b.ld + N) * 2, "%s: B buffer too small for K=%d N=%d", who, K, N);
    GREQ(A->bytes >= ((size_t)(M - 1) * a.ld + K) * 2, "%s: A buffer too small for M=%d K=%d", who, M, K);
    // TMA needs 16-byte aligned bases and row pitches.  The reference accepts any M, N, K, so
    // 16-bit operands whose rows are not 16-byte aligned are first copied into the scratch
    // arena with the pitch rounded up to 8 elements (the pad is never read: the tensor maps
    // keep the logical extents and zero-fill beyond them).
    auto misaligned = [](const void* p, int64_t ld) { return ((uintptr_t)p & 15) || (ld * 2) % 16; };
    const bool stage_a = misaligned(a.ptr, a.ld);
    const bool stage_b = !is_quant_type(B->type) && misaligned(b.ptr, b.ld);
    const int64_t a_ld = (K + 7) / 8 * 8;
    const int64_t b_rows = B->layout == MGPU_LAYOUT_NK ? N : K, b_cols = B->layout == MGPU_LAYOUT_NK ? K : N;
    const int64_t b_ld = (b_cols + 7) / 8 * 8;
    const size_t a_bytes = stage_a ? (((size_t)M * a_ld * 2 + 255) & ~(size_t)255) : 0;
    const size_t b_bytes = stage_b ? (((size_t)b_rows * b_ld * 2 + 255) & ~(size_t)255) : 0;
    // split-K partials (skinny M) go after the staged operands
    const size_t split_bytes = mgpu_k::gemm_split_bytes(ctx_of(dev), a, b, M, N, K);
    if (stage_a || stage_b || split_bytes)
        if (!ensure_workspace(dev, scratch_base + a_bytes + b_bytes + split_bytes)) return false;
    if (stage_a || stage_b) {
        char* ws = (char*)dev->workspace + scratch_base;
        if (stage_a) {
            if (!cuda_ok(cudaMemcpy2DAsync(ws, a_ld * 2, a.ptr, a.ld * 2, (size_t)K * 2, M, cudaMemcpyDeviceToDevice,
                                           dev->stream), "stage A"))
                return false;
            a.ptr = ws;
            a.ld = a_ld;
        }
        if (stage_b) {
            GREQ(B->bytes >= ((size_t)(b_rows - 1) * b.ld + b_cols) * 2, "%s: B buffer too small", who);
            if (!cuda_ok(cudaMemcpy2DAsync(ws + a_bytes, b_ld * 2, b.ptr, b.ld * 2, (size_t)b_cols * 2, b_rows,
                                           cudaMemcpyDeviceToDevice, dev->stream), "stage B"))
                return false;
            b.ptr = ws + a_bytes;
            b.ld = b_ld;
        }
    }
    const char* why = mgpu_k::gemm_check(a, b, c, M, N, K);
    GREQ(!why, "%s: %s", who, why ? why : "");
    GREQ(C->bytes >= ((size_t)(M - 1) * c.ld + N) * elem_size(C->type), "%s: C buffer too small", who);
    if (bias)
        GREQ(is_float_type(bias->type) && bias->bytes >= (size_t)N * elem_size(bias->type),
             "%s: bias must hold N float values", who);
    GREQ(act >= MGPU_ACT_NONE && act <= MGPU_ACT_GELU_AS_SHIPPED, "%s: unknown activation %d", who, act);
    mgpu_k::Epilogue epi;
    epi.act = act;
    // An [M][N] operand the epilogue reads (residual, multiplier): float type, room for M rows,
    // and either C itself (same type and pitch: each element is read and then written by one
    // thread) or disjoint from C (any other overlap would be read after another thread wrote it).
    auto operand_ok = [&](mgpu_buf* X, const char* what, int64_t* ld_out) -> bool {
        const int64_t ld = ld_or(X, N);
        *ld_out = ld;
        GREQ(is_float_type(X->type), "%s: %s must be f32, f16 or bf16", who, what);
        GREQ(ld >= N, "%s: %s row pitch %lld is below N=%d", who, what, (long long)ld, N);
        GREQ(X->bytes >= ((size_t)(M - 1) * ld + N) * elem_size(X->type), "%s: %s buffer too small for M=%d N=%d",
             who, what, M, N);
        if (X->ptr != C->ptr) {
            const char* r0 = (const char*)X->ptr;
            const char* r1 = r0 + ((size_t)(M - 1) * ld + N) * elem_size(X->type);
            const char* c0 = (const char*)C->ptr;
            const char* c1 = c0 + ((size_t)(M - 1) * c.ld + N) * elem_size(C->type);
            GREQ(r1 <= c0 || c1 <= r0, "%s: %s overlaps C without being C", who, what);
        } else {
            GREQ(X->type == C->type && ld == c.ld, "%s: an in-place %s must have C's type and pitch", who, what);
        }
        return true;
    };
    if (residual) {
        if (!operand_ok(residual, "residual", &epi.ldr)) return false;
        epi.resid = residual->ptr;
        epi.resid_type = residual->type;
    }
    if (mul) {
        if (!operand_ok(mul, "up", &epi.ldm)) return false;
        epi.mul = mul->ptr;
        epi.mul_type = mul->type;
    }
#undef GREQ
    mgpu_k::GemmSplitScratch split{};
    if (split_bytes) {
        split.tickets = (unsigned int*)((char*)dev->workspace + kGemmTicketOffset);
        split.max_tickets = kGemmTicketBytes / sizeof(unsigned int);
        split.partials = (float*)((char*)dev->workspace + scratch_base + a_bytes + b_bytes);
        split.max_partials = split_bytes / sizeof(float);
    }
    cudaError_t e = mgpu_k::gemm(ctx_of(dev), a, b, c, bias ? bias->ptr : nullptr, bias ? bias->type : 0, M, N, K,
                                 split_bytes ? &split : nullptr, epi);
    return cuda_ok(e, who);
}

mgpu_event* run_gemm(const mgpu_device* cdev, mgpu_buf* A, mgpu_buf* B, mgpu_buf* C, int M, int N, int K,
                     mgpu_buf* bias, const char* who, int act = MGPU_ACT_NONE, mgpu_buf* residual = nullptr,
                     mgpu_buf* mul = nullptr) {
    API_ENTRY();
    REQUIRE(cdev, "%s: null device", who);
    mgpu_device* dev = const_cast<mgpu_device*>(cdev);
    DeviceGuard g(dev->ordinal);
    mgpu_event* ev = event_begin(dev);
    if (!gemm_checked(dev, A, B, C, M, N, K, bias, who, kScratchOffset, act, residual, mul)) {
        if (ev) dev->event_pool.push_back(ev);
        return nullptr;
    }
    return event_end(dev, ev);
}

}  // namespace

extern "C" {

int mgpu_last_error(void) { return t_err; }
const char* mgpu_last_error_string(void) { return t_msg; }
void mgpu_clear_error(void) {
    t_err = MGPU_OK;
    t_msg[0] = 0;
}

// ------------------------------------------------------------------ device -----------
mgpu_device* mgpu_init_device(int ordinal) {
    API_ENTRY();
    int n = 0;
    if (!cuda_ok(cudaGetDeviceCount(&n), "cudaGetDeviceCount")) return nullptr;
    if (ordinal < 0 || ordinal >= n) {
        set_error(MGPU_ERR_INVALID_ARG, "device ordinal %d out of range (%d devices)", ordinal, n);
        return nullptr;
    }
    DeviceGuard g(ordinal);
    cudaDeviceProp p;
    if (!cuda_ok(cudaGetDeviceProperties(&p, ordinal), "cudaGetDeviceProperties")) return nullptr;
    if (p.major != 10) {
        set_error(MGPU_ERR_UNSUPPORTED, "device %d is sm_%d%d; this library is built for sm_100a only", ordinal,
                  p.major, p.minor);
        return nullptr;
    }
    mgpu_device* d = new mgpu_device();
    d->ordinal = ordinal;
    d->sm_count = p.multiProcessorCount;
    d->l2_bytes = (size_t)p.l2CacheSize;
    d->event_mode = 2;
    d->workspace = nullptr;
    d->workspace_bytes = 0;
    d->capturing = false;
    d->saved_event_mode = 2;
    if (!cuda_ok(cudaStreamCreateWithFlags(&d->own_stream, cudaStreamNonBlocking), "cudaStreamCreate") ||
        !cuda_ok(cudaMalloc(&d->d_status, 256), "cudaMalloc(status)") ||
        !cuda_ok(cudaMemsetAsync(d->d_status, 0, 256, d->own_stream), "cudaMemsetAsync(status)") ||
        !cuda_ok(cudaStreamSynchronize(d->own_stream), "cudaStreamSynchronize")) {
        delete d;
        return nullptr;
    }
    d->stream = d->own_stream;
    return d;
}

void mgpu_release_device(mgpu_device* d) {
    if (!d) return;
    DeviceGuard g(d->ordinal);
    cudaStreamSynchronize(d->stream);
    for (mgpu_event* ev : d->event_pool) {
        cudaEventDestroy(ev->start);
        cudaEventDestroy(ev->end);
        delete ev;
    }
    if (d->workspace) cudaFree(d->workspace);
    cudaFree(d->d_status);
    cudaStreamDestroy(d->own_stream);
    delete d;
}

int mgpu_device_ordinal(const mgpu_device* d) { return d ? d->ordinal : -1; }
int mgpu_device_sm_count(const mgpu_device* d) { return d ? d->sm_count : 0; }
size_t mgpu_device_l2_bytes(const mgpu_device* d) { return d ? d->l2_bytes : 0; }
void* mgpu_device_stream(const mgpu_device* d) { return d ? (void*)d->stream : nullptr; }

int mgpu_set_stream(mgpu_device* d, void* s) {
    if (!d) {
        set_error(MGPU_ERR_INVALID_ARG, "mgpu_set_stream: null device");
        return MGPU_ERR_INVALID_ARG;
    }
    d->stream = s ? (cudaStream_t)s : d->own_stream;
    return MGPU_OK;
}

int mgpu_set_event_mode(mgpu_device* d, int mode) {
    if (!d || mode < 0 || mode > 2) {
        set_error(MGPU_ERR_INVALID_ARG, "mgpu_set_event_mode: bad arguments");
        return MGPU_ERR_INVALID_ARG;
    }
    d->event_mode = mode;
    return MGPU_OK;
}

int mgpu_finish(mgpu_device* d) {
    if (!d) {
        set_error(MGPU_ERR_INVALID_ARG, "mgpu_finish: null device");
        return MGPU_ERR_INVALID_ARG;
    }
    DeviceGuard g(d->ordinal);
    if (!cuda_ok(cudaStreamSynchronize(d->stream), "cudaStreamSynchronize")) return t_err;
    if (!check_status(d)) return t_err;
    return MGPU_OK;
}

// ------------------------------------------------------------------ memory -----------
static mgpu_buf* new_buf(mgpu_device* d, void* p, size_t bytes, bool owned) {
    mgpu_buf* b = new mgpu_buf();
    b->dev = d;
    b->ptr = p;
    b->bytes = bytes;
    b->owned = owned;
    b->type = MGPU_F16;
    b->layout = MGPU_LAYOUT_KN;
    b->rows = b->cols = b->ld = 0;
    return b;
}

mgpu_buf* mgpu_create_buffer(mgpu_device* d, size_t bytes, const void* host_src) {
    API_ENTRY();
    REQUIRE(d && bytes > 0, "mgpu_create_buffer: null device or zero size");
    DeviceGuard g(d->ordinal);
    void* p = nullptr;
    // Allocation rounded up to 256 bytes so that 16-byte vector / bulk reads of the last
    // row never leave the allocation.
    if (!cuda_ok(cudaMalloc(&p, (bytes + 255) & ~(size_t)255), "cudaMalloc")) return nullptr;
    // On the device's stream, then waited for: a plain cudaMemcpy from pageable memory may
    // return before its last DMA lands, and it runs on the legacy default stream, which the
    // device's non-blocking stream does not wait for (a kernel launched next could read the
    // upload's tail before it arrived).
    if (host_src && (!cuda_ok(cudaMemcpyAsync(p, host_src, bytes, cudaMemcpyHostToDevice, d->stream), "upload") ||
                     !cuda_ok(cudaStreamSynchronize(d->stream), "cudaStreamSynchronize"))) {
        cudaFree(p);
        return nullptr;
    }
    return new_buf(d, p, bytes, true);
}

mgpu_buf* mgpu_create_weight_image(mgpu_device* d, int rows, int cols, const uint16_t* data) {
    API_ENTRY();
    REQUIRE(d && rows > 0 && cols > 0, "mgpu_create_weight_image: bad arguments");
    const int64_t ld = (cols + 7) / 8 * 8;
    mgpu_buf* b = mgpu_create_buffer(d, (size_t)rows * ld * 2, nullptr);
    if (!b) return nullptr;
    DeviceGuard g(d->ordinal);
    if (!cuda_ok(cudaMemsetAsync(b->ptr, 0, b->bytes, d->stream), "cudaMemsetAsync") ||
        (data && !cuda_ok(cudaMemcpy2DAsync(b->ptr, ld * 2, data, (size_t)cols * 2, (size_t)cols * 2, rows,
                                            cudaMemcpyHostToDevice, d->stream),
                          "cudaMemcpy2DAsync")) ||
        !cuda_ok(cudaStreamSynchronize(d->stream), "cudaStreamSynchronize")) {
        mgpu_release_buffer(b);
        return nullptr;
    }
    b->type = MGPU_F16;
    b->layout = MGPU_LAYOUT_KN;
    b->rows = rows;
    b->cols = cols;
    b->ld = ld;
    return b;
}

mgpu_buf* mgpu_wrap_buffer(mgpu_device* d, void* device_ptr, size_t bytes) {
    API_ENTRY();
    REQUIRE(d && device_ptr && bytes > 0, "mgpu_wrap_buffer: bad arguments");
    return new_buf(d, device_ptr, bytes, false);
}

mgpu_buf* mgpu_buf_view(mgpu_buf* b, size_t offset, size_t bytes) {
    API_ENTRY();
    REQUIRE(b && bytes > 0 && offset + bytes <= b->bytes, "mgpu_buf_view: range outside the buffer");
    mgpu_buf* v = new_buf(b->dev, (char*)b->ptr + offset, bytes, false);
    v->type = b->type;
    v->layout = b->layout;
    return v;
}

int mgpu_buf_set_format(mgpu_buf* b, int type, int layout, int64_t rows, int64_t cols, int64_t ld) {
    if (!b || !(is_float_type(type) || is_quant_type(type)) || (layout != MGPU_LAYOUT_KN && layout != MGPU_LAYOUT_NK) ||
        rows < 0 || cols < 0 || ld < 0) {
        set_error(MGPU_ERR_INVALID_ARG, "mgpu_buf_set_format: bad arguments");
        return MGPU_ERR_INVALID_ARG;
    }
    b->type = type;
    b->layout = layout;
    b->rows = rows;
    b->cols = cols;
    b->ld = ld;
    return MGPU_OK;
}

void* mgpu_buf_device_ptr(const mgpu_buf* b) { return b ? b->ptr : nullptr; }
size_t mgpu_buf_bytes(const mgpu_buf* b) { return b ? b->bytes : 0; }

int mgpu_buf_write(mgpu_buf* b, size_t off, const void* src, size_t bytes) {
    if (!b || !src || off + bytes > b->bytes) {
        set_error(MGPU_ERR_INVALID_ARG, "mgpu_buf_write: range outside the buffer");
        return MGPU_ERR_INVALID_ARG;
    }
    DeviceGuard g(b->dev->ordinal);
    if (!cuda_ok(cudaMemcpyAsync((char*)b->ptr + off, src, bytes, cudaMemcpyHostToDevice, b->dev->stream), "write") ||
        !cuda_ok(cudaStreamSynchronize(b->dev->stream), "write sync"))
        return t_err;
    return MGPU_OK;
}

int mgpu_buf_read(const mgpu_buf* b, size_t off, void* dst, size_t bytes) {
    if (!b || !dst || off + bytes > b->bytes) {
        set_error(MGPU_ERR_INVALID_ARG, "mgpu_buf_read: range outside the buffer");
        return MGPU_ERR_INVALID_ARG;
    }
    DeviceGuard g(b->dev->ordinal);
    if (!cuda_ok(cudaMemcpyAsync(dst, (const char*)b->ptr + off, bytes, cudaMemcpyDeviceToHost, b->dev->stream), "read") ||
        !cuda_ok(cudaStreamSynchronize(b->dev->stream), "read sync"))
        return t_err;
    if (!check_status(b->dev)) return t_err;
    return MGPU_OK;
}

int mgpu_buf_write_async(mgpu_buf* b, size_t off, const void* src, size_t bytes) {
    if (!b || !src || off + bytes > b->bytes) {
        set_error(MGPU_ERR_INVALID_ARG, "mgpu_buf_write_async: range outside the buffer");
        return MGPU_ERR_INVALID_ARG;
    }
    DeviceGuard g(b->dev->ordinal);
    if (!cuda_ok(cudaMemcpyAsync((char*)b->ptr + off, src, bytes, cudaMemcpyHostToDevice, b->dev->stream), "write_async"))
        return t_err;
    return MGPU_OK;
}

int mgpu_buf_read_async(const mgpu_buf* b, size_t off, void* dst, size_t bytes) {
    if (!b || !dst || off + bytes > b->bytes) {
        set_error(MGPU_ERR_INVALID_ARG, "mgpu_buf_read_async: range outside the buffer");
        return MGPU_ERR_INVALID_ARG;
    }
    DeviceGuard g(b->dev->ordinal);
    if (!cuda_ok(cudaMemcpyAsync(dst, (const char*)b->ptr + off, bytes, cudaMemcpyDeviceToHost, b->dev->stream), "read_async"))
        return t_err;
    return MGPU_OK;
}

int mgpu_buf_copy_async(mgpu_buf* dst, size_t dst_offset, const mgpu_buf* src, size_t src_offset, size_t bytes) {
    if (!dst || !src || src->dev != dst->dev || dst_offset + bytes > dst->bytes || src_offset + bytes > src->bytes) {
        set_error(MGPU_ERR_INVALID_ARG, "mgpu_buf_copy_async: bad arguments");
        return MGPU_ERR_INVALID_ARG;
    }
    if (bytes == 0) return MGPU_OK;
    DeviceGuard g(dst->dev->ordinal);
    if (!cuda_ok(cudaMemcpyAsync((char*)dst->ptr + dst_offset, (const char*)src->ptr + src_offset, bytes,
                                 cudaMemcpyDeviceToDevice, dst->dev->stream), "mgpu_buf_copy_async"))
        return t_err;
    return MGPU_OK;
}

void* mgpu_host_alloc(size_t bytes) {
    void* p = nullptr;
    if (!cuda_ok(cudaMallocHost(&p, bytes), "cudaMallocHost")) return nullptr;
    return p;
}
void mgpu_host_free(void* p) {
    if (p) cudaFreeHost(p);
}

void mgpu_release_buffer(mgpu_buf* b) {
    if (!b) return;
    if (b->owned && b->ptr) {
        DeviceGuard g(b->dev->ordinal);
        cudaStreamSynchronize(b->dev->stream);
        cudaFree(b->ptr);
    }
    delete b;
}

mgpu_buf* mgpu_upload_weight(mgpu_device* d, const mgpu_tensor_info* t, const void* host) {
    API_ENTRY();
    REQUIRE(d && t && host, "mgpu_upload_weight: null argument");
    REQUIRE(t->n_dims >= 1 && t->n_dims <= 4, "mgpu_upload_weight: '%s' has %u dims", t->name, t->n_dims);
    REQUIRE(is_float_type((int)t->type) || is_quant_type((int)t->type),
            "mgpu_upload_weight: '%s' has unsupported type %u", t->name, t->type);
    const int64_t cols = (int64_t)t->dims[0];
    int64_t rows = 1;
    for (uint32_t i = 1; i < t->n_dims; ++i) rows *= (int64_t)t->dims[i];
    if (is_quant_type((int)t->type)) REQUIRE(cols % 32 == 0, "mgpu_upload_weight: '%s' ne0 %% 32 != 0", t->name);
    const size_t row_bytes = is_quant_type((int)t->type) ? quant_row_bytes((int)t->type, cols) : (size_t)cols * elem_size((int)t->type);
    REQUIRE(t->data_size >= (size_t)rows * row_bytes, "mgpu_upload_weight: '%s' data_size %zu < %zu", t->name,
            t->data_size, (size_t)rows * row_bytes);
    mgpu_buf* b = mgpu_create_buffer(d, t->data_size, host);
    if (!b) return nullptr;
    b->type = (int)t->type;
    b->layout = MGPU_LAYOUT_NK;
    b->rows = rows;
    b->cols = cols;
    b->ld = is_quant_type((int)t->type) ? (int64_t)row_bytes : cols;
    return b;
}

// ------------------------------------------------------------------ dispatch ---------
mgpu_event* mgpu_dispatch_gemm_naive(const mgpu_device* d, mgpu_program, mgpu_buf* A, mgpu_buf* B, mgpu_buf* C,
                                     int M, int N, int K) {
    API_ENTRY();
    return run_gemm(d, A, B, C, M, N, K, nullptr, "dispatch_gemm_naive");
}
mgpu_event* mgpu_dispatch_gemm_tiled(const mgpu_device* d, mgpu_program, mgpu_buf* A, mgpu_buf* B, mgpu_buf* C,
                                     int M, int N, int K) {
    API_ENTRY();
    return run_gemm(d, A, B, C, M, N, K, nullptr, "dispatch_gemm_tiled");
}
mgpu_event* mgpu_dispatch_gemm_image(const mgpu_device* d, mgpu_program, mgpu_buf* A, mgpu_buf* B, mgpu_buf* C,
                                     int M, int N, int K) {
    API_ENTRY();
    return run_gemm(d, A, B, C, M, N, K, nullptr, "dispatch_gemm_image");
}
mgpu_event* mgpu_gemm(const mgpu_device* d, mgpu_buf* A, mgpu_buf* B, mgpu_buf* C, int M, int N, int K,
                      mgpu_buf* bias) {
    API_ENTRY();
    return run_gemm(d, A, B, C, M, N, K, bias, "mgpu_gemm");
}
mgpu_event* mgpu_gemm_fused(const mgpu_device* d, mgpu_buf* A, mgpu_buf* B, mgpu_buf* C, int M, int N, int K,
                            mgpu_buf* bias, int act, mgpu_buf* residual) {
    API_ENTRY();
    return run_gemm(d, A, B, C, M, N, K, bias, "mgpu_gemm_fused", act, residual);
}
mgpu_event* mgpu_gemm_silu_gate(const mgpu_device* d, mgpu_buf* A, mgpu_buf* W_gate, mgpu_buf* up, mgpu_buf* out,
                                int M, int N, int K) {
    API_ENTRY();
    REQUIRE(up, "mgpu_gemm_silu_gate: null up");
    return run_gemm(d, A, W_gate, out, M, N, K, nullptr, "mgpu_gemm_silu_gate", MGPU_ACT_SILU, nullptr, up);
}
mgpu_event* mgpu_gemm_q(const mgpu_device* d, mgpu_buf* A, mgpu_buf* W, mgpu_buf* C, int M, int N, int K, int type,
                        mgpu_buf* bias) {
    API_ENTRY();
    REQUIRE(W && is_quant_type(type), "mgpu_gemm_q: type must be Q4_0 or Q8_0");
    REQUIRE(W->type == type || W->type == MGPU_F16, "mgpu_gemm_q: W is tagged with type %d, not %d", W->type, type);
    W->type = type;
    W->layout = MGPU_LAYOUT_NK;
    return run_gemm(d, A, W, C, M, N, K, bias, "mgpu_gemm_q");
}

mgpu_event* mgpu_dispatch_gemv(const mgpu_device* cd, mgpu_program, mgpu_buf* x, mgpu_buf* W, mgpu_buf* y, int N,
                               int K) {
    API_ENTRY();
    REQUIRE(cd && x && W && y, "dispatch_gemv: null argument");
    REQUIRE(N > 0 && K > 0, "dispatch_gemv: N=%d K=%d", N, K);
    mgpu_device* d = const_cast<mgpu_device*>(cd);
    REQUIRE(is_float_type(x->type) && is_float_type(y->type), "dispatch_gemv: x and y must be f32/f16/bf16");
    REQUIRE(x->bytes >= (size_t)K * elem_size(x->type), "dispatch_gemv: x holds fewer than K=%d values", K);
    REQUIRE(y->bytes >= (size_t)N * elem_size(y->type), "dispatch_gemv: y holds fewer than N=%d values", N);
    DeviceGuard g(d->ordinal);
    cudaError_t e;
    mgpu_event* ev = nullptr;
    if (is_quant_type(W->type)) {
        REQUIRE(W->layout == MGPU_LAYOUT_NK, "dispatch_gemv: quantised W must be GGUF [N][K/32]");
        REQUIRE(K % 32 == 0, "dispatch_gemv: quantised W needs K %% 32 == 0 (K=%d)", K);
        const int64_t rb = ld_or(W, (int64_t)quant_row_bytes(W->type, K));
        REQUIRE(rb == (int64_t)quant_row_bytes(W->type, K), "dispatch_gemv: quantised rows must be dense");
        REQUIRE(W->bytes >= (size_t)N * rb, "dispatch_gemv: W holds fewer than N=%d rows", N);
        ev = event_begin(d);
        e = mgpu_k::gemv_q(ctx_of(d), W->type, (const uint8_t*)W->ptr, x->type, x->ptr, y->type, y->ptr, N, K);
    } else if (W->layout == MGPU_LAYOUT_NK) {
        const int64_t ld = ld_or(W, K);
        REQUIRE(ld >= K && W->bytes >= ((size_t)(N - 1) * ld + K) * elem_size(W->type), "dispatch_gemv: W too small");
        ev = event_begin(d);
        e = mgpu_k::gemv_nk(ctx_of(d), W->type, W->ptr, ld, x->type, x->ptr, y->type, y->ptr, N, K);
    } else {
        const int64_t ld = ld_or(W, N);
        REQUIRE(ld >= N && W->bytes >= ((size_t)(K - 1) * ld + N) * elem_size(W->type), "dispatch_gemv: W too small");
        const size_t need = mgpu_k::gemv_kn_scratch_bytes(N, K, d->sm_count, nullptr);
        REQUIRE((size_t)((N + 255) / 256) * 4 <= kGemvTicketBytes, "dispatch_gemv: N=%d too large for KN layout", N);
        if (!ensure_workspace(d, kScratchOffset + need)) return nullptr;
        unsigned int* counters = (unsigned int*)d->workspace;
        float* partials = (float*)((char*)d->workspace + kScratchOffset);
        ev = event_begin(d);
        e = mgpu_k::gemv_kn(ctx_of(d), W->type, W->ptr, ld, x->type, x->ptr, y->type, y->ptr, N, K, partials, counters);
    }
    if (!cuda_ok(e, "dispatch_gemv")) {
        if (ev) d->event_pool.push_back(ev);
        return nullptr;
    }
    return event_end(d, ev);
}

int mgpu_dispatch_gemv_noalloc(const mgpu_device* cd, mgpu_buf* x, mgpu_buf* W, mgpu_buf* y, int N, int K) {
    t_err = MGPU_OK;
    t_msg[0] = 0;
    auto fail = [](const char* fmt, auto... args) {
        set_error(MGPU_ERR_INVALID_ARG, fmt, args...);
        return (int)MGPU_ERR_INVALID_ARG;
    };
    if (!cd || !x || !W || !y) return fail("mgpu_dispatch_gemv_noalloc: null argument");
    if (N <= 0 || K <= 0) return fail("mgpu_dispatch_gemv_noalloc: N=%d K=%d must be positive", N, K);
    if ((size_t)N > mgpu_k::gemv_kn_noalloc_max_n())
        return fail("mgpu_dispatch_gemv_noalloc: N=%d exceeds the fixed scratch limit N <= %zu", N,
                    mgpu_k::gemv_kn_noalloc_max_n());
    if (!is_float_type(W->type) || W->layout != MGPU_LAYOUT_KN)
        return fail("mgpu_dispatch_gemv_noalloc: W must be dense f32/f16/bf16 stored [K][N]");
    if (!is_float_type(x->type) || !is_float_type(y->type))
        return fail("mgpu_dispatch_gemv_noalloc: x and y must be f32/f16/bf16");
    const int64_t ld = ld_or(W, N);
    if (ld < N || W->bytes < ((size_t)(K - 1) * ld + N) * elem_size(W->type))
        return fail("mgpu_dispatch_gemv_noalloc: W too small for K=%d N=%d", K, N);
    if (x->bytes < (size_t)K * elem_size(x->type)) return fail("mgpu_dispatch_gemv_noalloc: x holds fewer than K=%d values", K);
    if (y->bytes < (size_t)N * elem_size(y->type)) return fail("mgpu_dispatch_gemv_noalloc: y holds fewer than N=%d values", N);
    DeviceGuard g(cd->ordinal);
    if (!cuda_ok(mgpu_k::gemv_kn_noalloc(ctx_of(cd), W->type, W->ptr, ld, x->type, x->ptr, y->type, y->ptr, N, K),
                 "mgpu_dispatch_gemv_noalloc"))
        return t_err;
    return MGPU_OK;
}

mgpu_event* mgpu_gemv_q(const mgpu_device* d, mgpu_buf* x, mgpu_buf* W, mgpu_buf* y, int N, int K, int type) {
    API_ENTRY();
    REQUIRE(W && is_quant_type(type), "mgpu_gemv_q: type must be Q4_0 or Q8_0");
    REQUIRE(W->type == type || W->type == MGPU_F16, "mgpu_gemv_q: W is tagged with type %d, not %d", W->type, type);
    W->type = type;
    W->layout = MGPU_LAYOUT_NK;
    return mgpu_dispatch_gemv(d, nullptr, x, W, y, N, K);
}

mgpu_event* mgpu_dispatch_rms_norm(const mgpu_device* cd, mgpu_program, mgpu_buf* input, mgpu_buf* output,
                                   mgpu_buf* weight, int num_rows, int hidden_size, float eps) {
    API_ENTRY();
    REQUIRE(cd && input && output && weight, "dispatch_rms_norm: null argument");
    REQUIRE(num_rows > 0 && hidden_size > 0, "dispatch_rms_norm: num_rows=%d hidden_size=%d", num_rows, hidden_size);
    REQUIRE(is_float_type(input->type) && output->type == input->type,
            "dispatch_rms_norm: input and output must be f16 / bf16 / f32 of one type");
    REQUIRE(is_float_type(weight->type) && weight->bytes >= (size_t)hidden_size * elem_size(weight->type),
            "dispatch_rms_norm: weight must hold hidden_size float values");
    const size_t bytes = (size_t)num_rows * hidden_size * elem_size(input->type);
    REQUIRE(input->bytes >= bytes && output->bytes >= bytes, "dispatch_rms_norm: buffers smaller than rows x hidden");
    mgpu_device* d = const_cast<mgpu_device*>(cd);
    DeviceGuard g(d->ordinal);
    mgpu_event* ev = event_begin(d);
    if (!cuda_ok(mgpu_k::rms_norm(ctx_of(d), input->type, input->ptr, output->ptr, weight->type, weight->ptr, num_rows,
                                  hidden_size, eps), "dispatch_rms_norm")) {
        if (ev) d->event_pool.push_back(ev);
        return nullptr;
    }
    return event_end(d, ev);
}

mgpu_event* mgpu_gemv_q_rmsnorm(const mgpu_device* cd, mgpu_buf* x, mgpu_buf* gamma, float eps, mgpu_buf* W,
                                mgpu_buf* y, int N, int K, int type) {
    API_ENTRY();
    REQUIRE(cd && x && gamma && W && y, "gemv_q_rmsnorm: null argument");
    REQUIRE(N > 0 && K > 0 && K % 32 == 0, "gemv_q_rmsnorm: N=%d K=%d", N, K);
    REQUIRE(is_quant_type(type) && (W->type == type || W->type == MGPU_F16), "gemv_q_rmsnorm: W must be Q4_0 / Q8_0");
    REQUIRE(is_float_type(x->type) && is_float_type(y->type), "gemv_q_rmsnorm: x and y must be f32 / f16 / bf16");
    REQUIRE(is_float_type(gamma->type) && gamma->bytes >= (size_t)K * elem_size(gamma->type),
            "gemv_q_rmsnorm: norm_weight must hold K float values");
    REQUIRE(x->bytes >= (size_t)K * elem_size(x->type), "gemv_q_rmsnorm: x holds fewer than K=%d values", K);
    REQUIRE(y->bytes >= (size_t)N * elem_size(y->type), "gemv_q_rmsnorm: y holds fewer than N=%d values", N);
    const size_t rb = quant_row_bytes(type, K);
    REQUIRE(W->bytes >= (size_t)N * rb, "gemv_q_rmsnorm: W holds fewer than N=%d rows", N);
    W->type = type;
    W->layout = MGPU_LAYOUT_NK;
    mgpu_device* d = const_cast<mgpu_device*>(cd);
    DeviceGuard g(d->ordinal);
    mgpu_event* ev = event_begin(d);
    cudaError_t e = mgpu_k::gemv_q_norm(ctx_of(d), type, (const uint8_t*)W->ptr, x->type, x->ptr, gamma->type,
                                        gamma->ptr, eps, y->type, y->ptr, N, K);
    if (e == cudaErrorNotSupported) {
        // normalise into the scratch arena, then the plain GEMV (stream-ordered)
        const size_t xb = ((size_t)K * elem_size(x->type) + 255) & ~(size_t)255;
        if (!ensure_workspace(d, kScratchOffset + xb)) {
            if (ev) d->event_pool.push_back(ev);
            return nullptr;
        }
        void* xn = (char*)d->workspace + kScratchOffset;
        e = mgpu_k::rms_norm(ctx_of(d), x->type, x->ptr, xn, gamma->type, gamma->ptr, 1, K, eps);
        if (e == cudaSuccess)
            e = mgpu_k::gemv_q(ctx_of(d), type, (const uint8_t*)W->ptr, x->type, xn, y->type, y->ptr, N, K);
    }
    if (!cuda_ok(e, "gemv_q_rmsnorm")) {
        if (ev) d->event_pool.push_back(ev);
        return nullptr;
    }
    return event_end(d, ev);
}

// ------------------------------------------------------------------ GEMV chain -------
struct mgpu_gemv_chain {
    mgpu_device* dev;
    int n;
    int qtype;
    mgpu_k::ChainStage* d_stages;   // the stage table the kernel reads
    unsigned int* d_sync;           // launch counter (u64), finish ticket, poison
    unsigned long long* d_flags;    // per-stage counts of the CTAs that finished it
    unsigned long long* d_times;    // n + 1 words for timed runs (allocated on first use)
};

namespace {

struct Range {
    const char* lo;
    const char* hi;
    bool overlaps(const Range& o) const { return lo < o.hi && o.lo < hi; }
    bool contains(const Range& o) const { return lo <= o.lo && o.hi <= hi; }
};

Range range_of(const mgpu_buf* b, size_t bytes) {
    const char* p = static_cast<const char*>(b->ptr);
    return Range{p, p + bytes};
}

void free_chain(mgpu_gemv_chain* c) {
    if (!c) return;
    if (c->d_stages) cudaFree(c->d_stages);
    if (c->d_sync) cudaFree(c->d_sync);
    if (c->d_flags) cudaFree(c->d_flags);
    if (c->d_times) cudaFree(c->d_times);
    delete c;
}

}  // namespace

mgpu_gemv_chain* mgpu_gemv_chain_create(const mgpu_device* cd, const mgpu_gemv_link* links, int n) {
    API_ENTRY();
    REQUIRE(cd && links && n > 0, "gemv_chain_create: null device / links or n_links=%d", n);
    mgpu_device* d = const_cast<mgpu_device*>(cd);
    if (n > mgpu_k::chain_max_links()) {
        set_error(MGPU_ERR_UNSUPPORTED, "gemv_chain_create: %d links; a chain holds at most %d (split it)", n,
                  mgpu_k::chain_max_links());
        return nullptr;
    }
    const int qtype = links[0].W ? links[0].W->type : -1;
    REQUIRE(is_quant_type(qtype), "gemv_chain_create: link 0: W must be GGUF Q4_0 or Q8_0");
    std::vector<Range> yr(n), wr(n), xr(n);
    std::vector<int> src(n, -1);
    for (int i = 0; i < n; ++i) {
        const mgpu_gemv_link& L = links[i];
        REQUIRE(L.x && L.W && L.y, "gemv_chain_create: link %d: null buffer", i);
        REQUIRE(L.N > 0 && L.K > 0, "gemv_chain_create: link %d: N=%d K=%d", i, L.N, L.K);
        REQUIRE(L.W->type == qtype, "gemv_chain_create: link %d: W type %d differs from link 0's %d", i, L.W->type,
                qtype);
        REQUIRE(L.W->layout == MGPU_LAYOUT_NK, "gemv_chain_create: link %d: W must be GGUF [N][K/32]", i);
        const size_t rb = quant_row_bytes(qtype, L.K);
        REQUIRE(L.K % 32 == 0 && ld_or(L.W, (int64_t)rb) == (int64_t)rb,
                "gemv_chain_create: link %d: W rows must be dense GGUF blocks", i);
        REQUIRE(L.W->bytes >= (size_t)L.N * rb, "gemv_chain_create: link %d: W holds fewer than N=%d rows", i, L.N);
        REQUIRE(((uintptr_t)L.W->ptr & 15) == 0, "gemv_chain_create: link %d: W must be 16-byte aligned", i);
        REQUIRE(is_float_type(L.x->type) && is_float_type(L.y->type),
                "gemv_chain_create: link %d: x and y must be f32 / f16 / bf16", i);
        REQUIRE(L.x->bytes >= (size_t)L.K * elem_size(L.x->type), "gemv_chain_create: link %d: x holds fewer than K=%d",
                i, L.K);
        REQUIRE(L.y->bytes >= (size_t)L.N * elem_size(L.y->type), "gemv_chain_create: link %d: y holds fewer than N=%d",
                i, L.N);
        if (!mgpu_k::chain_shape_ok(L.K)) {
            set_error(MGPU_ERR_UNSUPPORTED, "gemv_chain_create: link %d: K=%d (the chain takes 1024 <= K <= 8192, "
                      "K %% 1024 == 0); run it with mgpu_gemv_q", i, L.K);
            return nullptr;
        }
        wr[i] = range_of(L.W, (size_t)L.N * rb);
        yr[i] = range_of(L.y, (size_t)L.N * elem_size(L.y->type));
        xr[i] = range_of(L.x, (size_t)L.K * elem_size(L.x->type));
        // x: the output of the latest earlier link whose y it touches, or an external vector
        for (int j = i - 1; j >= 0; --j) {
            if (!yr[j].overlaps(xr[i])) continue;
            REQUIRE(yr[j].contains(xr[i]) && links[j].y->type == L.x->type,
                    "gemv_chain_create: link %d: x overlaps link %d's y without being a view of it of the same type",
                    i, j);
            const size_t off = (size_t)(xr[i].lo - yr[j].lo);
            const size_t es = elem_size(L.x->type);
            REQUIRE(off % es == 0, "gemv_chain_create: link %d: x starts inside an element of link %d's y", i, j);
            src[i] = j;
            break;
        }
        // x is read four elements at a time
        REQUIRE(((uintptr_t)L.x->ptr % (4 * elem_size(L.x->type))) == 0,
                "gemv_chain_create: link %d: x must be aligned to 4 elements", i);
    }
    // hazards the chain's overlapped execution would expose: outputs must not overlap each other,
    // any weights or any external input
    for (int i = 0; i < n; ++i) {
        for (int j = 0; j < n; ++j) {
            REQUIRE(!yr[i].overlaps(wr[j]), "gemv_chain_create: link %d's y overlaps link %d's W", i, j);
            if (j != i) REQUIRE(!yr[i].overlaps(yr[j]), "gemv_chain_create: links %d and %d write overlapping y", i, j);
            if (src[j] < 0)
                REQUIRE(!yr[i].overlaps(xr[j]), "gemv_chain_create: link %d's y overlaps link %d's input x", i, j);
        }
    }
    std::vector<int> post(n, 0);
    for (int i = 0; i < n; ++i)
        if (src[i] >= 0) post[src[i]] = 1;
    DeviceGuard g(d->ordinal);
    mgpu_gemv_chain* c = new mgpu_gemv_chain();
    c->dev = d;
    c->n = n;
    c->qtype = qtype;
    auto fail = [&](cudaError_t e, const char* what) -> mgpu_gemv_chain* {
        cuda_ok(e, what);
        free_chain(c);
        return nullptr;
    };
    cudaError_t e = cudaMalloc(&c->d_stages, sizeof(mgpu_k::ChainStage) * n);
    if (e != cudaSuccess) return fail(e, "gemv_chain_create: cudaMalloc(stage table)");
    e = cudaMalloc(&c->d_sync, 64);
    if (e != cudaSuccess) return fail(e, "gemv_chain_create: cudaMalloc(sync)");
    const size_t flag_bytes = mgpu_k::chain_flag_bytes(d->sm_count);
    e = cudaMalloc(&c->d_flags, flag_bytes);
    if (e != cudaSuccess) return fail(e, "gemv_chain_create: cudaMalloc(flags)");
    std::vector<mgpu_k::ChainStage> st(n);
    for (int i = 0; i < n; ++i) {
        const mgpu_gemv_link& L = links[i];
        mgpu_k::ChainStage& s = st[i];
        memset(&s, 0, sizeof(s));
        s.W = static_cast<const uint8_t*>(L.W->ptr);
        s.x = L.x->ptr;
        s.y = L.y->ptr;
        s.N = L.N;
        s.K = L.K;
        s.row_bytes = (uint32_t)quant_row_bytes(qtype, L.K);
        s.xtype = L.x->type;
        s.ytype = L.y->type;
        s.dep = src[i];
        s.post = post[i];
    }
    e = cudaMemcpyAsync(c->d_stages, st.data(), sizeof(mgpu_k::ChainStage) * n, cudaMemcpyHostToDevice, d->stream);
    if (e != cudaSuccess) return fail(e, "gemv_chain_create: stage table upload");
    e = cudaMemsetAsync(c->d_sync, 0, 64, d->stream);
    if (e != cudaSuccess) return fail(e, "gemv_chain_create: clear sync words");
    e = cudaMemsetAsync(c->d_flags, 0, flag_bytes, d->stream);
    if (e != cudaSuccess) return fail(e, "gemv_chain_create: clear flags");
    e = cudaStreamSynchronize(d->stream);
    if (e != cudaSuccess) return fail(e, "gemv_chain_create: synchronize");
    return c;
}

mgpu_event* mgpu_gemv_chain_run(mgpu_gemv_chain* c) {
    API_ENTRY();
    REQUIRE(c, "gemv_chain_run: null chain");
    mgpu_device* d = c->dev;
    DeviceGuard g(d->ordinal);
    mgpu_event* ev = event_begin(d);
    if (!cuda_ok(mgpu_k::gemv_chain(ctx_of(d), c->qtype, c->d_stages, c->n, c->d_sync, c->d_flags, nullptr), "gemv_chain_run")) {
        if (ev) d->event_pool.push_back(ev);
        return nullptr;
    }
    return event_end(d, ev);
}

int mgpu_gemv_chain_run_timed(mgpu_gemv_chain* c, double* end_us) {
    t_err = MGPU_OK;
    if (!c || !end_us) {
        set_error(MGPU_ERR_INVALID_ARG, "gemv_chain_run_timed: null argument");
        return MGPU_ERR_INVALID_ARG;
    }
    mgpu_device* d = c->dev;
    if (d->capturing) {
        set_error(MGPU_ERR_INVALID_ARG, "gemv_chain_run_timed: synchronous, not capturable");
        return MGPU_ERR_INVALID_ARG;
    }
    DeviceGuard g(d->ordinal);
    const size_t words = (size_t)c->n + 1;
    if (!c->d_times && !cuda_ok(cudaMalloc(&c->d_times, words * 8), "gemv_chain_run_timed: cudaMalloc"))
        return t_err;
    if (!cuda_ok(cudaMemsetAsync(c->d_times, 0, (size_t)c->n * 8, d->stream), "gemv_chain_run_timed: clear") ||
        !cuda_ok(cudaMemsetAsync(c->d_times + c->n, 0xFF, 8, d->stream), "gemv_chain_run_timed: clear"))
        return t_err;
    if (!cuda_ok(mgpu_k::gemv_chain(ctx_of(d), c->qtype, c->d_stages, c->n, c->d_sync, c->d_flags, c->d_times),
                 "gemv_chain_run_timed"))
        return t_err;
    std::vector<unsigned long long> t(words);
    if (!cuda_ok(cudaMemcpyAsync(t.data(), c->d_times, words * 8, cudaMemcpyDeviceToHost, d->stream),
                 "gemv_chain_run_timed: read times") ||
        !cuda_ok(cudaStreamSynchronize(d->stream), "gemv_chain_run_timed: synchronize"))
        return t_err;
    if (!check_status(d)) return t_err;
    for (int i = 0; i < c->n; ++i) end_us[i] = t[i] >= t[c->n] ? (double)(t[i] - t[c->n]) * 1e-3 : 0.0;
    return MGPU_OK;
}

int mgpu_gemv_chain_links(const mgpu_gemv_chain* c) { return c ? c->n : 0; }

void mgpu_gemv_chain_destroy(mgpu_gemv_chain* c) {
    if (!c) return;
    DeviceGuard g(c->dev->ordinal);
    cudaStreamSynchronize(c->dev->stream);
    free_chain(c);
}

mgpu_event* mgpu_dispatch_patch_embed(const mgpu_device* cd, mgpu_program, mgpu_buf* image, mgpu_buf* proj_weight,
                                      mgpu_buf* proj_bias, mgpu_buf* patches, int C, int H, int W, int ph, int pw,
                                      int embed_dim) {
    API_ENTRY();
    REQUIRE(cd && image && proj_weight && patches, "dispatch_patch_embed: null argument");
    REQUIRE(C > 0 && ph > 0 && pw > 0 && H >= ph && W >= pw && embed_dim > 0, "dispatch_patch_embed: bad shape");
    REQUIRE(image->type == MGPU_F16 || image->type == MGPU_BF16, "dispatch_patch_embed: image must be fp16/bf16");
    REQUIRE(image->bytes >= (size_t)C * H * W * 2, "dispatch_patch_embed: image smaller than C*H*W");
    mgpu_device* d = const_cast<mgpu_device*>(cd);
    const int P = (H / ph) * (W / pw);
    const int pd = C * ph * pw;
    const int kpad = (pd + 7) / 8 * 8;
    const size_t ws = (size_t)P * kpad * 2;
    const size_t off = kScratchOffset;
    DeviceGuard g(d->ordinal);
    // Reserve room for a staged copy of proj_weight as well, so that the GEMM below never
    // has to grow (and reallocate) the arena that already holds the patches.
    const size_t b_stage = (size_t)pd * ((embed_dim + 7) / 8 * 8) * 2 + (size_t)embed_dim * ((pd + 7) / 8 * 8) * 2;
    if (!ensure_workspace(d, ((off + ws + 255) & ~(size_t)255) + b_stage)) return nullptr;
    mgpu_buf A;
    A.dev = d;
    A.ptr = (char*)d->workspace + off;
    A.bytes = ws;
    A.owned = false;
    A.type = image->type;
    A.layout = MGPU_LAYOUT_KN;
    A.rows = P;
    A.cols = pd;
    A.ld = kpad;
    mgpu_event* ev = event_begin(d);
    cudaError_t e = mgpu_k::im2col(ctx_of(d), image->type, image->ptr, A.ptr, C, H, W, ph, pw, kpad);
    if (!cuda_ok(e, "dispatch_patch_embed(im2col)")) {
        if (ev) d->event_pool.push_back(ev);
        return nullptr;
    }
    if (!gemm_checked(d, &A, proj_weight, patches, P, embed_dim, pd, proj_bias, "dispatch_patch_embed",
                      (off + ws + 255) & ~(size_t)255)) {
        if (ev) d->event_pool.push_back(ev);
        return nullptr;
    }
    return event_end(d, ev);
}

mgpu_event* mgpu_dispatch_vision_proj(const mgpu_device* d, mgpu_program, mgpu_buf* tokens, mgpu_buf* proj_weight,
                                      mgpu_buf* proj_bias, mgpu_buf* output, int num_patches, int vision_dim,
                                      int llm_dim) {
    API_ENTRY();
    return run_gemm(d, tokens, proj_weight, output, num_patches, llm_dim, vision_dim, proj_bias, "dispatch_vision_proj");
}

mgpu_event* mgpu_dequant(const mgpu_device* cd, mgpu_buf* W, mgpu_buf* out, int64_t n, int type) {
    API_ENTRY();
    REQUIRE(cd && W && out && is_quant_type(type) && n > 0 && n % 32 == 0, "mgpu_dequant: bad arguments");
    REQUIRE(is_float_type(out->type), "mgpu_dequant: out must be f32/f16/bf16");
    REQUIRE(W->bytes >= (size_t)(n / 32) * (type == MGPU_Q4_0 ? 18 : 34), "mgpu_dequant: W too small");
    REQUIRE(out->bytes >= (size_t)n * elem_size(out->type), "mgpu_dequant: out too small");
    mgpu_device* d = const_cast<mgpu_device*>(cd);
    DeviceGuard g(d->ordinal);
    mgpu_event* ev = event_begin(d);
    if (!cuda_ok(mgpu_k::dequant(ctx_of(d), type, (const uint8_t*)W->ptr, out->type, out->ptr, n), "mgpu_dequant")) {
        if (ev) d->event_pool.push_back(ev);
        return nullptr;
    }
    return event_end(d, ev);
}

// ------------------------------------------------------------------ argmax -----------
// Greedy decode over the lm_head's logits (moondream2.cpp:551-591 reads them back and scans on
// the host): one CTA on the device; out receives {int32 index, fp32 value}.
mgpu_event* mgpu_argmax(const mgpu_device* cd, mgpu_buf* logits, int n, mgpu_buf* out) {
    API_ENTRY();
    REQUIRE(cd && logits && out && n > 0, "mgpu_argmax: bad arguments");
    REQUIRE(is_float_type(logits->type), "mgpu_argmax: logits must be f32/f16/bf16");
    REQUIRE(logits->bytes >= (size_t)n * elem_size(logits->type), "mgpu_argmax: logits too small");
    REQUIRE(out->bytes >= 8, "mgpu_argmax: out needs 8 bytes");
    mgpu_device* d = const_cast<mgpu_device*>(cd);
    DeviceGuard g(d->ordinal);
    mgpu_event* ev = event_begin(d);
    if (!cuda_ok(mgpu_k::argmax(ctx_of(d), logits->type, logits->ptr, n, (int*)out->ptr), "mgpu_argmax")) {
        if (ev) d->event_pool.push_back(ev);
        return nullptr;
    }
    return event_end(d, ev);
}

mgpu_event* mgpu_argmax_rows(const mgpu_device* cd, mgpu_buf* logits, int rows, int n, int64_t ld, mgpu_buf* out) {
    API_ENTRY();
    REQUIRE(cd && logits && out && rows > 0 && n > 0 && ld >= n, "mgpu_argmax_rows: bad arguments");
    REQUIRE(is_float_type(logits->type), "mgpu_argmax_rows: logits must be f32/f16/bf16");
    REQUIRE(logits->bytes >= ((size_t)(rows - 1) * ld + n) * elem_size(logits->type),
            "mgpu_argmax_rows: logits too small");
    REQUIRE(out->bytes >= (size_t)rows * 8, "mgpu_argmax_rows: out needs 8 bytes per row");
    mgpu_device* d = const_cast<mgpu_device*>(cd);
    DeviceGuard g(d->ordinal);
    mgpu_event* ev = event_begin(d);
    if (!cuda_ok(mgpu_k::argmax_rows(ctx_of(d), logits->type, logits->ptr, rows, n, ld, (int*)out->ptr),
                 "mgpu_argmax_rows")) {
        if (ev) d->event_pool.push_back(ev);
        return nullptr;
    }
    return event_end(d, ev);
}

mgpu_event* mgpu_argmax_combine(const mgpu_device* cd, mgpu_buf* pairs, int n_ranks, int n_total, mgpu_buf* out) {
    API_ENTRY();
    REQUIRE(cd && pairs && out && n_ranks > 0 && n_total >= n_ranks, "mgpu_argmax_combine: bad arguments");
    REQUIRE(pairs->bytes >= (size_t)n_ranks * 8, "mgpu_argmax_combine: pairs holds fewer than %d pairs", n_ranks);
    REQUIRE(out->bytes >= 8, "mgpu_argmax_combine: out needs 8 bytes");
    mgpu_device* d = const_cast<mgpu_device*>(cd);
    DeviceGuard g(d->ordinal);
    mgpu_event* ev = event_begin(d);
    if (!cuda_ok(mgpu_k::argmax_combine(ctx_of(d), (const int*)pairs->ptr, n_ranks, n_total, (int*)out->ptr),
                 "mgpu_argmax_combine")) {
        if (ev) d->event_pool.push_back(ev);
        return nullptr;
    }
    return event_end(d, ev);
}

// The reference's argmax_logits(device, logits, vocab_size): the index, or -1 on error.  Waits
// for the device stream; the result goes through bytes 64..71 of the device's status block.
int mgpu_argmax_logits(const mgpu_device* cd, mgpu_buf* logits, int vocab_size) {
    API_ENTRY();
    if (!cd || !logits || vocab_size <= 0 || !is_float_type(logits->type) ||
        logits->bytes < (size_t)vocab_size * elem_size(logits->type)) {
        set_error(MGPU_ERR_INVALID_ARG, "mgpu_argmax_logits: bad arguments");
        return -1;
    }
    mgpu_device* d = const_cast<mgpu_device*>(cd);
    DeviceGuard g(d->ordinal);
    int* slot = d->d_status + 16;
    int host[2] = {-1, 0};
    if (!cuda_ok(mgpu_k::argmax(ctx_of(d), logits->type, logits->ptr, vocab_size, slot), "mgpu_argmax_logits") ||
        !cuda_ok(cudaMemcpyAsync(host, slot, sizeof(host), cudaMemcpyDeviceToHost, d->stream), "read argmax") ||
        !cuda_ok(cudaStreamSynchronize(d->stream), "cudaStreamSynchronize") || !check_status(d))
        return -1;
    return host[0];
}

// ------------------------------------------------------------------ events -----------
int mgpu_wait_event(mgpu_event* ev) {
    if (!ev) return MGPU_OK;
    DeviceGuard g(ev->dev->ordinal);
    if (!cuda_ok(cudaEventSynchronize(ev->end), "cudaEventSynchronize")) return t_err;
    if (!check_status(ev->dev)) return t_err;
    return MGPU_OK;
}

void mgpu_release_event(mgpu_event* ev) {
    if (ev) ev->dev->event_pool.push_back(ev);
}

double mgpu_profile_end(mgpu_event* ev) {
    if (!ev || !ev->timed) return 0.0;
    DeviceGuard g(ev->dev->ordinal);
    float ms = 0.0f;
    if (!cuda_ok(cudaEventSynchronize(ev->end), "cudaEventSynchronize")) return 0.0;
    if (!cuda_ok(cudaEventElapsedTime(&ms, ev->start, ev->end), "cudaEventElapsedTime")) return 0.0;
    return (double)ms;
}

float mgpu_event_elapsed_ms(mgpu_event* a, mgpu_event* b) {
    if (!a || !b) return 0.0f;
    DeviceGuard g(a->dev->ordinal);
    float ms = 0.0f;
    cudaEventSynchronize(b->end);
    if (!cuda_ok(cudaEventElapsedTime(&ms, a->end, b->end), "cudaEventElapsedTime")) return 0.0f;
    return ms;
}

mgpu_event* mgpu_record_event(mgpu_device* d) {
    API_ENTRY();
    REQUIRE(d, "mgpu_record_event: null device");
    DeviceGuard g(d->ordinal);
    mgpu_event* ev = nullptr;
    if (!d->event_pool.empty()) {
        ev = d->event_pool.back();
        d->event_pool.pop_back();
    } else {
        ev = new mgpu_event();
        ev->dev = d;
        cudaEventCreate(&ev->start);
        cudaEventCreate(&ev->end);
    }
    ev->timed = false;
    const unsigned flags = d->capturing ? cudaEventRecordExternal : cudaEventRecordDefault;
    if (!cuda_ok(cudaEventRecordWithFlags(ev->end, d->stream, flags), "cudaEventRecordWithFlags")) {
        d->event_pool.push_back(ev);
        return nullptr;
    }
    return ev;
}

// ------------------------------------------------------------------ graphs -----------
int mgpu_capture_begin(mgpu_device* d) {
    if (!d || d->capturing) {
        set_error(MGPU_ERR_INVALID_ARG, "mgpu_capture_begin: null device or capture already open");
        return MGPU_ERR_INVALID_ARG;
    }
    DeviceGuard g(d->ordinal);
    if (!cuda_ok(cudaStreamBeginCapture(d->stream, cudaStreamCaptureModeThreadLocal), "cudaStreamBeginCapture"))
        return t_err;
    d->capturing = true;
    d->saved_event_mode = d->event_mode;
    d->event_mode = 0;
    return MGPU_OK;
}

mgpu_graph* mgpu_capture_end(mgpu_device* d) {
    API_ENTRY();
    REQUIRE(d && d->capturing, "mgpu_capture_end: no capture open");
    DeviceGuard g(d->ordinal);
    d->capturing = false;
    d->event_mode = d->saved_event_mode;
    cudaGraph_t graph = nullptr;
    if (!cuda_ok(cudaStreamEndCapture(d->stream, &graph), "cudaStreamEndCapture")) return nullptr;
    cudaGraphExec_t exec = nullptr;
    if (!cuda_ok(cudaGraphInstantiate(&exec, graph, 0), "cudaGraphInstantiate")) {
        cudaGraphDestroy(graph);
        return nullptr;
    }
    mgpu_graph* gr = new mgpu_graph();
    gr->dev = d;
    gr->graph = graph;
    gr->exec = exec;
    return gr;
}

int mgpu_graph_launch(mgpu_graph* gr) {
    if (!gr) {
        set_error(MGPU_ERR_INVALID_ARG, "mgpu_graph_launch: null graph");
        return MGPU_ERR_INVALID_ARG;
    }
    DeviceGuard g(gr->dev->ordinal);
    if (!cuda_ok(cudaGraphLaunch(gr->exec, gr->dev->stream), "cudaGraphLaunch")) return t_err;
    return MGPU_OK;
}

void mgpu_graph_release(mgpu_graph* gr) {
    if (!gr) return;
    DeviceGuard g(gr->dev->ordinal);
    cudaGraphExecDestroy(gr->exec);
    cudaGraphDestroy(gr->graph);
    delete gr;
}

int mgpu_selftest_bounded_wait(mgpu_device* d, uint64_t limit_ns) {
    if (!d) {
        set_error(MGPU_ERR_INVALID_ARG, "mgpu_selftest_bounded_wait: null device");
        return MGPU_ERR_INVALID_ARG;
    }
    DeviceGuard g(d->ordinal);
    if (!cuda_ok(mgpu_k::selftest_bounded_wait(ctx_of(d), limit_ns), "selftest_bounded_wait")) return t_err;
    return MGPU_OK;
}

// ------------------------------------------------------------------ ggml table -------
size_t mgpu_ggml_type_size(int t) {
    switch (t) {
        case MGPU_F32: return 4;
        case MGPU_F16: return 2;
        case MGPU_BF16: return 2;
        case MGPU_Q4_0: return 18;
        case MGPU_Q8_0: return 34;
        default: return 0;
    }
}
int mgpu_ggml_type_block_size(int t) {
    switch (t) {
        case MGPU_F32:
        case MGPU_F16:
        case MGPU_BF16: return 1;
        case MGPU_Q4_0:
        case MGPU_Q8_0: return 32;
        default: return 0;
    }
}

// ------------------------------------------------------------------ synthetic data ---
int mgpu_fill_uniform(const mgpu_device* cd, mgpu_buf* out, int64_t n, uint64_t seed, float lo, float hi) {
    if (!cd || !out || !is_float_type(out->type) || out->bytes < (size_t)n * elem_size(out->type)) {
        set_error(MGPU_ERR_INVALID_ARG, "mgpu_fill_uniform: bad arguments");
        return MGPU_ERR_INVALID_ARG;
    }
    DeviceGuard g(cd->ordinal);
    if (!cuda_ok(mgpu_k::fill_uniform(ctx_of(cd), out->type, out->ptr, n, seed, lo, hi), "fill_uniform")) return t_err;
    return MGPU_OK;
}

int mgpu_fill_normal(const mgpu_device* cd, mgpu_buf* out, int64_t n, uint64_t seed, float sigma) {
    if (!cd || !out || !is_float_type(out->type) || out->bytes < (size_t)n * elem_size(out->type)) {
        set_error(MGPU_ERR_INVALID_ARG, "mgpu_fill_normal: bad arguments");
        return MGPU_ERR_INVALID_ARG;
    }
    DeviceGuard g(cd->ordinal);
    if (!cuda_ok(mgpu_k::fill_normal(ctx_of(cd), out->type, out->ptr, n, seed, sigma), "fill_normal")) return t_err;
    return MGPU_OK;
}

int mgpu_quantize(const mgpu_device* cd, mgpu_buf* src, mgpu_buf* dst, int64_t n, int type) {
    if (!cd || !src || !dst || !is_quant_type(type) || n % 32 != 0 || src->type != MGPU_F32 ||
        src->bytes < (size_t)n * 4 || dst->bytes < (size_t)(n / 32) * (type == MGPU_Q4_0 ? 18 : 34)) {
        set_error(MGPU_ERR_INVALID_ARG, "mgpu_quantize: bad arguments");
        return MGPU_ERR_INVALID_ARG;
    }
    DeviceGuard g(cd->ordinal);
    if (!cuda_ok(mgpu_k::quantize(ctx_of(cd), type, (const float*)src->ptr, (uint8_t*)dst->ptr, n), "quantize"))
        return t_err;
    return MGPU_OK;
}

int mgpu_convert(const mgpu_device* cd, mgpu_buf* src, mgpu_buf* dst, int64_t n) {
    if (!cd || !src || !dst || !is_float_type(src->type) || !is_float_type(dst->type) ||
        src->bytes < (size_t)n * elem_size(src->type) || dst->bytes < (size_t)n * elem_size(dst->type)) {
        set_error(MGPU_ERR_INVALID_ARG, "mgpu_convert: bad arguments");
        return MGPU_ERR_INVALID_ARG;
    }
    DeviceGuard g(cd->ordinal);
    if (!cuda_ok(mgpu_k::convert(ctx_of(cd), src->type, src->ptr, dst->type, dst->ptr, n), "convert")) return t_err;
    return MGPU_OK;
}

}  // extern "C"

// ------------------------------------------------------------------ peer groups ------
// Exchanges between the GPUs of one node through peer memory (peer.cu).  One allocation per GPU:
// [world slots of slot_bytes, padded to 256][world u64 flags][u64 epoch], zeroed at creation.
struct mgpu_peer_group {
    mgpu_device* dev;
    int rank, world;
    size_t slot_bytes;
    size_t slots_bytes;  // world * slot_bytes, rounded up to 256
    void* base;
    void* peer[mgpu_k::kMaxPeers];
    bool opened[mgpu_k::kMaxPeers];  // mapped through CUDA IPC (unmapped on destroy)
    bool connected;
    uint64_t limit_ns;
    mgpu_buf* slots;  // view of this GPU's slots, owned by the group
};

mgpu_peer_group* mgpu_peer_group_create(mgpu_device* d, int rank, int world, size_t slot_bytes) {
    API_ENTRY();
    REQUIRE(d && world >= 1 && world <= mgpu_k::kMaxPeers && rank >= 0 && rank < world && slot_bytes > 0,
            "mgpu_peer_group_create: bad arguments (world 1..%d)", mgpu_k::kMaxPeers);
    DeviceGuard g(d->ordinal);
    mgpu_peer_group* pg = new mgpu_peer_group();
    pg->dev = d;
    pg->rank = rank;
    pg->world = world;
    pg->slot_bytes = (slot_bytes + 7) / 8 * 8;
    pg->slots_bytes = ((size_t)world * pg->slot_bytes + 255) / 256 * 256;
    pg->limit_ns = 2000000000ull;  // the kernels' bounded-wait limit: 2 s
    const size_t total = pg->slots_bytes + 256;
    if (!cuda_ok(cudaMalloc(&pg->base, total), "cudaMalloc(peer group)")) {
        delete pg;
        return nullptr;
    }
    if (!cuda_ok(cudaMemsetAsync(pg->base, 0, total, d->stream), "cudaMemsetAsync(peer group)") ||
        !cuda_ok(cudaStreamSynchronize(d->stream), "cudaStreamSynchronize")) {
        cudaFree(pg->base);
        delete pg;
        return nullptr;
    }
    pg->slots = new_buf(d, pg->base, (size_t)world * pg->slot_bytes, false);
    return pg;
}

int mgpu_peer_group_handle(const mgpu_peer_group* pg, void* out64) {
    if (!pg || !out64) {
        set_error(MGPU_ERR_INVALID_ARG, "mgpu_peer_group_handle: null argument");
        return MGPU_ERR_INVALID_ARG;
    }
    static_assert(sizeof(cudaIpcMemHandle_t) == 64, "CUDA IPC handles are 64 bytes");
    DeviceGuard g(pg->dev->ordinal);
    cudaIpcMemHandle_t h;
    if (!cuda_ok(cudaIpcGetMemHandle(&h, pg->base), "cudaIpcGetMemHandle")) return t_err;
    memcpy(out64, &h, sizeof(h));
    return MGPU_OK;
}

int mgpu_peer_group_connect(mgpu_peer_group* pg, const void* handles) {
    if (!pg || !handles || pg->connected) {
        set_error(MGPU_ERR_INVALID_ARG, "mgpu_peer_group_connect: null argument or already connected");
        return MGPU_ERR_INVALID_ARG;
    }
    DeviceGuard g(pg->dev->ordinal);
    for (int p = 0; p < pg->world; ++p) {
        if (p == pg->rank) {
            pg->peer[p] = pg->base;
            continue;
        }
        cudaIpcMemHandle_t h;
        memcpy(&h, static_cast<const char*>(handles) + (size_t)p * sizeof(h), sizeof(h));
        if (!cuda_ok(cudaIpcOpenMemHandle(&pg->peer[p], h, cudaIpcMemLazyEnablePeerAccess),
                     "cudaIpcOpenMemHandle")) {
            for (int q = 0; q < p; ++q)
                if (pg->opened[q]) cudaIpcCloseMemHandle(pg->peer[q]);
            memset(pg->opened, 0, sizeof(pg->opened));
            return t_err;
        }
        pg->opened[p] = true;
    }
    pg->connected = true;
    return MGPU_OK;
}

int mgpu_peer_group_connect_ptrs(mgpu_peer_group* pg, void* const* peer_slots) {
    if (!pg || !peer_slots || pg->connected) {
        set_error(MGPU_ERR_INVALID_ARG, "mgpu_peer_group_connect_ptrs: null argument or already connected");
        return MGPU_ERR_INVALID_ARG;
    }
    for (int p = 0; p < pg->world; ++p) {
        pg->peer[p] = p == pg->rank ? pg->base : peer_slots[p];
        if (!pg->peer[p]) {
            set_error(MGPU_ERR_INVALID_ARG, "mgpu_peer_group_connect_ptrs: no address for rank %d", p);
            return MGPU_ERR_INVALID_ARG;
        }
    }
    pg->connected = true;
    return MGPU_OK;
}

void* mgpu_peer_group_local_ptr(const mgpu_peer_group* pg) { return pg ? pg->base : nullptr; }

mgpu_buf* mgpu_peer_group_slots(mgpu_peer_group* pg) { return pg ? pg->slots : nullptr; }

int mgpu_peer_group_set_wait_limit(mgpu_peer_group* pg, uint64_t limit_ns) {
    if (!pg || limit_ns == 0) {
        set_error(MGPU_ERR_INVALID_ARG, "mgpu_peer_group_set_wait_limit: bad arguments");
        return MGPU_ERR_INVALID_ARG;
    }
    pg->limit_ns = limit_ns;
    return MGPU_OK;
}

static mgpu_event* peer_exchange(mgpu_peer_group* pg, const mgpu_buf* src, size_t bytes, size_t stride,
                                 const char* what) {
    API_ENTRY();
    REQUIRE(pg && src && pg->connected, "%s: group not connected or null source", what);
    REQUIRE(bytes > 0 && bytes % 8 == 0 && bytes <= pg->slot_bytes, "%s: %zu bytes (a multiple of 8, at most %zu)",
            what, bytes, pg->slot_bytes);
    REQUIRE((reinterpret_cast<uintptr_t>(src->ptr) & 15) == 0, "%s: source not 16-byte aligned", what);
    REQUIRE(src->bytes >= (stride ? (size_t)pg->world * stride : bytes), "%s: source too small", what);
    mgpu_device* d = pg->dev;
    DeviceGuard g(d->ordinal);
    mgpu_k::PeerExchangeArgs a = {};
    a.src = static_cast<const uint8_t*>(src->ptr);
    a.src_stride = stride;
    a.bytes = bytes;
    a.slot_bytes = pg->slot_bytes;
    for (int p = 0; p < pg->world; ++p) {
        a.dst[p] = static_cast<uint8_t*>(pg->peer[p]);
        a.dst_flag[p] = reinterpret_cast<unsigned long long*>(static_cast<char*>(pg->peer[p]) + pg->slots_bytes);
    }
    a.my_flags = reinterpret_cast<unsigned long long*>(static_cast<char*>(pg->base) + pg->slots_bytes);
    a.epoch = a.my_flags + pg->world;
    a.rank = pg->rank;
    a.world = pg->world;
    a.limit_ns = pg->limit_ns;
    a.status = d->d_status;
    mgpu_event* ev = event_begin(d);
    if (!cuda_ok(mgpu_k::peer_exchange(ctx_of(d), a), what)) {
        if (ev) d->event_pool.push_back(ev);
        return nullptr;
    }
    return event_end(d, ev);
}

mgpu_event* mgpu_peer_allgather(mgpu_peer_group* pg, const mgpu_buf* src, size_t bytes) {
    return peer_exchange(pg, src, bytes, 0, "mgpu_peer_allgather");
}

mgpu_event* mgpu_peer_alltoall(mgpu_peer_group* pg, const mgpu_buf* src, size_t bytes_per_peer) {
    return peer_exchange(pg, src, bytes_per_peer, bytes_per_peer, "mgpu_peer_alltoall");
}

void mgpu_peer_group_destroy(mgpu_peer_group* pg) {
    if (!pg) return;
    DeviceGuard g(pg->dev->ordinal);
    cudaStreamSynchronize(pg->dev->stream);
    for (int p = 0; p < pg->world; ++p)
        if (pg->opened[p]) cudaIpcCloseMemHandle(pg->peer[p]);
    cudaFree(pg->base);
    delete pg->slots;
    delete pg;
}
