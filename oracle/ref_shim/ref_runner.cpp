// ref_runner.cpp - host NDRange runner for the reference's gemm.cl kernels compiled as C++
// under clshim.hpp.  TEST INFRASTRUCTURE ONLY (oracle/_ref/).
//
// The launch geometry of each entry point is the reference dispatcher's:
//   ref_gemm_naive  <- dispatch_gemm_naive  src/engine/compute.cpp:47-48 (global {M^16, N^16}, local {16,16})
//   ref_gemm_tiled  <- dispatch_gemm_tiled  compute.cpp:76-80           (global {M^8, N^8},  local {8,8})
//   ref_gemm_image  <- dispatch_gemm_image  compute.cpp:109-112         (global {M^16, ceil(N/4)^4}, local {16,4})
//   ref_gemv        <- dispatch_gemv        compute.cpp:140-144         (ceil(N/4) groups x 256)
// Image weights are built the way create_weight_image (src/engine/memory.cpp:28-79) builds
// them: columns zero-padded to a multiple of 4, one RGBA-half texel per 4 columns.
#include <ucontext.h>

#include <cstdint>
#include <cstdlib>
#include <cstring>
#include <vector>

#include "clshim.hpp"

namespace clshim {
thread_local const WorkItem* g_current = nullptr;

namespace {
struct Fiber {
    ucontext_t ctx;
    WorkItem wi;
    bool done;
    std::vector<char> stack;
};
thread_local ucontext_t* g_sched = nullptr;
thread_local Fiber* g_fiber = nullptr;

using KernelThunk = void (*)(void*);
struct FiberStart {
    KernelThunk fn;
    void* args;
    Fiber* self;
};

void fiber_entry(unsigned lo, unsigned hi) {
    FiberStart* fs = (FiberStart*)(((uintptr_t)hi << 32) | (uintptr_t)lo);
    fs->fn(fs->args);
    fs->self->done = true;
    swapcontext(&fs->self->ctx, g_sched);
}
}  // namespace

void barrier(int) {
    Fiber* f = g_fiber;
    if (f == nullptr) return;  // work-item run without fibers: barrier-free kernel
    swapcontext(&f->ctx, g_sched);
}

// Run one NDRange.  Barrier kernels run every work-item of a group as a fiber and
// round-robin them between barriers; barrier-free kernels run work-items one by one.
static void run_ndrange(int dims, const size_t* global, const size_t* local, KernelThunk fn,
                        void* args, bool has_barrier) {
    size_t groups[3] = {1, 1, 1}, lsz[3] = {1, 1, 1};
    for (int d = 0; d < dims; ++d) {
        lsz[d] = local[d];
        groups[d] = global[d] / local[d];
    }
    const size_t lcount = lsz[0] * lsz[1] * lsz[2];
    std::vector<Fiber> fibers(has_barrier ? lcount : 0);
    std::vector<FiberStart> starts(has_barrier ? lcount : 0);
    for (size_t g2 = 0; g2 < groups[2]; ++g2)
        for (size_t g1 = 0; g1 < groups[1]; ++g1)
            for (size_t g0 = 0; g0 < groups[0]; ++g0) {
                size_t idx = 0;
                std::vector<WorkItem> items(lcount);
                for (size_t l2 = 0; l2 < lsz[2]; ++l2)
                    for (size_t l1 = 0; l1 < lsz[1]; ++l1)
                        for (size_t l0 = 0; l0 < lsz[0]; ++l0, ++idx) {
                            WorkItem& w = items[idx];
                            w.lid[0] = l0; w.lid[1] = l1; w.lid[2] = l2;
                            w.grp[0] = g0; w.grp[1] = g1; w.grp[2] = g2;
                            w.gid[0] = g0 * lsz[0] + l0;
                            w.gid[1] = g1 * lsz[1] + l1;
                            w.gid[2] = g2 * lsz[2] + l2;
                        }
                if (!has_barrier) {
                    for (size_t i = 0; i < lcount; ++i) {
                        g_current = &items[i];
                        fn(args);
                    }
                    continue;
                }
                ucontext_t sched;
                g_sched = &sched;
                for (size_t i = 0; i < lcount; ++i) {
                    Fiber& f = fibers[i];
                    f.wi = items[i];
                    f.done = false;
                    f.stack.resize(1 << 16);
                    getcontext(&f.ctx);
                    f.ctx.uc_stack.ss_sp = f.stack.data();
                    f.ctx.uc_stack.ss_size = f.stack.size();
                    f.ctx.uc_link = nullptr;
                    starts[i] = FiberStart{fn, args, &f};
                    uintptr_t p = (uintptr_t)&starts[i];
                    makecontext(&f.ctx, (void (*)())fiber_entry, 2, (unsigned)(p & 0xffffffffu),
                                (unsigned)(p >> 32));
                }
                bool all_done = false;
                while (!all_done) {
                    all_done = true;
                    for (size_t i = 0; i < lcount; ++i) {
                        Fiber& f = fibers[i];
                        if (f.done) continue;
                        g_current = &f.wi;
                        g_fiber = &f;
                        swapcontext(&sched, &f.ctx);
                        g_fiber = nullptr;
                        if (!f.done) all_done = false;
                    }
                }
                g_sched = nullptr;
            }
    g_current = nullptr;
}
}  // namespace clshim

// Kernel symbols from the reference's gemm.cl (compiled separately under the shim).
extern "C" {
void gemm_naive(const clshim::half* A, const clshim::half* B, clshim::half* C, const int M,
                const int N, const int K);
void gemm_tiled(const clshim::half* A, const clshim::half* B, clshim::half* C, const int M,
                const int N, const int K);
void gemm_image(const clshim::half* A, const clshim::image2d* B_img, clshim::half* C, const int M,
                const int N, const int K);
void gemv(const clshim::half* x, const clshim::image2d* W_img, clshim::half* y, const int N,
          const int K);
}

namespace {
struct GemmArgs {
    const clshim::half* A;
    const void* B;
    clshim::half* C;
    int M, N, K;
};
size_t round_up(size_t v, size_t m) { return (v + m - 1) / m * m; }

std::vector<clshim::half> make_image(const uint16_t* B, int rows, int cols, clshim::image2d* img) {
    int padded = (cols + 3) / 4 * 4;
    std::vector<clshim::half> tex((size_t)rows * padded);
    std::memset(tex.data(), 0, tex.size() * sizeof(clshim::half));
    for (int r = 0; r < rows; ++r)
        std::memcpy(tex.data() + (size_t)r * padded, B + (size_t)r * cols, (size_t)cols * 2);
    img->width = padded / 4;
    img->height = rows;
    img->texels = tex.data();
    return tex;
}
}  // namespace

extern "C" {

void ref_gemm_naive(const uint16_t* A, const uint16_t* B, uint16_t* C, int M, int N, int K) {
    GemmArgs a{(const clshim::half*)A, B, (clshim::half*)C, M, N, K};
    size_t global[2] = {round_up(M, 16), round_up(N, 16)}, local[2] = {16, 16};
    clshim::run_ndrange(2, global, local, [](void* p) {
        GemmArgs* g = (GemmArgs*)p;
        gemm_naive(g->A, (const clshim::half*)g->B, g->C, g->M, g->N, g->K);
    }, &a, false);
}

void ref_gemm_tiled(const uint16_t* A, const uint16_t* B, uint16_t* C, int M, int N, int K) {
    GemmArgs a{(const clshim::half*)A, B, (clshim::half*)C, M, N, K};
    size_t global[2] = {round_up(M, 8), round_up(N, 8)}, local[2] = {8, 8};
    clshim::run_ndrange(2, global, local, [](void* p) {
        GemmArgs* g = (GemmArgs*)p;
        gemm_tiled(g->A, (const clshim::half*)g->B, g->C, g->M, g->N, g->K);
    }, &a, true);
}

void ref_gemm_image(const uint16_t* A, const uint16_t* B, uint16_t* C, int M, int N, int K) {
    clshim::image2d img;
    std::vector<clshim::half> tex = make_image(B, K, N, &img);
    GemmArgs a{(const clshim::half*)A, &img, (clshim::half*)C, M, N, K};
    size_t n4 = ((size_t)N + 3) / 4;
    size_t global[2] = {round_up(M, 16), round_up(n4, 4)}, local[2] = {16, 4};
    clshim::run_ndrange(2, global, local, [](void* p) {
        GemmArgs* g = (GemmArgs*)p;
        gemm_image(g->A, (const clshim::image2d*)g->B, g->C, g->M, g->N, g->K);
    }, &a, false);
}

void ref_gemv(const uint16_t* x, const uint16_t* W, uint16_t* y, int N, int K) {
    clshim::image2d img;
    std::vector<clshim::half> tex = make_image(W, K, N, &img);
    GemmArgs a{(const clshim::half*)x, &img, (clshim::half*)y, 1, N, K};
    size_t global[1] = {((size_t)N + 3) / 4 * 256}, local[1] = {256};
    clshim::run_ndrange(1, global, local, [](void* p) {
        GemmArgs* g = (GemmArgs*)p;
        gemv(g->A, (const clshim::image2d*)g->B, g->C, g->N, g->K);
    }, &a, true);
}

}  // extern "C"

clshim::half operator"" h(long double v) { return clshim::half((float)v); }
