// mgpu_compute.hpp - C++ mirror of MVLM's engine interface over the C ABI in mgpu_cuda.h.
//
// Same namespace, function names, argument order and return conventions as the reference's
// src/engine/compute.h:16-33, :101-105, :128-131, memory.h:16-19, device.h:58 and
// profiler.h:16, so that its dispatch call sites (the GEMV / GEMM calls of moondream2_forward,
// src/models/moondream2.cpp:370-540, and of moondream2_encode_vision, :791-918) read the same:
//
//   cl_event ev = dispatch_gemv(device, model->gemm_program, x, lw->q_proj_weight, y, N, K);
//   if (ev) { clWaitForEvents(1, &ev); clReleaseEvent(ev); }
//
// cl_mem / cl_event / cl_program are aliases of the C ABI handles; the OpenCL helper calls
// those call sites use on them (clWaitForEvents, clReleaseEvent, clReleaseMemObject) are
// provided as inline shims.  Header-only: for code written against this header.  To build the
// reference's own engine headers and model code unchanged, use include/cl_compat/CL/cl.h with
// mvlm_b200/engine/engine_cuda.cpp instead (DeviceInfo keeps its OpenCL fields there).
#pragma once

#include <cstddef>
#include <cstdint>

#include "mgpu_cuda.h"

namespace mgpu {

using cl_mem = mgpu_buf*;
using cl_event = mgpu_event*;
using cl_program = mgpu_program;
using cl_half = uint16_t;
using DeviceInfo = mgpu_device;

// --- device.h:58 ---
inline bool init_device(DeviceInfo** out, int ordinal = 0) {
    *out = mgpu_init_device(ordinal);
    return *out != nullptr;
}

// --- memory.h:16-19 ---
inline cl_mem create_weight_image(const DeviceInfo* info, int rows, int cols, const cl_half* data) {
    return mgpu_create_weight_image(const_cast<DeviceInfo*>(info), rows, cols, data);
}
inline cl_mem create_buffer(const DeviceInfo* info, size_t size_bytes, unsigned long /*flags*/ = 0,
                            void* host_ptr = nullptr) {
    return mgpu_create_buffer(const_cast<DeviceInfo*>(info), size_bytes, host_ptr);
}

// --- compute.h:16-33 ---
inline cl_event dispatch_gemm_naive(const DeviceInfo* dev, cl_program program, cl_mem A, cl_mem B, cl_mem C, int M,
                                    int N, int K) {
    return mgpu_dispatch_gemm_naive(dev, program, A, B, C, M, N, K);
}
inline cl_event dispatch_gemm_tiled(const DeviceInfo* dev, cl_program program, cl_mem A, cl_mem B, cl_mem C, int M,
                                    int N, int K) {
    return mgpu_dispatch_gemm_tiled(dev, program, A, B, C, M, N, K);
}
inline cl_event dispatch_gemm_image(const DeviceInfo* dev, cl_program program, cl_mem A, cl_mem B_img, cl_mem C,
                                    int M, int N, int K) {
    return mgpu_dispatch_gemm_image(dev, program, A, B_img, C, M, N, K);
}
inline cl_event dispatch_gemv(const DeviceInfo* dev, cl_program program, cl_mem x, cl_mem W_img, cl_mem y, int N,
                              int K) {
    return mgpu_dispatch_gemv(dev, program, x, W_img, y, N, K);
}

// --- compute.h:101-105, :128-131 ---
inline cl_event dispatch_patch_embed(const DeviceInfo* dev, cl_program program, cl_mem image, cl_mem proj_weight,
                                     cl_mem proj_bias, cl_mem patches, int C, int H, int W, int patch_h,
                                     int patch_w, int embed_dim) {
    return mgpu_dispatch_patch_embed(dev, program, image, proj_weight, proj_bias, patches, C, H, W, patch_h, patch_w,
                                     embed_dim);
}
inline cl_event dispatch_vision_proj(const DeviceInfo* dev, cl_program program, cl_mem visual_tokens,
                                     cl_mem proj_weight, cl_mem proj_bias, cl_mem output, int num_patches,
                                     int vision_dim, int llm_dim) {
    return mgpu_dispatch_vision_proj(dev, program, visual_tokens, proj_weight, proj_bias, output, num_patches,
                                     vision_dim, llm_dim);
}

// --- profiler.h:16 ---
inline double profile_end(cl_event event) { return mgpu_profile_end(event); }

// moondream2.cpp:551 argmax_logits(device, logits, vocab_size): on the device.
inline int argmax_logits(const DeviceInfo* dev, cl_mem logits, int vocab_size) {
    return mgpu_argmax_logits(dev, logits, vocab_size);
}

}  // namespace mgpu

// OpenCL helpers used by the reference's call sites on these handles.
inline int clWaitForEvents(unsigned num, const mgpu::cl_event* evs) {
    int rc = 0;
    for (unsigned i = 0; i < num; ++i)
        if (int r = mgpu_wait_event(evs[i])) rc = r;
    return rc;
}
inline int clReleaseEvent(mgpu::cl_event ev) {
    mgpu_release_event(ev);
    return 0;
}
inline int clReleaseMemObject(mgpu::cl_mem m) {
    mgpu_release_buffer(m);
    return 0;
}
