// engine_cuda.cpp - MVLM's engine API for the matmul path, implemented on libmgpu (CUDA).
//
// Compiled against the reference's own headers (src/engine/device.h, memory.h, compute.h, with
// include/cl_compat first on the include path in place of the OpenCL SDK), this file takes the
// place of src/engine/device.cpp, memory.cpp and the matmul half of compute.cpp: every handle is
// an mgpu C ABI handle behind its OpenCL type (cl_mem = mgpu_buf*, cl_event = mgpu_event*,
// DeviceInfo::context = DeviceInfo::queue = mgpu_device*), so the reference's model code
// (moondream2_forward, moondream2_encode_vision) calls the B200 kernels unchanged.
//
// Defined here: init_device / destroy_device / print_device_info / has_extension and the
// program builders (device.h); create_weight_image / create_buffer / create_onchip_buffer and
// the buffer pool (memory.h); dispatch_gemm_naive / _tiled / _image, dispatch_gemv,
// dispatch_rms_norm, dispatch_patch_embed, dispatch_vision_proj (compute.h); and the OpenCL
// calls the model code makes on those handles (cl_compat/CL/cl.h).  The other compute.h
// entries (attention, RoPE, activations, embedding, image preprocessing, the SigLIP layer
// placeholders) are not on the matmul path and are not defined: an engine links its own.
#include <cstdio>
#include <cstring>

#include "../../include/mgpu_cuda.h"
#include "compute.h"
#include "device.h"
#include "memory.h"

namespace {

inline mgpu_device* dev_of(const mgpu::DeviceInfo* d) { return reinterpret_cast<mgpu_device*>(d->context); }
inline mgpu_buf* buf_of(cl_mem m) { return reinterpret_cast<mgpu_buf*>(m); }
inline cl_mem mem_of(mgpu_buf* b) { return reinterpret_cast<cl_mem>(b); }
inline cl_event event_of(mgpu_event* e) { return reinterpret_cast<cl_event>(e); }
inline mgpu_event* ev_of(cl_event e) { return reinterpret_cast<mgpu_event*>(e); }
inline mgpu_device* queue_dev(cl_command_queue q) { return reinterpret_cast<mgpu_device*>(q); }

// The reference logs failures as "OpenCL error %d at file:line" and returns nullptr
// (compute.cpp:12-17); the same here with the library's message.
cl_event checked(mgpu_event* e, const char* what) {
    if (!e && mgpu_last_error() != MGPU_OK) fprintf(stderr, "%s failed: %s\n", what, mgpu_last_error_string());
    return event_of(e);
}

// A token that stands for a compiled program: the kernels are compiled into libmgpu.
cl_program program_token() {
    static char token;
    return reinterpret_cast<cl_program>(&token);
}

}  // namespace

namespace mgpu {

// ------------------------------------------------------------------ device.h --------
bool init_device(DeviceInfo* info) {
    if (!info) return false;
    memset(info, 0, sizeof(*info));
    mgpu_device* d = mgpu_init_device(0);
    if (!d) {
        fprintf(stderr, "init_device: %s\n", mgpu_last_error_string());
        return false;
    }
    info->context = reinterpret_cast<cl_context>(d);
    info->queue = reinterpret_cast<cl_command_queue>(d);
    snprintf(info->device_name, sizeof(info->device_name), "CUDA device 0 (sm_100a)");
    snprintf(info->vendor, sizeof(info->vendor), "NVIDIA");
    info->compute_units = (cl_uint)mgpu_device_sm_count(d);
    info->has_fp16 = true;
    info->has_subgroups = true;
    info->has_image = true;
    info->image_support = CL_TRUE;
    return true;
}

void print_device_info(const DeviceInfo* info) {
    if (info) printf("Device: %s, %u SMs\n", info->device_name, info->compute_units);
}

bool has_extension(cl_device_id, const char*) { return false; }

cl_program build_program_from_source(const DeviceInfo*, const char*, size_t, const char*) { return program_token(); }
cl_program build_program_from_file(const DeviceInfo*, const char*, const char*) { return program_token(); }

void destroy_device(DeviceInfo* info) {
    if (info && info->context) mgpu_release_device(dev_of(info));
    if (info) info->context = nullptr, info->queue = nullptr;
}

// ------------------------------------------------------------------ memory.h --------
cl_mem create_weight_image(const DeviceInfo* info, int rows, int cols, const cl_half* data) {
    return mem_of(mgpu_create_weight_image(dev_of(info), rows, cols, data));
}

cl_mem create_buffer(const DeviceInfo* info, size_t size_bytes, cl_mem_flags flags, void* host_ptr) {
    return mem_of(mgpu_create_buffer(dev_of(info), size_bytes, (flags & CL_MEM_COPY_HOST_PTR) ? host_ptr : nullptr));
}

cl_mem create_onchip_buffer(const DeviceInfo* info, size_t size_bytes) {
    return create_buffer(info, size_bytes, CL_MEM_READ_WRITE, nullptr);
}

bool init_buffer_pool(BufferPool* pool, const DeviceInfo* info, size_t size_bytes) {
    pool->buffers[0] = create_buffer(info, size_bytes, CL_MEM_READ_WRITE, nullptr);
    pool->buffers[1] = create_buffer(info, size_bytes, CL_MEM_READ_WRITE, nullptr);
    pool->size = size_bytes;
    pool->current = 0;
    return pool->buffers[0] && pool->buffers[1];
}
cl_mem get_current_buffer(BufferPool* pool) { return pool->buffers[pool->current]; }
cl_mem get_next_buffer(BufferPool* pool) { return pool->buffers[1 - pool->current]; }
void swap_buffers(BufferPool* pool) { pool->current = 1 - pool->current; }
void destroy_buffer_pool(BufferPool* pool) {
    for (cl_mem& b : pool->buffers) {
        if (b) mgpu_release_buffer(buf_of(b));
        b = nullptr;
    }
}

// ------------------------------------------------------------------ compute.h -------
cl_event dispatch_gemm_naive(const DeviceInfo* dev, cl_program program, cl_mem A, cl_mem B, cl_mem C, int M, int N,
                             int K) {
    return checked(mgpu_dispatch_gemm_naive(dev_of(dev), program, buf_of(A), buf_of(B), buf_of(C), M, N, K),
                   "dispatch_gemm_naive");
}
cl_event dispatch_gemm_tiled(const DeviceInfo* dev, cl_program program, cl_mem A, cl_mem B, cl_mem C, int M, int N,
                             int K) {
    return checked(mgpu_dispatch_gemm_tiled(dev_of(dev), program, buf_of(A), buf_of(B), buf_of(C), M, N, K),
                   "dispatch_gemm_tiled");
}
cl_event dispatch_gemm_image(const DeviceInfo* dev, cl_program program, cl_mem A, cl_mem B_img, cl_mem C, int M,
                             int N, int K) {
    return checked(mgpu_dispatch_gemm_image(dev_of(dev), program, buf_of(A), buf_of(B_img), buf_of(C), M, N, K),
                   "dispatch_gemm_image");
}
cl_event dispatch_gemv(const DeviceInfo* dev, cl_program program, cl_mem x, cl_mem W_img, cl_mem y, int N, int K) {
    return checked(mgpu_dispatch_gemv(dev_of(dev), program, buf_of(x), buf_of(W_img), buf_of(y), N, K),
                   "dispatch_gemv");
}
cl_event dispatch_rms_norm(const DeviceInfo* dev, cl_program program, cl_mem input, cl_mem output, cl_mem weight,
                           int num_rows, int hidden_size, float eps) {
    return checked(mgpu_dispatch_rms_norm(dev_of(dev), program, buf_of(input), buf_of(output), buf_of(weight),
                                          num_rows, hidden_size, eps),
                   "dispatch_rms_norm");
}
cl_event dispatch_patch_embed(const DeviceInfo* dev, cl_program program, cl_mem image, cl_mem proj_weight,
                              cl_mem proj_bias, cl_mem patches, int C, int H, int W, int patch_h, int patch_w,
                              int embed_dim) {
    return checked(mgpu_dispatch_patch_embed(dev_of(dev), program, buf_of(image), buf_of(proj_weight),
                                             buf_of(proj_bias), buf_of(patches), C, H, W, patch_h, patch_w,
                                             embed_dim),
                   "dispatch_patch_embed");
}
cl_event dispatch_vision_proj(const DeviceInfo* dev, cl_program program, cl_mem visual_tokens, cl_mem proj_weight,
                              cl_mem proj_bias, cl_mem output, int num_patches, int vision_dim, int llm_dim) {
    return checked(mgpu_dispatch_vision_proj(dev_of(dev), program, buf_of(visual_tokens), buf_of(proj_weight),
                                             buf_of(proj_bias), buf_of(output), num_patches, vision_dim, llm_dim),
                   "dispatch_vision_proj");
}

}  // namespace mgpu

// ------------------------------------------------------------------ CL/cl.h ---------
extern "C" {

cl_mem clCreateBuffer(cl_context context, cl_mem_flags flags, size_t size, void* host_ptr, cl_int* err) {
    mgpu_buf* b = mgpu_create_buffer(reinterpret_cast<mgpu_device*>(context), size,
                                     (flags & CL_MEM_COPY_HOST_PTR) ? host_ptr : nullptr);
    if (err) *err = b ? CL_SUCCESS : CL_OUT_OF_RESOURCES;
    return mem_of(b);
}

cl_mem clCreateSubBuffer(cl_mem buffer, cl_mem_flags, cl_buffer_create_type type, const void* info, cl_int* err) {
    const cl_buffer_region* r = static_cast<const cl_buffer_region*>(info);
    mgpu_buf* v = (type == CL_BUFFER_CREATE_TYPE_REGION && r) ? mgpu_buf_view(buf_of(buffer), r->origin, r->size)
                                                             : nullptr;
    if (err) *err = v ? CL_SUCCESS : CL_INVALID_VALUE;
    return mem_of(v);
}

cl_int clEnqueueReadBuffer(cl_command_queue, cl_mem buffer, cl_bool blocking, size_t offset, size_t size, void* ptr,
                           cl_uint, const cl_event*, cl_event* event) {
    if (event) *event = nullptr;
    const int rc = blocking ? mgpu_buf_read(buf_of(buffer), offset, ptr, size)
                            : mgpu_buf_read_async(buf_of(buffer), offset, ptr, size);
    return rc == MGPU_OK ? CL_SUCCESS : CL_INVALID_VALUE;
}

cl_int clEnqueueWriteBuffer(cl_command_queue, cl_mem buffer, cl_bool blocking, size_t offset, size_t size,
                            const void* ptr, cl_uint, const cl_event*, cl_event* event) {
    if (event) *event = nullptr;
    const int rc = blocking ? mgpu_buf_write(buf_of(buffer), offset, ptr, size)
                            : mgpu_buf_write_async(buf_of(buffer), offset, ptr, size);
    return rc == MGPU_OK ? CL_SUCCESS : CL_INVALID_VALUE;
}

cl_int clEnqueueCopyBuffer(cl_command_queue, cl_mem src, cl_mem dst, size_t src_offset, size_t dst_offset,
                           size_t size, cl_uint, const cl_event*, cl_event* event) {
    if (event) *event = nullptr;
    return mgpu_buf_copy_async(buf_of(dst), dst_offset, buf_of(src), src_offset, size) == MGPU_OK
               ? CL_SUCCESS
               : CL_INVALID_VALUE;
}

cl_int clWaitForEvents(cl_uint num, const cl_event* events) {
    cl_int rc = CL_SUCCESS;
    for (cl_uint i = 0; i < num; ++i)
        if (mgpu_wait_event(ev_of(events[i])) != MGPU_OK) rc = CL_INVALID_VALUE;
    return rc;
}

cl_int clReleaseEvent(cl_event event) {
    mgpu_release_event(ev_of(event));
    return CL_SUCCESS;
}

cl_int clReleaseMemObject(cl_mem mem) {
    mgpu_release_buffer(buf_of(mem));
    return CL_SUCCESS;
}

cl_int clReleaseProgram(cl_program) { return CL_SUCCESS; }

cl_int clFinish(cl_command_queue queue) { return mgpu_finish(queue_dev(queue)) == MGPU_OK ? CL_SUCCESS : CL_INVALID_VALUE; }

}  // extern "C"
