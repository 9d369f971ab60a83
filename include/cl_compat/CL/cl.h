/*
 * cl_compat/CL/cl.h - the subset of the OpenCL API that MVLM's engine headers
 * (src/engine/device.h, memory.h, compute.h) and its model code around the matmul path
 * (src/models/moondream2.cpp: buffers, sub-buffers, events, finish, copies, reads) use, with
 * every handle an alias of an mgpu C ABI handle (include/mgpu_cuda.h):
 *   cl_mem -> mgpu_buf*, cl_event -> mgpu_event*, cl_context / cl_command_queue -> mgpu_device*.
 * Put this directory first on the include path in place of the OpenCL SDK and link
 * mvlm_b200/engine/engine_cuda.cpp and libmgpu.so in place of src/engine/{device,memory,compute}.cpp:
 * the reference's headers and the call sites of its matmul path then compile unchanged and run
 * on CUDA.  Types and constant values follow the OpenCL 1.2 headers where a caller could see
 * them; only what those sources use is declared.
 */
#ifndef MGPU_CL_COMPAT_H
#define MGPU_CL_COMPAT_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef int32_t cl_int;
typedef uint32_t cl_uint;
typedef uint64_t cl_ulong;
typedef uint32_t cl_bool;
typedef uint16_t cl_half;
typedef cl_ulong cl_mem_flags;
typedef cl_uint cl_buffer_create_type;

typedef struct _cl_platform_id* cl_platform_id;
typedef struct _cl_device_id* cl_device_id;
typedef struct _cl_context* cl_context;          /* an mgpu_device* */
typedef struct _cl_command_queue* cl_command_queue; /* the same mgpu_device* */
typedef struct _cl_program* cl_program;          /* accepted and ignored */
typedef struct _cl_mem* cl_mem;                  /* an mgpu_buf* */
typedef struct _cl_event* cl_event;              /* an mgpu_event* */

typedef struct _cl_buffer_region {
    size_t origin;
    size_t size;
} cl_buffer_region;

#define CL_SUCCESS 0
#define CL_INVALID_VALUE (-30)
#define CL_OUT_OF_RESOURCES (-5)
#define CL_FALSE 0
#define CL_TRUE 1
#define CL_MEM_READ_WRITE (1 << 0)
#define CL_MEM_WRITE_ONLY (1 << 1)
#define CL_MEM_READ_ONLY (1 << 2)
#define CL_MEM_USE_HOST_PTR (1 << 3)
#define CL_MEM_ALLOC_HOST_PTR (1 << 4)
#define CL_MEM_COPY_HOST_PTR (1 << 5)
#define CL_BUFFER_CREATE_TYPE_REGION 0x1220

cl_mem clCreateBuffer(cl_context context, cl_mem_flags flags, size_t size, void* host_ptr, cl_int* errcode_ret);
cl_mem clCreateSubBuffer(cl_mem buffer, cl_mem_flags flags, cl_buffer_create_type type, const void* info,
                         cl_int* errcode_ret);
cl_int clEnqueueReadBuffer(cl_command_queue queue, cl_mem buffer, cl_bool blocking, size_t offset, size_t size,
                           void* ptr, cl_uint num_events, const cl_event* wait_list, cl_event* event);
cl_int clEnqueueWriteBuffer(cl_command_queue queue, cl_mem buffer, cl_bool blocking, size_t offset, size_t size,
                            const void* ptr, cl_uint num_events, const cl_event* wait_list, cl_event* event);
cl_int clEnqueueCopyBuffer(cl_command_queue queue, cl_mem src, cl_mem dst, size_t src_offset, size_t dst_offset,
                           size_t size, cl_uint num_events, const cl_event* wait_list, cl_event* event);
cl_int clWaitForEvents(cl_uint num_events, const cl_event* event_list);
cl_int clReleaseEvent(cl_event event);
cl_int clReleaseMemObject(cl_mem mem);
cl_int clReleaseProgram(cl_program program);
cl_int clFinish(cl_command_queue queue);

#ifdef __cplusplus
}
#endif

#endif
