// clshim.hpp - lets the reference's OpenCL C kernel source (src/kernels/gemm.cl of
// drxddy/MVLM) compile unmodified as C++ on the host.  TEST INFRASTRUCTURE ONLY.
//
// It is force-included (-include) ahead of the .cl file by oracle/Makefile; the kernel
// bodies are the reference's own.  Work-items run as cooperative fibers (ucontext) so that
// barrier() and __local memory keep their OpenCL meaning: __local arrays become function
// statics shared by the work-group, and barrier() yields to the next work-item of the group.
// The built library (oracle/_ref/) stands in for the CPU OpenCL runtime that the container
// lacks.
#pragma once
#include <cmath>
#include <cstddef>
#include <cstdint>
#include <cstring>

namespace clshim {

// --- binary16 storage type with IEEE round-to-nearest-even conversion ---
struct half {
    uint16_t bits;
    half() = default;
    half(float f) { _Float16 v = (_Float16)f; std::memcpy(&bits, &v, 2); }
    half(double f) : half((float)f) {}
    operator float() const { _Float16 v; std::memcpy(&v, &bits, 2); return (float)v; }
};

struct float4 {
    float v[4];
    float4() = default;
    float4(float s) { v[0] = v[1] = v[2] = v[3] = s; }
    float& operator[](int i) { return v[i]; }
    float operator[](int i) const { return v[i]; }
    float4& operator+=(const float4& o) { for (int i = 0; i < 4; ++i) v[i] += o.v[i]; return *this; }
};
inline float4 operator+(float4 a, const float4& b) { a += b; return a; }

struct half4 { half v[4]; };
struct int2v { int x, y; };

inline float4 fma(const float4& a, const float4& b, const float4& c) {
    float4 r;
    for (int i = 0; i < 4; ++i) r.v[i] = std::fma(a.v[i], b.v[i], c.v[i]);
    return r;
}
inline float fma(float a, float b, float c) { return std::fma(a, b, c); }
inline float4 convert_float4(const half4& h) {
    float4 r;
    for (int i = 0; i < 4; ++i) r.v[i] = (float)h.v[i];
    return r;
}
inline half4 convert_half4(const float4& f) {
    half4 r;
    for (int i = 0; i < 4; ++i) r.v[i] = half(f.v[i]);
    return r;
}
inline int2v make_int2(int x, int y) { return int2v{x, y}; }

// RGBA half image: width texels per row, 4 halves per texel, clamp-to-edge addressing
// (the only sampler gemm.cl uses, gemm.cl:152-155).
struct image2d {
    int width, height;
    const half* texels;
};
inline half4 read_imageh(const image2d* img, int /*sampler*/, int2v c) {
    int x = c.x < 0 ? 0 : (c.x >= img->width ? img->width - 1 : c.x);
    int y = c.y < 0 ? 0 : (c.y >= img->height ? img->height - 1 : c.y);
    half4 r;
    std::memcpy(&r, img->texels + ((size_t)y * img->width + x) * 4, sizeof(r));
    return r;
}

inline float vload_half(size_t off, const half* p) { return (float)p[off]; }
inline void vstore_half(float f, size_t off, half* p) { p[off] = half(f); }
inline void vstore_half4(const float4& f, size_t off, half* p) {
    for (int i = 0; i < 4; ++i) p[off * 4 + i] = half(f.v[i]);
}
inline int mad24(int a, int b, int c) { return a * b + c; }
inline int mul24(int a, int b) { return a * b; }

// Work-item identity of the currently running fiber (set by the runner).
struct WorkItem {
    size_t gid[3], lid[3], grp[3];
};
extern thread_local const WorkItem* g_current;
inline size_t get_global_id(int d) { return g_current->gid[d]; }
inline size_t get_local_id(int d) { return g_current->lid[d]; }
inline size_t get_group_id(int d) { return g_current->grp[d]; }
void barrier(int flags);

}  // namespace clshim

clshim::half operator"" h(long double v);

using clshim::half;
using clshim::float4;
using clshim::half4;
using clshim::fma;
using clshim::convert_float4;
using clshim::convert_half4;
using clshim::read_imageh;
using clshim::vload_half;
using clshim::vstore_half;
using clshim::vstore_half4;
using clshim::mad24;
using clshim::mul24;
using clshim::get_global_id;
using clshim::get_local_id;
using clshim::get_group_id;
using clshim::barrier;
typedef const clshim::image2d* image2d_t;
typedef int sampler_t;

// OpenCL C keywords and built-in constants.
#define __kernel extern "C"
#define __global
#define __read_only
#define __constant static const
#define __local static
#define restrict __restrict__
#define int2 clshim::make_int2
#define CLK_NORMALIZED_COORDS_FALSE 0
#define CLK_ADDRESS_CLAMP_TO_EDGE 2
#define CLK_FILTER_NEAREST 0x10
#define CLK_LOCAL_MEM_FENCE 1
#define CLK_GLOBAL_MEM_FENCE 2
