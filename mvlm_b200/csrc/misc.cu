// misc.cu - element-wise device kernels around the matmul path: GGUF block dequantisation
// (standalone, for testing the in-kernel decoders), the ggml reference quantiser (to build
// synthetic GGUF weights on the device for benchmarks), seeded generators, type
// conversion, the patch_embed im2col gather (vision.cl:154-176 order) and the greedy-decode
// argmax over the lm_head's logits (src/models/moondream2.cpp:551-591, done there on the host).
#include "common.cuh"
#include "kernels.h"
#include "qdot.cuh"

using namespace mgpu_dev;

namespace {

__device__ __forceinline__ uint64_t splitmix64(uint64_t& s) {
    uint64_t z = (s += 0x9E3779B97F4A7C15ull);
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

template <typename T> __device__ __forceinline__ void store_as(void* out, int64_t i, float v) {
    reinterpret_cast<T*>(out)[i] = from_f32<T>(v);
}
__device__ __forceinline__ void store_typed(int otype, void* out, int64_t i, float v) {
    if (otype == MGPU_F32) store_as<float>(out, i, v);
    else if (otype == MGPU_F16) store_as<__half>(out, i, v);
    else store_as<__nv_bfloat16>(out, i, v);
}
__device__ __forceinline__ float load_typed(int itype, const void* in, int64_t i) {
    if (itype == MGPU_F32) return reinterpret_cast<const float*>(in)[i];
    if (itype == MGPU_F16) return __half2float(reinterpret_cast<const __half*>(in)[i]);
    return __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(in)[i]);
}

// One thread per 32-element block: w = (q - 8) * d (Q4_0) or q * d (Q8_0), exact in fp32.
__global__ void dequant_kernel(int qtype, const uint8_t* __restrict__ W, int otype, void* out, int64_t nblocks) {
    const int64_t b = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
    if (b >= nblocks) return;
    if (qtype == MGPU_Q4_0) {
        const uint8_t* p = W + b * 18;
        const float d = __half2float(__ushort_as_half((unsigned short)(p[0] | (p[1] << 8))));
        for (int j = 0; j < 16; ++j) {
            store_typed(otype, out, b * 32 + j, (float)((int)(p[2 + j] & 0xF) - 8) * d);
            store_typed(otype, out, b * 32 + j + 16, (float)((int)(p[2 + j] >> 4) - 8) * d);
        }
    } else {
        const uint8_t* p = W + b * 34;
        const float d = __half2float(__ushort_as_half((unsigned short)(p[0] | (p[1] << 8))));
        for (int j = 0; j < 32; ++j) store_typed(otype, out, b * 32 + j, (float)(int8_t)p[2 + j] * d);
    }
}

// ggml reference quantiser, one thread per block.  __fmul_rn / __fadd_rn keep the
// multiply and the +8.5 as two roundings (no FMA contraction), as the reference does.
__global__ void quantize_kernel(int qtype, const float* __restrict__ src, uint8_t* __restrict__ dst, int64_t nblocks) {
    const int64_t b = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
    if (b >= nblocks) return;
    const float* v = src + b * 32;
    if (qtype == MGPU_Q4_0) {
        float amax = 0.0f, vmax = 0.0f;
        for (int j = 0; j < 32; ++j) {
            const float a = fabsf(v[j]);
            if (amax < a) { amax = a; vmax = v[j]; }
        }
        const float d = __fdiv_rn(vmax, -8.0f);
        const float id = d != 0.0f ? __fdiv_rn(1.0f, d) : 0.0f;
        uint8_t qs[16];
        for (int j = 0; j < 16; ++j) {
            int q0 = (int)__fadd_rn(__fmul_rn(v[j], id), 8.5f);
            int q1 = (int)__fadd_rn(__fmul_rn(v[j + 16], id), 8.5f);
            q0 = min(q0, 15);
            q1 = min(q1, 15);
            qs[j] = (uint8_t)(q0 | (q1 << 4));
        }
        uint16_t* o = reinterpret_cast<uint16_t*>(dst + b * 18);  // blocks start on 2-byte boundaries
        o[0] = __half_as_ushort(__float2half_rn(d));
        for (int j = 0; j < 8; ++j) o[1 + j] = (uint16_t)(qs[2 * j] | ((uint16_t)qs[2 * j + 1] << 8));
    } else {
        float amax = 0.0f;
        for (int j = 0; j < 32; ++j) amax = fmaxf(amax, fabsf(v[j]));
        const float d = __fdiv_rn(amax, 127.0f);
        const float id = d != 0.0f ? __fdiv_rn(1.0f, d) : 0.0f;
        uint16_t* o = reinterpret_cast<uint16_t*>(dst + b * 34);
        o[0] = __half_as_ushort(__float2half_rn(d));
        for (int j = 0; j < 16; ++j) {
            const uint8_t q0 = (uint8_t)(int8_t)roundf(__fmul_rn(v[2 * j], id));
            const uint8_t q1 = (uint8_t)(int8_t)roundf(__fmul_rn(v[2 * j + 1], id));
            o[1 + j] = (uint16_t)(q0 | ((uint16_t)q1 << 8));
        }
    }
}

__global__ void fill_uniform_kernel(int otype, void* out, int64_t n, uint64_t seed, float lo, float hi) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
        uint64_t s = seed + (uint64_t)i;
        const float u = (float)(splitmix64(s) >> 40) * (1.0f / 16777216.0f);  // [0, 1)
        store_typed(otype, out, i, lo + (hi - lo) * u);
    }
}

__global__ void fill_normal_kernel(int otype, void* out, int64_t n, uint64_t seed, float sigma) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
        uint64_t s = seed + (uint64_t)i * 0x2545F4914F6CDD1Dull;
        const float u1 = ((float)(splitmix64(s) >> 40) + 1.0f) * (1.0f / 16777216.0f);  // (0, 1]
        const float u2 = (float)(splitmix64(s) >> 40) * (1.0f / 16777216.0f);
        store_typed(otype, out, i, sigma * sqrtf(-2.0f * logf(u1)) * cospif(2.0f * u2));
    }
}

__global__ void convert_kernel(int itype, const void* in, int otype, void* out, int64_t n) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
        store_typed(otype, out, i, load_typed(itype, in, i));
}

// patches[p][k]: p over the (H/ph) x (W/pw) grid row-major, k = c*ph*pw + py*pw + px,
// zero for k in [C*ph*pw, kpad).  16-bit element copy (no rounding).
template <typename T>
__global__ void im2col_kernel(const T* __restrict__ img, T* __restrict__ patches, int C, int H, int W, int ph,
                              int pw, int kpad, int64_t total) {
    const int gw = W / pw;
    const int pd = C * ph * pw;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t p = i / kpad;
        const int k = (int)(i % kpad);
        T v;
        if (k < pd) {
            const int c = k / (ph * pw), r = k % (ph * pw), py = r / pw, px = r % pw;
            const int pr = (int)(p / gw), pc = (int)(p % gw);
            v = img[(size_t)c * H * W + (size_t)(pr * ph + py) * W + (pc * pw + px)];
        } else {
            v = from_f32<T>(0.0f);
        }
        patches[i] = v;
    }
}

// Waits for a phase of an mbarrier on which no thread ever arrives: the bounded wait must
// expire, record the timeout in *status and return.
__global__ void selftest_wait_kernel(int* status, uint64_t limit_ns) {
    __shared__ __align__(8) uint64_t bar;
    if (threadIdx.x == 0) {
        mbar_init(&bar, 1);
        fence_mbar_init();
    }
    __syncthreads();
    if (threadIdx.x == 0) mbar_wait(&bar, 0, status, limit_ns);
}

// A logit as the reference's argmax compares it (moondream2.cpp:567-582, written there for
// fp16): exponent field zero (zero or subnormal) -> 0, all ones (Inf or NaN) -> +-1e30 by the
// sign bit, else the value.  bf16 and fp32 logits follow the same rule on their own fields.
__device__ __forceinline__ float argmax_value(int type, const void* x, int64_t i) {
    if (type == MGPU_F16) {
        const uint32_t h = reinterpret_cast<const uint16_t*>(x)[i];
        const uint32_t e = (h >> 10) & 0x1Fu;
        if (e == 0) return 0.0f;
        if (e == 31) return (h & 0x8000u) ? -1e30f : 1e30f;
        return __half2float(__ushort_as_half((unsigned short)h));
    }
    const uint32_t b = type == MGPU_F32 ? reinterpret_cast<const uint32_t*>(x)[i]
                                        : (uint32_t)reinterpret_cast<const uint16_t*>(x)[i] << 16;
    const uint32_t e = (b >> 23) & 0xFFu;
    if (e == 0) return 0.0f;
    if (e == 255) return (b & 0x80000000u) ? -1e30f : 1e30f;
    return __uint_as_float(b);
}

// RMSNorm over rows (src/kernels/layernorm.cl:41-146, dispatched by compute.cpp:156-184): one
// CTA of kRmsThreads threads per row, y = x * rsqrt(mean(x^2) + eps) * w in fp32, stored in y's type.
// Rows of a multiple of 4 elements at 16-byte (fp32) / 8-byte (16-bit) aligned addresses use
// the word order and reduction of rms_scale, the same as the fused GEMV prologue, so the two
// give the same bits; other rows take a per-element loop.
template <typename T>
__global__ void __launch_bounds__(kRmsThreads) rms_norm_kernel(const T* __restrict__ in, T* __restrict__ out, int wtype,
                                                       const void* __restrict__ w, int H, float eps, bool words) {
    __shared__ float red[kRmsThreads / 32];
    const int tid = threadIdx.x;
    const T* x = in + (size_t)blockIdx.x * H;
    T* y = out + (size_t)blockIdx.x * H;
    float ss = 0.0f;
    if (words) {
        for (int i = tid; i < H / 4; i += kRmsThreads) {
            float v[4];
            load_word4(x, i, v);
#pragma unroll
            for (int j = 0; j < 4; ++j) ss = fmaf(v[j], v[j], ss);
        }
    } else {
        for (int i = tid; i < H; i += kRmsThreads) {
            const float v = to_f32<T>(x[i]);
            ss = fmaf(v, v, ss);
        }
    }
    const float r = rms_scale(ss, red, tid, kRmsThreads, H, eps);
    if (words) {
        for (int i = tid; i < H / 4; i += kRmsThreads) {
            float v[4], g[4];
            load_word4(x, i, v);
            load_word4_typed(wtype, w, i, g);
#pragma unroll
            for (int j = 0; j < 4; ++j) y[4 * i + j] = from_f32<T>(v[j] * r * g[j]);
        }
    } else {
        for (int i = tid; i < H; i += kRmsThreads) y[i] = from_f32<T>(to_f32<T>(x[i]) * r * load_typed(wtype, w, i));
    }
}

// The ranks' (index, value) argmax pairs of a column-sharded row, in rank order, into the
// global first maximum: rank r's columns start at r * (n / R) + min(r, n % R); a strictly
// larger value wins, so equal values keep the lower rank's (smaller) index; nothing above
// -1e30 leaves index 0, as argmax_kernel starts.
__global__ void argmax_combine_kernel(const int* __restrict__ pairs, int n_ranks, int n_total, int* out) {
    if (threadIdx.x != 0) return;
    const int base = n_total / n_ranks, extra = n_total % n_ranks;
    float best = -1e30f;
    int bi = 0;
    for (int r = 0; r < n_ranks; ++r) {
        const float v = __int_as_float(pairs[2 * r + 1]);
        if (v > best) {
            best = v;
            bi = r * base + min(r, extra) + pairs[2 * r];
        }
    }
    out[0] = bi;
    out[1] = __float_as_int(best);
}

// One CTA: the first index whose value is greater than every earlier one, starting from
// (-1e30, index 0) as the reference does; out[0] = index, out[1] = its value (fp32 bits).
// Each thread scans a strided subsequence in index order keeping its first maximum; the
// pairs then combine by larger value, then smaller index, which gives the same index.
// One CTA per row (row r of the batch at element r * ld); its pair at out[2r].
__global__ void __launch_bounds__(1024) argmax_kernel(int type, const void* __restrict__ x, int n, int64_t ld,
                                                      int* out) {
    __shared__ float sv[32];
    __shared__ int si[32];
    const int64_t base = (int64_t)blockIdx.x * ld;
    out += 2 * blockIdx.x;
    float best = -1e30f;
    int bi = 0x7FFFFFFF;
    // eight of a thread's values loaded before any is compared, so that their loads are in
    // flight together; the comparisons stay in index order (first maximum)
    constexpr int U = 8;
    int i0 = threadIdx.x;
    for (; i0 + (U - 1) * (int)blockDim.x < n; i0 += U * blockDim.x) {
        float v[U];
#pragma unroll
        for (int u = 0; u < U; ++u) v[u] = argmax_value(type, x, base + i0 + u * blockDim.x);
#pragma unroll
        for (int u = 0; u < U; ++u)
            if (v[u] > best) {
                best = v[u];
                bi = i0 + u * blockDim.x;
            }
    }
    for (int i = i0; i < n; i += blockDim.x) {
        const float v = argmax_value(type, x, base + i);
        if (v > best) {
            best = v;
            bi = i;
        }
    }
    auto better = [](float v, int i, float w, int j) { return w > v || (w == v && j < i); };
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) {
        const float w = __shfl_xor_sync(0xffffffffu, best, off);
        const int j = __shfl_xor_sync(0xffffffffu, bi, off);
        if (better(best, bi, w, j)) {
            best = w;
            bi = j;
        }
    }
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (lane == 0) {
        sv[warp] = best;
        si[warp] = bi;
    }
    __syncthreads();
    if (warp == 0) {
        const int nw = (blockDim.x + 31) >> 5;
        best = lane < nw ? sv[lane] : -1e30f;
        bi = lane < nw ? si[lane] : 0x7FFFFFFF;
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) {
            const float w = __shfl_xor_sync(0xffffffffu, best, off);
            const int j = __shfl_xor_sync(0xffffffffu, bi, off);
            if (better(best, bi, w, j)) {
                best = w;
                bi = j;
            }
        }
        if (lane == 0) {
            // nothing above -1e30: the reference's initial index 0
            out[0] = best > -1e30f ? bi : 0;
            out[1] = __float_as_int(best);
        }
    }
}

int grid_for(int64_t n, int sm_count) {
    const int64_t want = (n + 255) / 256;
    const int64_t cap = (int64_t)sm_count * 16;
    return (int)(want < cap ? want : cap);
}

}  // namespace

namespace mgpu_k {

cudaError_t dequant(const LaunchCtx& c, int qtype, const uint8_t* W, int otype, void* out, int64_t n) {
    const int64_t nb = n / 32;
    if (nb <= 0) return cudaSuccess;
    dequant_kernel<<<(unsigned)((nb + 255) / 256), 256, 0, c.stream>>>(qtype, W, otype, out, nb);
    return cudaGetLastError();
}

cudaError_t quantize(const LaunchCtx& c, int qtype, const float* src, uint8_t* dst, int64_t n) {
    const int64_t nb = n / 32;
    if (nb <= 0) return cudaSuccess;
    quantize_kernel<<<(unsigned)((nb + 255) / 256), 256, 0, c.stream>>>(qtype, src, dst, nb);
    return cudaGetLastError();
}

cudaError_t fill_uniform(const LaunchCtx& c, int otype, void* out, int64_t n, uint64_t seed, float lo, float hi) {
    if (n <= 0) return cudaSuccess;
    fill_uniform_kernel<<<grid_for(n, c.sm_count), 256, 0, c.stream>>>(otype, out, n, seed, lo, hi);
    return cudaGetLastError();
}

cudaError_t fill_normal(const LaunchCtx& c, int otype, void* out, int64_t n, uint64_t seed, float sigma) {
    if (n <= 0) return cudaSuccess;
    fill_normal_kernel<<<grid_for(n, c.sm_count), 256, 0, c.stream>>>(otype, out, n, seed, sigma);
    return cudaGetLastError();
}

cudaError_t convert(const LaunchCtx& c, int itype, const void* in, int otype, void* out, int64_t n) {
    if (n <= 0) return cudaSuccess;
    convert_kernel<<<grid_for(n, c.sm_count), 256, 0, c.stream>>>(itype, in, otype, out, n);
    return cudaGetLastError();
}

cudaError_t argmax(const LaunchCtx& c, int type, const void* logits, int n, int* out) {
    return argmax_rows(c, type, logits, 1, n, n, out);
}

cudaError_t argmax_rows(const LaunchCtx& c, int type, const void* logits, int rows, int n, int64_t ld, int* out) {
    argmax_kernel<<<rows, 1024, 0, c.stream>>>(type, logits, n, ld, out);
    return cudaGetLastError();
}

cudaError_t rms_norm(const LaunchCtx& c, int type, const void* in, void* out, int wtype, const void* w, int rows,
                     int H, float eps) {
    if (rows <= 0) return cudaSuccess;
    const size_t align = type == MGPU_F32 ? 16 : 8;
    const bool words = H % 4 == 0 && ((uintptr_t)in % align) == 0 && ((uintptr_t)out % align) == 0 &&
                       ((uintptr_t)w % (wtype == MGPU_F32 ? 16 : 8)) == 0 && (H * (type == MGPU_F32 ? 4 : 2)) % align == 0;
    if (type == MGPU_F32)
        rms_norm_kernel<float><<<rows, kRmsThreads, 0, c.stream>>>((const float*)in, (float*)out, wtype, w, H, eps, words);
    else if (type == MGPU_F16)
        rms_norm_kernel<__half><<<rows, kRmsThreads, 0, c.stream>>>((const __half*)in, (__half*)out, wtype, w, H, eps, words);
    else
        rms_norm_kernel<__nv_bfloat16><<<rows, kRmsThreads, 0, c.stream>>>((const __nv_bfloat16*)in, (__nv_bfloat16*)out,
                                                                   wtype, w, H, eps, words);
    return cudaGetLastError();
}

cudaError_t argmax_combine(const LaunchCtx& c, const int* pairs, int n_ranks, int n_total, int* out) {
    argmax_combine_kernel<<<1, 32, 0, c.stream>>>(pairs, n_ranks, n_total, out);
    return cudaGetLastError();
}

cudaError_t selftest_bounded_wait(const LaunchCtx& c, uint64_t limit_ns) {
    selftest_wait_kernel<<<1, 32, 0, c.stream>>>(c.status, limit_ns);
    return cudaGetLastError();
}

cudaError_t im2col(const LaunchCtx& c, int type, const void* img, void* patches, int C, int H, int W, int ph,
                   int pw, int kpad) {
    const int64_t total = (int64_t)(H / ph) * (W / pw) * kpad;
    if (total <= 0) return cudaSuccess;
    const int g = grid_for(total, c.sm_count);
    if (type == MGPU_F16)
        im2col_kernel<__half><<<g, 256, 0, c.stream>>>((const __half*)img, (__half*)patches, C, H, W, ph, pw, kpad, total);
    else if (type == MGPU_BF16)
        im2col_kernel<__nv_bfloat16><<<g, 256, 0, c.stream>>>((const __nv_bfloat16*)img, (__nv_bfloat16*)patches, C, H,
                                                             W, ph, pw, kpad, total);
    else
        return cudaErrorInvalidValue;
    return cudaGetLastError();
}

}  // namespace mgpu_k
