// qdot.cuh - exact integer inner products of GGUF Q4_0 / Q8_0 blocks against activations held
// in 16-bit fixed point, shared by the decode GEMV kernels (gemv.cu) and the persistent
// decode-step kernel (chain.cu).  Q4_0: 32 weights = fp16 d + 16 bytes, element j < 16 the low
// nibble of byte j, element j + 16 its high nibble, w = (q - 8) d; Q8_0: fp16 d + 32 int8,
// w = q d (the ggml block format, gguf_loader.cpp:17,21,39,43 of the reference).
#pragma once
#include "common.cuh"

namespace mgpu_dev {

template <int QT> struct QTraits;
template <> struct QTraits<MGPU_Q4_0> {
    static constexpr int kBlockBytes = 18;
    static constexpr int kWords = 5;  // 20 aligned bytes cover an 18-byte block at offset 0 or 2
};
template <> struct QTraits<MGPU_Q8_0> {
    static constexpr int kBlockBytes = 34;
    static constexpr int kWords = 9;
};

// ---- integer inner product ---------------------------------------------------------
// Each consumer thread owns one 32-element block column for the whole launch.  Its 32
// activations are converted once to 16-bit fixed point relative to their own max
// (x_i = X_i * 2^(e-15), -2^15 <= X_i < 2^15, |x| < 2^e over the block) and split into two byte
// planes X = b1 * 2^8 + b0 (b0 unsigned, b1 signed), packed four elements per word in the
// order the quant bytes arrive.  A block's sum_k X_k q_k is then exact integer arithmetic: one
// dp4a per four weights and byte plane, straight on the packed nibbles (Q4_0: q & 0x0F0F0F0F,
// and (q & 0xF0F0F0F0) = 16 * the high nibbles) or int8 (Q8_0).  The only rounding before the
// fp32 block scale is X itself: at most 2^-16 of the block's largest |x| per element.
__device__ __forceinline__ int dp4a_uu(uint32_t a, uint32_t b, int c) {
    int d;
    asm("dp4a.u32.u32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}
__device__ __forceinline__ int dp4a_us(uint32_t a, uint32_t b, int c) {
    int d;
    asm("dp4a.u32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}
__device__ __forceinline__ int dp4a_su(uint32_t a, uint32_t b, int c) {
    int d;
    asm("dp4a.s32.u32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}
__device__ __forceinline__ int dp4a_ss(uint32_t a, uint32_t b, int c) {
    int d;
    asm("dp4a.s32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}

constexpr int kXPlanes = 2;

// The thread's activations in fixed point.  p[plane][w]: plane 0, 1 = b0, b1; w = 0..7 =
// elements 4w..4w+3.  scale = 2^(e-15); scale16 = scale / 16; xs128 = 128 * sum_k X_k.
struct XFixed {
    uint32_t p[kXPlanes][8];
    float scale;
    float scale16;
    int xs128;
};

// Where word w of a plane is kept.  A thread reads its block column c as two 16-byte halves
// (words 8c .. 8c+3 and 8c+4 .. 8c+7); a quarter warp's eight 16-byte reads hit distinct bank
// groups only if the halves of columns 4 .. 7 (mod 8) swap places, so they do.
__device__ __forceinline__ int plane_slot(int w) { return w ^ ((w >> 3) & 4); }

// Word w (elements 4w .. 4w+3) of the activations into fixed point: the 8 lanes holding the
// words of one 32-element block (lanes 8j .. 8j+7 of a warp, w % 8 == lane % 8) call this
// together and agree on the block's exponent with shuffles; `leader` (lane % 8 == 0) stores the
// block's scale.
__device__ __forceinline__ void convert_x_word(const float (&v)[4], int w, int words, uint32_t* planes, float* bscale,
                                               bool leader) {
    float amax = fmaxf(fmaxf(fabsf(v[0]), fabsf(v[1])), fmaxf(fabsf(v[2]), fabsf(v[3])));
#pragma unroll
    for (int off = 1; off < 8; off <<= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, off));
    int e = 0;
    frexpf(amax, &e);  // the block's |x| < 2^e
    const float up = __int_as_float((127 + 15 - e) << 23);  // 2^(15-e); |e| < 100 for finite x
    // X = round-to-nearest-even(v * 2^(15-e)) in [-2^15, 2^15]: one fma against 1.5 * 2^23 puts
    // X + 2^23 + 2^22 in [2^23, 2^24] with a unit step, so its bits minus those of 1.5 * 2^23
    // are X (v * up is exact, so this equals __float2int_rn(v * up)); the one value that can
    // round up to 2^15 is clamped to 2^15 - 1 so that b1 stays a signed byte.  The byte planes of
    // the four elements are gathered with byte permutes.
    uint32_t X[4];
#pragma unroll
    for (int j = 0; j < 4; ++j)
        X[j] = (uint32_t)min(__float_as_int(fmaf(v[j], up, 12582912.0f)) - 0x4B400000, 32767);
    const uint32_t t01 = prmt(X[0], X[1], 0x5140u), t23 = prmt(X[2], X[3], 0x5140u);
    const int ws = plane_slot(w);
    planes[ws] = prmt(t01, t23, 0x5410u);          // byte 0 of X[0..3]
    planes[words + ws] = prmt(t01, t23, 0x7632u);  // byte 1
    if (leader) bscale[w >> 3] = __int_as_float((127 + e - 15) << 23);  // 2^(e-15)
}

// The CTA converts all K activations once, cooperatively: thread t takes 4 consecutive
// elements at a time, the 8 threads of a 32-element block agree on the block's exponent
// with shuffles, and the packed byte planes go to shared memory:
//   planes[p * (K/4) + plane_slot(w)]  (w = word index = element / 4), bscale[b] per block b.
// Consumer threads then read their own block's 16 words.  Costs one round trip to L2 plus a
// handful of instructions per thread, instead of 32 loads and conversions per thread.
// words = K / 4 is a multiple of 256 (K % 1024 == 0); thread t converts words it * nthreads + t
// for it < ITERS = ceil(words / nthreads) (a compile-time count, so that all loads are issued
// before any is used and the activation vector costs one round trip).  Whole warps fall
// outside `words` when it is smaller than nthreads, so the shuffles stay warp-uniform.
template <typename XT, int ITERS>
__device__ __forceinline__ void prepare_x_n(const XT* __restrict__ x, int K, uint32_t* planes, float* bscale,
                                            int tid, int nthreads) {
    const int words = K / 4;
    float v[ITERS][4];
#pragma unroll
    for (int it = 0; it < ITERS; ++it) {
        const int w = it * nthreads + tid;
        if (w < words) {
            if constexpr (sizeof(XT) == 4) {
                const float4 f = __ldg(reinterpret_cast<const float4*>(x) + w);
                v[it][0] = f.x; v[it][1] = f.y; v[it][2] = f.z; v[it][3] = f.w;
            } else {
                const uint2 u = __ldg(reinterpret_cast<const uint2*>(x) + w);
                const uint32_t uu[2] = {u.x, u.y};
#pragma unroll
                for (int j = 0; j < 2; ++j) {
                    XT lo, hi;
                    uint16_t l16 = (uint16_t)(uu[j] & 0xFFFF), h16 = (uint16_t)(uu[j] >> 16);
                    memcpy(&lo, &l16, 2);
                    memcpy(&hi, &h16, 2);
                    v[it][2 * j] = to_f32<XT>(lo);
                    v[it][2 * j + 1] = to_f32<XT>(hi);
                }
            }
        }
    }
#pragma unroll
    for (int it = 0; it < ITERS; ++it) {
        const int w = it * nthreads + tid;
        if (w < words) convert_x_word(v[it], w, words, planes, bscale, (tid & 7) == 0);
    }
}

// Four consecutive values of a float-typed vector (f32 / f16 / bf16) at word w, as fp32.
template <typename T>
__device__ __forceinline__ void load_word4(const T* __restrict__ p, int w, float (&v)[4]) {
    if constexpr (sizeof(T) == 4) {
        const float4 f = __ldg(reinterpret_cast<const float4*>(p) + w);
        v[0] = f.x; v[1] = f.y; v[2] = f.z; v[3] = f.w;
    } else {
        const uint2 u = __ldg(reinterpret_cast<const uint2*>(p) + w);
        const uint32_t uu[2] = {u.x, u.y};
#pragma unroll
        for (int j = 0; j < 2; ++j) {
            T lo, hi;
            uint16_t l16 = (uint16_t)(uu[j] & 0xFFFF), h16 = (uint16_t)(uu[j] >> 16);
            memcpy(&lo, &l16, 2);
            memcpy(&hi, &h16, 2);
            v[2 * j] = to_f32<T>(lo);
            v[2 * j + 1] = to_f32<T>(hi);
        }
    }
}
__device__ __forceinline__ void load_word4_typed(int type, const void* p, int w, float (&v)[4]) {
    if (type == MGPU_F32) load_word4(reinterpret_cast<const float*>(p), w, v);
    else if (type == MGPU_F16) load_word4(reinterpret_cast<const __half*>(p), w, v);
    else load_word4(reinterpret_cast<const __nv_bfloat16*>(p), w, v);
}

// RMSNorm's scale rsqrt(mean(x^2) + eps) (src/kernels/layernorm.cl:41-146), K values held by
// `nthreads` threads (a multiple of 32) as 4-element words it * nthreads + tid, from each
// thread's partial sum of squares `ss` (its words in order, fmaf per value): a xor butterfly in
// each warp, then the warps' sums added in warp order through red[nthreads / 32], shared with
// named barrier 1.  The standalone kernel and the GEMV prologue both call this with
// kRmsThreads threads, so their normalised vectors have the same bits.
constexpr int kRmsThreads = 512;
__device__ __forceinline__ float rms_scale(float ss, float* red, int tid, int nthreads, int K, float eps) {
#pragma unroll
    for (int off = 16; off >= 1; off >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, off);
    if ((tid & 31) == 0) red[tid >> 5] = ss;
    named_barrier_sync(1, nthreads);
    float total = 0.0f;
    for (int w = 0; w < nthreads / 32; ++w) total += red[w];
    return rsqrtf(total / (float)K + eps);
}

// prepare_x with the RMSNorm of x in front: x_k * rsqrt(mean(x^2) + eps) * gamma_k, rounded to
// x's own type, as the reference's rms_norm writes its output in the input's type before the
// projection reads it; then the fixed-point conversion.  red: nthreads / 32 floats of scratch.
template <typename XT, int ITERS>
__device__ __forceinline__ void prepare_x_norm_n(const XT* __restrict__ x, const void* gamma, int gtype, float eps,
                                                 int K, uint32_t* planes, float* bscale, float* red,
                                                 int tid, int nthreads) {
    const int words = K / 4;
    float v[ITERS][4];
    float ss = 0.0f;
#pragma unroll
    for (int it = 0; it < ITERS; ++it)
        if (it * nthreads + tid < words) load_word4(x, it * nthreads + tid, v[it]);
#pragma unroll
    for (int it = 0; it < ITERS; ++it)
        if (it * nthreads + tid < words)
#pragma unroll
            for (int j = 0; j < 4; ++j) ss = fmaf(v[it][j], v[it][j], ss);
    const float r = rms_scale(ss, red, tid, nthreads, K, eps);
#pragma unroll
    for (int it = 0; it < ITERS; ++it) {
        const int w = it * nthreads + tid;
        if (w < words) {
            float g[4];
            load_word4_typed(gtype, gamma, w, g);
#pragma unroll
            for (int j = 0; j < 4; ++j) v[it][j] = to_f32<XT>(from_f32<XT>(v[it][j] * r * g[j]));
            convert_x_word(v[it], w, words, planes, bscale, (tid & 7) == 0);
        }
    }
}

// The conversion loops for K % 1024 == 0, 1024 <= K <= 8192 * nthreads / 256.
template <typename XT>
__device__ __forceinline__ void prepare_x_norm(const XT* __restrict__ x, const void* gamma, int gtype, float eps,
                                               int K, uint32_t* planes, float* bscale, float* red, int tid,
                                               int nthreads) {
    const int iters = (K / 4 + nthreads - 1) / nthreads;
    if (iters <= 1) prepare_x_norm_n<XT, 1>(x, gamma, gtype, eps, K, planes, bscale, red, tid, nthreads);
    else if (iters <= 2) prepare_x_norm_n<XT, 2>(x, gamma, gtype, eps, K, planes, bscale, red, tid, nthreads);
    else if (iters <= 4) prepare_x_norm_n<XT, 4>(x, gamma, gtype, eps, K, planes, bscale, red, tid, nthreads);
    else prepare_x_norm_n<XT, 8>(x, gamma, gtype, eps, K, planes, bscale, red, tid, nthreads);
}

template <typename XT>
__device__ __forceinline__ void prepare_x(const XT* __restrict__ x, int K, uint32_t* planes, float* bscale,
                                          int tid, int nthreads) {
    const int iters = (K / 4 + nthreads - 1) / nthreads;
    if (iters <= 1) prepare_x_n<XT, 1>(x, K, planes, bscale, tid, nthreads);
    else if (iters <= 2) prepare_x_n<XT, 2>(x, K, planes, bscale, tid, nthreads);
    else if (iters <= 4) prepare_x_n<XT, 4>(x, K, planes, bscale, tid, nthreads);
    else prepare_x_n<XT, 8>(x, K, planes, bscale, tid, nthreads);
}

// The thread's block column `col` of the planes, its block scale and 128 * sum_k X_k (the
// Q4_0 offset term, from the planes with dp4a: sum b0 + 256 * sum b1).
__device__ __forceinline__ void load_xfixed(const uint32_t* planes, const float* bscale, int words, int col,
                                            XFixed& xf) {
    const int sw = (col >> 2) & 1;  // plane_slot: columns 4 .. 7 (mod 8) keep their halves swapped
#pragma unroll
    for (int p = 0; p < kXPlanes; ++p) {
        const uint4* src = reinterpret_cast<const uint4*>(planes + p * words + col * 8);
        const uint4 a = src[sw], b = src[sw ^ 1];
        xf.p[p][0] = a.x; xf.p[p][1] = a.y; xf.p[p][2] = a.z; xf.p[p][3] = a.w;
        xf.p[p][4] = b.x; xf.p[p][5] = b.y; xf.p[p][6] = b.z; xf.p[p][7] = b.w;
    }
    xf.scale = bscale[col];
    xf.scale16 = xf.scale * 0.0625f;
    int s0 = 0, s1 = 0;
#pragma unroll
    for (int w = 0; w < 8; ++w) {
        s0 = dp4a_uu(0x01010101u, xf.p[0][w], s0);
        s1 = dp4a_us(0x01010101u, xf.p[1][w], s1);
    }
    xf.xs128 = 128 * (s0 + 256 * s1);
}

// One Q4_0 block against the thread's activations.  w = the 20 aligned bytes containing the
// block; `sel` realigns the 16 quant bytes, `dsel` extracts the fp16 scale.  Element j < 16
// is the low nibble of qs[j], element j + 16 the high nibble.
// Returns d * sum_k x_k (q_k - 8).
__device__ __forceinline__ float q4_0_block_dot(const uint32_t (&w)[5], uint32_t sel, uint32_t dsel,
                                                const XFixed& xf) {
    const float d = __half2float(__ushort_as_half((unsigned short)prmt(w[0], 0u, dsel)));
    int lo0 = 0, lo1 = 0, hi0 = 0, hi1 = 0;
#pragma unroll
    for (int m = 0; m < 4; ++m) {
        const uint32_t q = prmt(w[m], w[m + 1], sel);
        const uint32_t lo = q & 0x0F0F0F0Fu;  // elements 4m..4m+3
        const uint32_t hi = q & 0xF0F0F0F0u;  // 16 x elements 16+4m..16+4m+3
        lo0 = dp4a_uu(lo, xf.p[0][m], lo0);
        lo1 = dp4a_us(lo, xf.p[1][m], lo1);
        hi0 = dp4a_uu(hi, xf.p[0][4 + m], hi0);
        hi1 = dp4a_us(hi, xf.p[1][4 + m], hi1);
    }
    // 16 * sum X (q - 8) = 16 * sum X q - 128 * sum X, exact in int32 (|X| <= 2^15: each plane's
    // 16 * sum stays below 2^21, the total below 2^29)
    const int s = (lo0 * 16 + hi0) + 256 * (lo1 * 16 + hi1) - xf.xs128;
    return d * xf.scale16 * (float)s;
}

// One Q8_0 block: 32 signed bytes, w = q * d.
__device__ __forceinline__ float q8_0_block_dot(const uint32_t (&w)[9], uint32_t sel, uint32_t dsel,
                                                const XFixed& xf) {
    const float d = __half2float(__ushort_as_half((unsigned short)prmt(w[0], 0u, dsel)));
    int a0 = 0, a1 = 0;
#pragma unroll
    for (int m = 0; m < 8; ++m) {
        const uint32_t q = prmt(w[m], w[m + 1], sel);  // elements 4m..4m+3
        a0 = dp4a_su(q, xf.p[0][m], a0);
        a1 = dp4a_ss(q, xf.p[1][m], a1);
    }
    // sum X q, exact in int32 (|sum| <= 32 * 128 * 2^15 = 2^27)
    return d * xf.scale * (float)(a0 + 256 * a1);
}

template <int QT, int NW>
__device__ __forceinline__ float q_block_dot(const uint32_t (&w)[NW], uint32_t sel, uint32_t dsel,
                                             const XFixed& xf) {
    if constexpr (QT == MGPU_Q4_0) return q4_0_block_dot(w, sel, dsel, xf);
    else return q8_0_block_dot(w, sel, dsel, xf);
}

// Transposing butterfly: v[0..R) per lane in, the 32-lane sum of row `row` out, where lanes
// with lane % (32 / R) == 0 hold distinct rows.
template <int R>
__device__ __forceinline__ float warp_reduce_rows(float (&v)[R], int lane, int& row) {
    constexpr int LOG = (R == 1) ? 0 : (R == 2) ? 1 : (R == 4) ? 2 : 3;
    row = 0;
#pragma unroll
    for (int step = 0; step < LOG; ++step) {
        const int h = R >> (step + 1);
        const int off = 16 >> step;
        const bool up = (lane & off) != 0;
#pragma unroll
        for (int k = 0; k < (R >> 1); ++k) {
            if (k < h) {
                const float send = up ? v[k] : v[k + h];
                const float keep = up ? v[k + h] : v[k];
                v[k] = keep + __shfl_xor_sync(0xffffffffu, send, off);
            }
        }
        if (up) row += h;
    }
#pragma unroll
    for (int off = 16 >> LOG; off >= 1; off >>= 1) v[0] += __shfl_xor_sync(0xffffffffu, v[0], off);
    return v[0];
}

}  // namespace mgpu_dev
