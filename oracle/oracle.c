/*
 * oracle.c - CPU restatement of MVLM's matmul hot path.  TEST INFRASTRUCTURE ONLY.
 *
 * Loaded by tests/, __graft_entry__.smoke() and the CPU-baseline leg of bench.py, as the
 * checker.  Nothing in the product (mvlm_b200/) links or calls it.
 *
 * Reference files restated (paths relative to the drxddy/MVLM project root):
 *   src/kernels/gemm.cl            gemm_naive :26-51, gemm_tiled :74-136, gemm_image :157-200,
 *                                  gemv :219-270 (WG size 256 :215-217)
 *   src/kernels/vision.cl          patch_embed im2col order :154-176, bias :180-186,
 *                                  vision_proj bias :430-434
 *   src/models/gguf_loader.cpp     ggml_type_size :13-33, ggml_type_block_size :35-55
 *   GGUF Q4_0 / Q8_0 block format  (no code in the reference: gguf_loader.h:12-30 only names
 *                                  the types).  Restated from the published ggml format and
 *                                  pinned against gguf-py 0.19.0 (tests/golden/make_golden.py).
 */
#include "oracle.h"

#include <math.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

/* ------------------------------------------------------------------------------------ */
/* IEEE conversions.  binary16 uses the compiler's _Float16 (IEEE round-to-nearest-even    */
/* conversion, GCC >= 12 on x86-64); bfloat16 is the upper half of binary32 with RNE.      */
/* ------------------------------------------------------------------------------------ */
float ora_f16_to_f32(uint16_t h) {
    _Float16 v;
    memcpy(&v, &h, 2);
    return (float)v;
}

uint16_t ora_f32_to_f16(float f) {
    _Float16 v = (_Float16)f;
    uint16_t h;
    memcpy(&h, &v, 2);
    return h;
}

float ora_bf16_to_f32(uint16_t h) {
    uint32_t u = (uint32_t)h << 16;
    float f;
    memcpy(&f, &u, 4);
    return f;
}

uint16_t ora_f32_to_bf16(float f) {
    uint32_t u;
    memcpy(&u, &f, 4);
    if ((u & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((u >> 16) | 0x40u); /* quiet NaN */
    u += 0x7fffu + ((u >> 16) & 1u);
    return (uint16_t)(u >> 16);
}

void ora_f32_to_f16_n(const float* x, uint16_t* y, size_t n) {
    for (size_t i = 0; i < n; ++i) y[i] = ora_f32_to_f16(x[i]);
}
void ora_f16_to_f32_n(const uint16_t* x, float* y, size_t n) {
    for (size_t i = 0; i < n; ++i) y[i] = ora_f16_to_f32(x[i]);
}
void ora_f32_to_bf16_n(const float* x, uint16_t* y, size_t n) {
    for (size_t i = 0; i < n; ++i) y[i] = ora_f32_to_bf16(x[i]);
}
void ora_bf16_to_f32_n(const uint16_t* x, float* y, size_t n) {
    for (size_t i = 0; i < n; ++i) y[i] = ora_bf16_to_f32(x[i]);
}

/* ------------------------------------------------------------------------------------ */
/* ggml type table (gguf_loader.cpp:13-55, the entries this path uses).                   */
/* ------------------------------------------------------------------------------------ */
size_t ora_type_size(int type) {
    switch (type) {
        case ORA_F32: return 4;
        case ORA_F16: return 2;
        case ORA_BF16: return 2;
        case ORA_Q4_0: return 18; /* fp16 d + 16 nibble bytes */
        case ORA_Q8_0: return 34; /* fp16 d + 32 int8 */
        default: return 0;
    }
}

int ora_block_size(int type) {
    switch (type) {
        case ORA_F32: case ORA_F16: case ORA_BF16: return 1;
        case ORA_Q4_0: case ORA_Q8_0: return 32;
        default: return 0;
    }
}

size_t ora_row_bytes(int type, int64_t k) {
    int bs = ora_block_size(type);
    if (bs == 0) return 0;
    return (size_t)((k + bs - 1) / bs) * ora_type_size(type);
}

/* ------------------------------------------------------------------------------------ */
/* Seeded generators.                                                                     */
/* ------------------------------------------------------------------------------------ */
uint64_t ora_splitmix64(uint64_t* state) {
    uint64_t z = (*state += 0x9E3779B97F4A7C15ull);
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

void ora_fill_uniform(float* out, size_t n, uint64_t seed) {
    uint64_t s = seed;
    for (size_t i = 0; i < n; ++i) {
        uint64_t u = ora_splitmix64(&s);
        out[i] = (float)(u >> 40) * (1.0f / 8388608.0f) - 1.0f;
    }
}

void ora_fill_normal(float* out, size_t n, uint64_t seed, float sigma) {
    uint64_t s = seed;
    const double two_pi = 6.283185307179586476925286766559;
    for (size_t i = 0; i < n; i += 2) {
        double u1 = ((double)(ora_splitmix64(&s) >> 11) + 1.0) * (1.0 / 9007199254740992.0);
        double u2 = (double)(ora_splitmix64(&s) >> 11) * (1.0 / 9007199254740992.0);
        double r = sqrt(-2.0 * log(u1));
        out[i] = (float)(sigma * r * cos(two_pi * u2));
        if (i + 1 < n) out[i + 1] = (float)(sigma * r * sin(two_pi * u2));
    }
}

/* ------------------------------------------------------------------------------------ */
/* GGUF block quantisation.  Q4_0: d = (signed value of largest magnitude) / -8,          */
/* q = min(15, trunc(x/d + 8.5)); element j in the low nibble of byte j, element j+16 in  */
/* the high nibble.  Q8_0: d = max|x| / 127, q = round-half-away(x/d).  The reciprocal is  */
/* taken from the fp32 d; the block stores d rounded to fp16.                              */
/* ------------------------------------------------------------------------------------ */
void ora_quantize_q4_0(const float* x, uint8_t* blocks, int64_t n) {
    int64_t nb = n / 32;
    for (int64_t b = 0; b < nb; ++b) {
        const float* v = x + b * 32;
        uint8_t* out = blocks + b * 18;
        float amax = 0.0f, vmax = 0.0f;
        for (int j = 0; j < 32; ++j) {
            float a = fabsf(v[j]);
            if (amax < a) { amax = a; vmax = v[j]; }
        }
        float d = vmax / -8.0f;
        float id = d != 0.0f ? 1.0f / d : 0.0f;
        uint16_t dh = ora_f32_to_f16(d);
        memcpy(out, &dh, 2);
        for (int j = 0; j < 16; ++j) {
            float x0 = v[j] * id + 8.5f;
            float x1 = v[j + 16] * id + 8.5f;
            int q0 = (int)x0, q1 = (int)x1; /* trunc toward zero; x0, x1 >= 0.5 */
            if (q0 > 15) q0 = 15;
            if (q1 > 15) q1 = 15;
            out[2 + j] = (uint8_t)(q0 | (q1 << 4));
        }
    }
}

void ora_quantize_q8_0(const float* x, uint8_t* blocks, int64_t n) {
    int64_t nb = n / 32;
    for (int64_t b = 0; b < nb; ++b) {
        const float* v = x + b * 32;
        uint8_t* out = blocks + b * 34;
        float amax = 0.0f;
        for (int j = 0; j < 32; ++j) {
            float a = fabsf(v[j]);
            if (a > amax) amax = a;
        }
        float d = amax / 127.0f;
        float id = d != 0.0f ? 1.0f / d : 0.0f;
        uint16_t dh = ora_f32_to_f16(d);
        memcpy(out, &dh, 2);
        for (int j = 0; j < 32; ++j) {
            float q = roundf(v[j] * id);
            out[2 + j] = (uint8_t)(int8_t)q;
        }
    }
}

void ora_dequant(const uint8_t* blocks, float* out, int64_t n, int type) {
    int64_t nb = n / 32;
    for (int64_t b = 0; b < nb; ++b) {
        if (type == ORA_Q4_0) {
            const uint8_t* p = blocks + b * 18;
            float d = ora_f16_to_f32((uint16_t)(p[0] | (p[1] << 8)));
            for (int j = 0; j < 16; ++j) {
                out[b * 32 + j] = (float)((int)(p[2 + j] & 0x0F) - 8) * d;
                out[b * 32 + j + 16] = (float)((int)(p[2 + j] >> 4) - 8) * d;
            }
        } else if (type == ORA_Q8_0) {
            const uint8_t* p = blocks + b * 34;
            float d = ora_f16_to_f32((uint16_t)(p[0] | (p[1] << 8)));
            for (int j = 0; j < 32; ++j) out[b * 32 + j] = (float)(int8_t)p[2 + j] * d;
        }
    }
}

/* ------------------------------------------------------------------------------------ */
/* gemm.cl restatements.                                                                  */
/* ------------------------------------------------------------------------------------ */

/* gemm_naive (gemm.cl:26-51): one output per work-item; acc = fma(a, b, acc) in k order,
 * operands widened from fp16 (vload_half), single fp16 store (vstore_half, RNE).
 * gemm_tiled (:74-136) reads the same fp16 values through __local tiles and adds
 * fma(0, 0, acc) for zero-padded k >= K, which leaves acc unchanged; gemm_image
 * (:157-200) reads B through 4-column texels whose padding is never stored.  All three
 * therefore produce this exact sequence of roundings. */
void ora_gemm_naive_f16(const uint16_t* A, const uint16_t* B, uint16_t* C, int M, int N, int K) {
    for (int m = 0; m < M; ++m)
        for (int n = 0; n < N; ++n) {
            float acc = 0.0f;
            for (int k = 0; k < K; ++k)
                acc = fmaf(ora_f16_to_f32(A[(size_t)m * K + k]), ora_f16_to_f32(B[(size_t)k * N + n]), acc);
            C[(size_t)m * N + n] = ora_f32_to_f16(acc);
        }
}

void ora_gemm_naive_f32(const float* A, const float* B, float* C, int M, int N, int K) {
    for (int m = 0; m < M; ++m)
        for (int n = 0; n < N; ++n) {
            float acc = 0.0f;
            for (int k = 0; k < K; ++k) acc = fmaf(A[(size_t)m * K + k], B[(size_t)k * N + n], acc);
            C[(size_t)m * N + n] = acc;
        }
}

/* gemv (gemm.cl:219-270): work-item lid of a 256-wide group accumulates k = lid,
 * lid+256, ... with fma; the group then tree-reduces scratch[lid] += scratch[lid+stride]
 * for stride = 128, 64, ..., 1.  Components of the float4 are independent, so each
 * output column follows this order on its own. */
#define ORA_GEMV_WG 256
static float gemv_column_f32(const float* x, const float* W, int n, int N, int K) {
    float part[ORA_GEMV_WG];
    for (int lid = 0; lid < ORA_GEMV_WG; ++lid) {
        float p = 0.0f;
        for (int k = lid; k < K; k += ORA_GEMV_WG) p = fmaf(x[k], W[(size_t)k * N + n], p);
        part[lid] = p;
    }
    for (int s = ORA_GEMV_WG >> 1; s > 0; s >>= 1)
        for (int lid = 0; lid < s; ++lid) part[lid] += part[lid + s];
    return part[0];
}

void ora_gemv_f32(const float* x, const float* W, float* y, int N, int K) {
    for (int n = 0; n < N; ++n) y[n] = gemv_column_f32(x, W, n, N, K);
}

void ora_gemv_f16(const uint16_t* x, const uint16_t* W, uint16_t* y, int N, int K) {
    float part[ORA_GEMV_WG];
    for (int n = 0; n < N; ++n) {
        for (int lid = 0; lid < ORA_GEMV_WG; ++lid) {
            float p = 0.0f;
            for (int k = lid; k < K; k += ORA_GEMV_WG)
                p = fmaf(ora_f16_to_f32(x[k]), ora_f16_to_f32(W[(size_t)k * N + n]), p);
            part[lid] = p;
        }
        for (int s = ORA_GEMV_WG >> 1; s > 0; s >>= 1)
            for (int lid = 0; lid < s; ++lid) part[lid] += part[lid + s];
        y[n] = ora_f32_to_f16(part[0]);
    }
}

/* Quantised path: dequantise one weight row (exact) then the gemm_naive fp32 loop. */
void ora_gemm_q(const float* A, const uint8_t* W, float* C, int M, int N, int K, int type) {
    size_t rb = ora_row_bytes(type, K);
    float row[65536];
    for (int n = 0; n < N; ++n) {
        ora_dequant(W + (size_t)n * rb, row, K, type);
        for (int m = 0; m < M; ++m) {
            float acc = 0.0f;
            for (int k = 0; k < K; ++k) acc = fmaf(A[(size_t)m * K + k], row[k], acc);
            C[(size_t)m * N + n] = acc;
        }
    }
}

static float load_dense(const void* W, int wtype, size_t i) {
    if (wtype == ORA_F32) return ((const float*)W)[i];
    if (wtype == ORA_F16) return ora_f16_to_f32(((const uint16_t*)W)[i]);
    return ora_bf16_to_f32(((const uint16_t*)W)[i]);
}

void ora_gemm_nk(const float* A, const void* W, int wtype, float* C, int M, int N, int K) {
    for (int n = 0; n < N; ++n)
        for (int m = 0; m < M; ++m) {
            float acc = 0.0f;
            for (int k = 0; k < K; ++k)
                acc = fmaf(A[(size_t)m * K + k], load_dense(W, wtype, (size_t)n * K + k), acc);
            C[(size_t)m * N + n] = acc;
        }
}

void ora_add_bias(float* C, const float* bias, int M, int N) {
    for (int m = 0; m < M; ++m)
        for (int n = 0; n < N; ++n) C[(size_t)m * N + n] += bias[n];
}

/* Elementwise kernels of src/kernels/activations.cl, one element as the kernels' scalar tails
 * compute it (fp32 math; native_exp and native_recip taken as exp and 1/x):
 *   act 2, silu (:30-65): x * 1 / (1 + exp(-x));
 *   act 3, gelu as the kernel computes it (:78-117): inner = 0.7978845608 * fma(0.044715, x^3, x),
 *          tanh_val = 1 - 2 / (1 + exp(-2 inner)), 0.5 x (1 + tanh_val);
 *   act 1, gelu as compute.h:48 states it: the same with tanh_val = tanh(inner). */
float ora_activate(float x, int act) {
    if (act == 2) return x * (1.0f / (1.0f + expf(-x)));
    if (act == 1 || act == 3) {
        float x3 = x * x * x;
        float inner = 0.7978845608f * fmaf(0.044715f, x3, x);
        float t = act == 3 ? 1.0f - 2.0f * (1.0f / (1.0f + expf(-2.0f * inner))) : tanhf(inner);
        return 0.5f * x * (1.0f + t);
    }
    return x;
}

void ora_activate_n(float* x, size_t n, int act) {
    for (size_t i = 0; i < n; ++i) x[i] = ora_activate(x[i], act);
}

/* rms_norm (src/kernels/layernorm.cl:41-146), one row as its work-group computes it: the sum of
 * squares in fp32 with fma, rms_scale = rsqrt(sum / hidden + eps) (native_rsqrt taken as
 * 1 / sqrt), then val * rms_scale * w in fp32 in that order; the caller rounds to the output
 * type (the kernel stores half). */
void ora_rms_norm(const float* x, const float* w, float* out, int rows, int hidden, float eps) {
    for (int r = 0; r < rows; ++r) {
        const float* xr = x + (size_t)r * hidden;
        float ss = 0.0f;
        for (int i = 0; i < hidden; ++i) ss = fmaf(xr[i], xr[i], ss);
        const float scale = 1.0f / sqrtf(ss / (float)hidden + eps);
        for (int i = 0; i < hidden; ++i) out[(size_t)r * hidden + i] = xr[i] * scale * w[i];
    }
}

/* silu_gate_multiply (activations.cl:219-265), scalar tail: gf * (1 / (1 + exp(-gf))) * uf. */
void ora_silu_gate_n(const float* gate, const float* up, float* out, size_t n) {
    for (size_t i = 0; i < n; ++i) {
        float g = gate[i];
        float sig = 1.0f / (1.0f + expf(-g));
        out[i] = g * sig * up[i];
    }
}

/* patch_embed (vision.cl:118-197): patch p = (row, col) of a (H/ph) x (W/pw) grid; its
 * feature index runs over c, then py, then px (the loop nest at :154-176). */
void ora_im2col(const float* img, float* patches, int C, int H, int W, int ph, int pw) {
    int gw = W / pw, gh = H / ph, pd = C * ph * pw;
    for (int p = 0; p < gh * gw; ++p) {
        int pr = p / gw, pc = p % gw, idx = 0;
        for (int c = 0; c < C; ++c)
            for (int py = 0; py < ph; ++py)
                for (int px = 0; px < pw; ++px)
                    patches[(size_t)p * pd + idx++] =
                        img[(size_t)c * H * W + (size_t)(pr * ph + py) * W + (pc * pw + px)];
    }
}

/* ------------------------------------------------------------------------------------ */
/* Multithreaded variants (timed CPU baseline).  Same per-output arithmetic.             */
/* ------------------------------------------------------------------------------------ */
/* Use n host threads in the multithreaded variants (a launcher may have set OMP_NUM_THREADS=1). */
void ora_set_threads(int n) {
#ifdef _OPENMP
    if (n > 0) omp_set_num_threads(n);
#else
    (void)n;
#endif
}

int ora_max_threads(void) {
#ifdef _OPENMP
    return omp_get_max_threads();
#else
    return 1;
#endif
}

void ora_gemv_q_mt(const float* x, const uint8_t* W, float* y, int N, int K, int type) {
    size_t rb = ora_row_bytes(type, K);
#pragma omp parallel
    {
        float row[65536];
#pragma omp for schedule(static)
        for (int n = 0; n < N; ++n) {
            ora_dequant(W + (size_t)n * rb, row, K, type);
            float acc = 0.0f;
            for (int k = 0; k < K; ++k) acc = fmaf(x[k], row[k], acc);
            y[n] = acc;
        }
    }
}

void ora_gemm_q_mt(const float* A, const uint8_t* W, float* C, int M, int N, int K, int type) {
    size_t rb = ora_row_bytes(type, K);
#pragma omp parallel
    {
        float row[65536];
#pragma omp for schedule(static)
        for (int n = 0; n < N; ++n) {
            ora_dequant(W + (size_t)n * rb, row, K, type);
            for (int m = 0; m < M; ++m) {
                float acc = 0.0f;
                for (int k = 0; k < K; ++k) acc = fmaf(A[(size_t)m * K + k], row[k], acc);
                C[(size_t)m * N + n] = acc;
            }
        }
    }
}

void ora_gemv_f32_kn_mt(const float* x, const float* W, float* y, int N, int K) {
#pragma omp parallel for schedule(static)
    for (int n = 0; n < N; ++n) y[n] = gemv_column_f32(x, W, n, N, K);
}

void ora_gemm_naive_f32_mt(const float* A, const float* B, float* C, int M, int N, int K) {
#pragma omp parallel for schedule(static)
    for (int m = 0; m < M; ++m)
        for (int n = 0; n < N; ++n) {
            float acc = 0.0f;
            for (int k = 0; k < K; ++k) acc = fmaf(A[(size_t)m * K + k], B[(size_t)k * N + n], acc);
            C[(size_t)m * N + n] = acc;
        }
}

void ora_gemm_nk_mt(const float* A, const void* W, int wtype, float* C, int M, int N, int K) {
#pragma omp parallel for schedule(static)
    for (int n = 0; n < N; ++n)
        for (int m = 0; m < M; ++m) {
            float acc = 0.0f;
            for (int k = 0; k < K; ++k)
                acc = fmaf(A[(size_t)m * K + k], load_dense(W, wtype, (size_t)n * K + k), acc);
            C[(size_t)m * N + n] = acc;
        }
}
