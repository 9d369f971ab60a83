/*
 * oracle.h - CPU restatement of MVLM's matmul hot path.  TEST INFRASTRUCTURE ONLY.
 *
 * This library is the parity checker for the CUDA path in mvlm_b200/.  Only tests/,
 * __graft_entry__.smoke() and bench.py's CPU-baseline leg may load it.  The product path
 * never calls it and has no CPU fallback.
 *
 * Every function names the reference file:line whose arithmetic it restates (paths are
 * relative to the drxddy/MVLM project root).  Where the reference has no code (GGUF
 * Q4_0/Q8_0 dequantisation and quantisation), the function restates the published ggml
 * block format and is pinned against the gguf-py 0.19.0 package (tests/golden/).
 */
#ifndef MVLM_ORACLE_H
#define MVLM_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ggml type tags, values as in src/models/gguf_loader.h:12-30 (BF16 = 30 as in ggml). */
enum { ORA_F32 = 0, ORA_F16 = 1, ORA_Q4_0 = 2, ORA_Q8_0 = 8, ORA_BF16 = 30 };

/* --- scalar conversions (IEEE 754 binary16 / bfloat16, round to nearest even) --- */
float ora_f16_to_f32(uint16_t h);
uint16_t ora_f32_to_f16(float f);
float ora_bf16_to_f32(uint16_t h);
uint16_t ora_f32_to_bf16(float f);
void ora_f32_to_f16_n(const float* x, uint16_t* y, size_t n);
void ora_f16_to_f32_n(const uint16_t* x, float* y, size_t n);
void ora_f32_to_bf16_n(const float* x, uint16_t* y, size_t n);
void ora_bf16_to_f32_n(const uint16_t* x, float* y, size_t n);

/* --- ggml type table: src/models/gguf_loader.cpp:13-55 --- */
size_t ora_type_size(int type);
int ora_block_size(int type);
size_t ora_row_bytes(int type, int64_t k);

/* --- seeded generators: SplitMix64 ---
 * U(-1,1) = (u >> 40) * 2^-23 - 1 ; N(0, sigma) by Box-Muller on two uniforms in (0,1]. */
uint64_t ora_splitmix64(uint64_t* state);
void ora_fill_uniform(float* out, size_t n, uint64_t seed);
void ora_fill_normal(float* out, size_t n, uint64_t seed, float sigma);

/* --- GGUF block quantisation (ggml reference quantiser, restated) --- */
void ora_quantize_q4_0(const float* x, uint8_t* blocks, int64_t n);
void ora_quantize_q8_0(const float* x, uint8_t* blocks, int64_t n);
/* --- GGUF block dequantisation: w = (q-8)*d (Q4_0), w = q*d (Q8_0), exact in fp32 --- */
void ora_dequant(const uint8_t* blocks, float* out, int64_t n, int type);

/* --- GEMM / GEMV restatements of src/kernels/gemm.cl --- */
/* gemm_naive gemm.cl:26-51 (also gemm_tiled :74-136 and gemm_image :157-200, which
 * perform the identical fp32 fma sequence over k): C = A[M,K] * B[K,N], fp16 io. */
void ora_gemm_naive_f16(const uint16_t* A, const uint16_t* B, uint16_t* C, int M, int N, int K);
/* same loop, fp32 everywhere (the fp32 config path). */
void ora_gemm_naive_f32(const float* A, const float* B, float* C, int M, int N, int K);
/* gemv gemm.cl:219-270: 256 strided partial sums + local tree reduction, fp16 io. */
void ora_gemv_f16(const uint16_t* x, const uint16_t* W, uint16_t* y, int N, int K);
/* same reduction order in fp32 (x, W[K,N], y all fp32). */
void ora_gemv_f32(const float* x, const float* W, float* y, int N, int K);
/* quantised path: GGUF dequant of W[N][K/32 blocks] then the gemm_naive fp32 loop:
 * C[m,n] = sum_k A[m,k] * w[n,k], accumulated with fmaf in increasing k. */
void ora_gemm_q(const float* A, const uint8_t* W, float* C, int M, int N, int K, int type);
/* dense weights stored [N][K] (GGUF-native f32/f16/bf16 tensors), same fp32 loop. */
void ora_gemm_nk(const float* A, const void* W, int wtype, float* C, int M, int N, int K);
/* bias epilogue of patch_embed / vision_proj (vision.cl:180-186, :430-434): C[m,n] += bias[n]. */
void ora_add_bias(float* C, const float* bias, int M, int N);
/* activations.cl elementwise kernels on one fp32 value (act: 1 gelu with tanh, 2 silu,
 * 3 gelu as activations.cl:78-117 computes it); the _n form works in place. */
float ora_activate(float x, int act);
void ora_activate_n(float* x, size_t n, int act);
/* silu_gate_multiply (activations.cl:219-265) on fp32 values: out = silu(gate) * up. */
void ora_silu_gate_n(const float* gate, const float* up, float* out, size_t n);
/* patch_embed im2col order (vision.cl:154-176): patches[p][c*ph*pw + py*pw + px]. */
void ora_im2col(const float* img, float* patches, int C, int H, int W, int ph, int pw);

/* --- multithreaded variants for the timed CPU baseline (OpenMP over output columns) --- */
void ora_gemv_q_mt(const float* x, const uint8_t* W, float* y, int N, int K, int type);
void ora_gemm_q_mt(const float* A, const uint8_t* W, float* C, int M, int N, int K, int type);
void ora_gemv_f32_kn_mt(const float* x, const float* W, float* y, int N, int K);
void ora_gemm_naive_f32_mt(const float* A, const float* B, float* C, int M, int N, int K);
void ora_gemm_nk_mt(const float* A, const void* W, int wtype, float* C, int M, int N, int K);
int ora_max_threads(void);
void ora_set_threads(int n);

#ifdef __cplusplus
}
#endif
void ora_rms_norm(const float* x, const float* w, float* out, int rows, int hidden, float eps);
#endif
