// skinny.cu - skinny GEMM for batched decode (replaces dispatch_gemm_image / gemm_image,
// src/kernels/gemm.cl:157-200, when M is a handful of sequences and W is GGUF Q4_0).
//
// C[S][N] = A[S][K] . dequant(W[N][K])^T for S <= 32 concurrent sequences, A bf16 or fp16.
// The shape is the decode GEMV's with a few activation rows, so the kernel is built like it:
// each CTA owns an even share of W's rows and streams them once from HBM, while the weight
// decode happens in registers straight into tensor-core fragments.
//   * A producer thread stages, per 256-k slice, the CTA's packed rows (a 2-D TMA box over the
//     rows' 16-bit units: 144 bytes = 8 blocks per row) and the activation rows of that slice
//     (two 2-D TMA boxes of 136 x S elements: each row lands at a 272-byte pitch, which puts a
//     fragment's 8 rows on distinct banks; rows past S and columns past K read as zeros).
//     Three TMA instructions per stage: one small bulk copy per activation row was measured to
//     cost ~50 ns of issue each, which serialised the ring.  Weights are never written by the
//     preceding kernel, so the first slices stream before griddepcontrol.wait; activations
//     after it.
//   * A stage holds 1, 2 or 4 such 256-k sub-slices, so that each warp has several independent
//     blocks to decode per stage (one block per stage left a warp with a single serial chain).
//   * Eight consumer warps: warp w takes 16-row group (w % RG) and a contiguous run of the
//     stage's blocks (the 8/RG warps of a row group split K).  Every warp consumes every
//     stage, in order, so a warp's parity wait on a slot is never more than one phase ahead.  A lane turns its two quant
//     bytes per row and block into bf16 / fp16 pairs: nibble | 0x4300 (bf16 128 + q) or
//     | 0x6400 (fp16 1024 + q), minus 136 / 1032 gives q - 8 exactly, times the block's d.
//     Those are the A fragments of mma.sync.m16n8k16 (weights as M = 16 rows), the staged
//     activations the B fragments (sequences as N = 8 per tile), fp32 accumulation over all K.
//   * After the last slice of a row chunk the warps' partial sums meet in shared memory and
//     the CTA writes C (+ bias) for its rows.
// (Larger batches are tensor-bound enough for the tcgen05 GEMM, which takes them.)
#include <cuda.h>

#include "common.cuh"
#include "kernels.h"

using namespace mgpu_dev;

namespace {

constexpr int kSkThreads = 288;        // 8 consumer warps + 1 producer warp
constexpr int kSkSlice = 256;          // k per stage: 8 GGUF blocks
constexpr int kSkWRowBytes = 144;      // 8 Q4_0 blocks
constexpr int kSkXBox = 136;           // activation elements per TMA box (128 used + 8 pad)
constexpr int kSkXPitch = kSkXBox * 2;  // 272 bytes per activation row in shared memory
constexpr int kSkMaxStages = 6;
constexpr uint32_t kSkSmemBudget = 100 * 1024;  // two CTAs (this and the next launch) per SM

struct SkinnyArgs {
    const void* A;  // [S][lda] activations
    int64_t lda;
    void* C;        // [S][ldc]
    int64_t ldc;
    int c_type;
    const void* bias;
    int bias_type;
    mgpu_k::Epilogue epi;  // activation / residual after the bias
    int S, N, K;
    int stages;
    uint32_t sub_bytes;    // one sub-slice: TR x 144 weight bytes, then 2 x 8 NT x 272 activation bytes
    uint32_t stage_bytes;  // subs x sub_bytes, rounded up to 1 KB
    uint32_t x_offset;     // offset of the activation rows inside a sub-slice
    int* status;
};

template <typename T> struct Magic;
template <> struct Magic<__nv_bfloat16> {
    static constexpr uint32_t kOr = 0x43004300u;  // bf16 128.0 in each half
    static constexpr float kSub = 136.0f;
};
template <> struct Magic<__half> {
    static constexpr uint32_t kOr = 0x64006400u;  // fp16 1024.0 in each half
    static constexpr float kSub = 1032.0f;
};

template <typename T>
__device__ __forceinline__ uint32_t sub_mul2(uint32_t v, uint32_t sub2, uint32_t d2) {
    uint32_t r;
    if constexpr (std::is_same<T, __nv_bfloat16>::value) {
        asm("{\n .reg .b32 t;\n sub.rn.bf16x2 t, %1, %2;\n mul.rn.bf16x2 %0, t, %3;\n}\n"
            : "=r"(r)
            : "r"(v), "r"(sub2), "r"(d2));
    } else {
        asm("{\n .reg .b32 t;\n sub.rn.f16x2 t, %1, %2;\n mul.rn.f16x2 %0, t, %3;\n}\n"
            : "=r"(r)
            : "r"(v), "r"(sub2), "r"(d2));
    }
    return r;
}

template <typename T>
__device__ __forceinline__ void mma16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    if constexpr (std::is_same<T, __nv_bfloat16>::value)
        asm volatile(
            "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
            "{%0,%1,%2,%3};"
            : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
            : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
    else
        asm volatile(
            "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
            "{%0,%1,%2,%3};"
            : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
            : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

template <typename T>
__device__ __forceinline__ uint32_t pack_pair(float v);
template <>
__device__ __forceinline__ uint32_t pack_pair<__nv_bfloat16>(float v) {
    __nv_bfloat162 h = __floats2bfloat162_rn(v, v);
    return *reinterpret_cast<uint32_t*>(&h);
}
template <>
__device__ __forceinline__ uint32_t pack_pair<__half>(float v) {
    __half2 h = __floats2half2_rn(v, v);
    return *reinterpret_cast<uint32_t*>(&h);
}

__device__ __forceinline__ float bias_value(const void* bias, int type, int n) {
    if (type == MGPU_F32) return reinterpret_cast<const float*>(bias)[n];
    if (type == MGPU_F16) return __half2float(reinterpret_cast<const __half*>(bias)[n]);
    return __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(bias)[n]);
}
__device__ __forceinline__ void store_value(void* C, int type, size_t idx, float v) {
    if (type == MGPU_F32) reinterpret_cast<float*>(C)[idx] = v;
    else if (type == MGPU_F16) reinterpret_cast<__half*>(C)[idx] = __float2half_rn(v);
    else reinterpret_cast<__nv_bfloat16*>(C)[idx] = __float2bfloat16_rn(v);
}

// NT = 8-sequence tiles per CTA (S per CTA <= 8 NT); RG = 16-row groups per chunk; SUBS =
// 256-k sub-slices per stage.
template <int NT, int RG, int SUBS, typename T>
__global__ void __launch_bounds__(kSkThreads, 1)
    gemm_q4_skinny(const __grid_constant__ CUtensorMap tmW, const __grid_constant__ CUtensorMap tmX, SkinnyArgs a) {
    constexpr int TR = 16 * RG;         // rows per chunk
    constexpr int WPG = 8 / RG;         // warps per row group (split K)
    constexpr int BPW = RG * SUBS;      // blocks of a stage per warp
    constexpr int SP = 8 * NT;          // sequences per CTA
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
    __shared__ __align__(8) uint64_t full_bar[kSkMaxStages];
    __shared__ __align__(8) uint64_t empty_bar[kSkMaxStages];
    // end of a row chunk: partials written (red_bar), partials consumed (done_bar); mbarriers
    // rather than bar.sync so that every wait is bounded
    __shared__ __align__(8) uint64_t red_bar;
    __shared__ __align__(8) uint64_t done_bar;

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int G = gridDim.x;
    const int r0 = (int)((long long)a.N * blockIdx.x / G);
    const int r1 = (int)((long long)a.N * (blockIdx.x + 1) / G);
    const int seq0 = blockIdx.y * SP;
    const int ns = min(SP, a.S - seq0);  // sequences of this CTA
    const int nchunks = (r1 - r0 + TR - 1) / TR;
    const int nslices = a.K / (kSkSlice * SUBS);  // stages per chunk
    const int total = nchunks * nslices;
    float* red = reinterpret_cast<float*>(smem + (size_t)a.stages * a.stage_bytes);  // [WPG][TR][SP]

    if (tid == 0) {
        for (int s = 0; s < a.stages; ++s) {
            mbar_init(&full_bar[s], 1);
            mbar_init(&empty_bar[s], 8);
        }
        mbar_init(&red_bar, 8);
        mbar_init(&done_bar, 8);
        fence_mbar_init();
        asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    }
    __syncthreads();

    if (warp == 8) {
        // ---- producer (one thread) ----
        if (lane == 0) {
            prefetch_tensormap(&tmW);
            prefetch_tensormap(&tmX);
            const uint32_t bytes = (uint32_t)SUBS * a.sub_bytes;
            auto w_load = [&](int it, int s) {
                const int c = it / nslices, ks = it % nslices;
                for (int u = 0; u < SUBS; ++u)
                    tma_load_2d(smem + (size_t)s * a.stage_bytes + (size_t)u * a.sub_bytes, &tmW,
                                (ks * SUBS + u) * (kSkWRowBytes / 2), r0 + c * TR, &full_bar[s]);
            };
            auto x_load = [&](int it, int s) {
                const int ks = it % nslices;
                for (int u = 0; u < SUBS; ++u) {
                    uint8_t* xdst = smem + (size_t)s * a.stage_bytes + (size_t)u * a.sub_bytes + a.x_offset;
                    const int k0 = (ks * SUBS + u) * kSkSlice;
                    tma_load_2d(xdst, &tmX, k0, seq0, &full_bar[s]);
                    tma_load_2d(xdst + SP * kSkXPitch, &tmX, k0 + 128, seq0, &full_bar[s]);
                }
            };
            // weights of the first stages before the dependency wait, activations after it
            const int pre = min(a.stages, total);
            for (int it = 0; it < pre; ++it) {
                mbar_arrive_expect_tx(&full_bar[it], bytes);
                w_load(it, it);
            }
            asm volatile("griddepcontrol.wait;" ::: "memory");
            for (int it = 0; it < pre; ++it) x_load(it, it);
            int s = pre % a.stages;
            uint32_t ph = (uint32_t)(pre / a.stages) & 1u;
            for (int it = pre; it < total; ++it) {
                if (!mbar_wait(&empty_bar[s], ph ^ 1u, a.status)) {
                    // Timed out: let the copies already issued land before the CTA exits.
                    for (int k = max(0, it - a.stages); k < it; ++k)
                        mbar_wait(&full_bar[k % a.stages], (uint32_t)(k / a.stages) & 1u, nullptr);
                    break;
                }
                mbar_arrive_expect_tx(&full_bar[s], bytes);
                w_load(it, s);
                x_load(it, s);
                if (++s == a.stages) {
                    s = 0;
                    ph ^= 1u;
                }
            }
        }
        return;
    }

    // ---- consumers ----
    const int g = lane >> 2, t = lane & 3;
    const int rg = warp % RG, kw = warp / RG;
    const uint32_t sub2 = pack_pair<T>(Magic<T>::kSub);
    int s = 0;
    uint32_t ph = 0;
    for (int c = 0; c < nchunks; ++c) {
        float acc[NT][4];
#pragma unroll
        for (int j = 0; j < NT; ++j) acc[j][0] = acc[j][1] = acc[j][2] = acc[j][3] = 0.0f;
        for (int ks = 0; ks < nslices; ++ks) {
            if (!mbar_wait(&full_bar[s], ph, a.status)) return;
            const uint8_t* stg = smem + (size_t)s * a.stage_bytes;
#pragma unroll
            for (int bi = 0; bi < BPW; ++bi) {
                const int bb = kw * BPW + bi;  // block within the stage
                const uint8_t* wst = stg + (size_t)(bb >> 3) * a.sub_bytes;  // its sub-slice
                const uint8_t* xst = wst + a.x_offset;
                const int b = bb & 7;                                         // block within the sub-slice
                const uint8_t* rowg = wst + (size_t)(rg * 16 + g) * kSkWRowBytes;
                const uint8_t* rowg8 = rowg + 8 * kSkWRowBytes;
                // quant bytes 2t, 2t+1 (elements 2t, 2t+1 and 16+2t, 17+2t) and 8+2t, 9+2t
                const uint8_t* qg = rowg + b * 18 + 2;
                const uint8_t* qg8 = rowg8 + b * 18 + 2;
                const uint32_t wg = (uint32_t)*reinterpret_cast<const uint16_t*>(qg + 2 * t) |
                                    ((uint32_t)*reinterpret_cast<const uint16_t*>(qg + 8 + 2 * t) << 16);
                const uint32_t wg8 = (uint32_t)*reinterpret_cast<const uint16_t*>(qg8 + 2 * t) |
                                     ((uint32_t)*reinterpret_cast<const uint16_t*>(qg8 + 8 + 2 * t) << 16);
                const uint32_t dg2 = pack_pair<T>(__half2float(*reinterpret_cast<const __half*>(rowg + b * 18)));
                const uint32_t dg82 = pack_pair<T>(__half2float(*reinterpret_cast<const __half*>(rowg8 + b * 18)));
                // bytes [q(2t), q(2t+1), q(8+2t), q(9+2t)]: low nibbles are elements of the first
                // k16 step, high nibbles of the second
                const uint32_t lo = wg & 0x0F0F0F0Fu, hi = (wg >> 4) & 0x0F0F0F0Fu;
                const uint32_t lo8 = wg8 & 0x0F0F0F0Fu, hi8 = (wg8 >> 4) & 0x0F0F0F0Fu;
                uint32_t a1[4], a2[4];
                a1[0] = sub_mul2<T>(prmt(lo, 0u, 0x4140u) | Magic<T>::kOr, sub2, dg2);    // row g, k 2t..
                a1[1] = sub_mul2<T>(prmt(lo8, 0u, 0x4140u) | Magic<T>::kOr, sub2, dg82);  // row g+8
                a1[2] = sub_mul2<T>(prmt(lo, 0u, 0x4342u) | Magic<T>::kOr, sub2, dg2);    // row g, k 8+2t..
                a1[3] = sub_mul2<T>(prmt(lo8, 0u, 0x4342u) | Magic<T>::kOr, sub2, dg82);
                a2[0] = sub_mul2<T>(prmt(hi, 0u, 0x4140u) | Magic<T>::kOr, sub2, dg2);
                a2[1] = sub_mul2<T>(prmt(hi8, 0u, 0x4140u) | Magic<T>::kOr, sub2, dg82);
                a2[2] = sub_mul2<T>(prmt(hi, 0u, 0x4342u) | Magic<T>::kOr, sub2, dg2);
                a2[3] = sub_mul2<T>(prmt(hi8, 0u, 0x4342u) | Magic<T>::kOr, sub2, dg82);
#pragma unroll
                for (int j = 0; j < NT; ++j) {
                    // block b's 32 activations: box b / 4, elements 32 (b % 4) .. + 31
                    const uint8_t* xr = xst + (size_t)(b >> 2) * (SP * kSkXPitch) + (size_t)(8 * j + g) * kSkXPitch +
                                        (size_t)(b & 3) * 64 + 4 * t;
                    const uint32_t b0 = *reinterpret_cast<const uint32_t*>(xr);
                    const uint32_t b1 = *reinterpret_cast<const uint32_t*>(xr + 16);
                    const uint32_t b2 = *reinterpret_cast<const uint32_t*>(xr + 32);
                    const uint32_t b3 = *reinterpret_cast<const uint32_t*>(xr + 48);
                    mma16816<T>(acc[j], a1, b0, b1);
                    mma16816<T>(acc[j], a2, b2, b3);
                }
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty_bar[s]);
            if (++s == a.stages) {
                s = 0;
                ph ^= 1u;
            }
        }
        // partial sums of this warp: rows g, g+8 of its group, sequences 8j + 2t, 8j + 2t + 1
#pragma unroll
        for (int j = 0; j < NT; ++j) {
            float* rp = red + ((size_t)kw * TR + rg * 16 + g) * SP + 8 * j + 2 * t;
            rp[0] = acc[j][0];
            rp[1] = acc[j][1];
            rp[8 * SP] = acc[j][2];
            rp[8 * SP + 1] = acc[j][3];
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&red_bar);
        if (!mbar_wait(&red_bar, (uint32_t)c & 1u, a.status)) return;
        const int row0 = r0 + c * TR;
        const int nrows = min(TR, r1 - row0);
        const bool fused = epilogue_active(a.epi);
        for (int i = tid; i < nrows * ns; i += 256) {
            const int sq = i / nrows, r = i % nrows;  // consecutive threads: consecutive rows
            float v = 0.0f;
#pragma unroll
            for (int w = 0; w < WPG; ++w) v += red[((size_t)w * TR + r) * SP + sq];
            if (a.bias) v += bias_value(a.bias, a.bias_type, row0 + r);
            if (fused) v = epilogue_finish(a.epi, seq0 + sq, row0 + r, v);
            store_value(a.C, a.c_type, (size_t)(seq0 + sq) * a.ldc + row0 + r, v);
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&done_bar);
        if (!mbar_wait(&done_bar, (uint32_t)c & 1u, a.status)) return;
    }
}

template <int NT, int RG, int SUBS, typename T>
cudaError_t launch_skinny(const mgpu_k::LaunchCtx& c, const CUtensorMap& tm, const CUtensorMap& tx,
                          const SkinnyArgs& a, dim3 grid, size_t smem) {
    auto kern = gemm_q4_skinny<NT, RG, SUBS, T>;
    static thread_local uint64_t configured = 0;  // one bit per device ordinal
    int ordinal = 0;
    cudaGetDevice(&ordinal);
    if (!(configured & (1ull << (ordinal & 63)))) {
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kSkSmemBudget);
        if (e != cudaSuccess) return e;
        e = cudaFuncSetAttribute(kern, cudaFuncAttributePreferredSharedMemoryCarveout,
                                 (int)cudaSharedmemCarveoutMaxShared);
        if (e != cudaSuccess) return e;
        configured |= 1ull << (ordinal & 63);
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = dim3(kSkThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = c.stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kern, tm, tx, a);
}

template <int NT, typename T>
cudaError_t dispatch_rg(const mgpu_k::LaunchCtx& c, int rg, int subs, const CUtensorMap& tm, const CUtensorMap& tx,
                        const SkinnyArgs& a, dim3 grid, size_t smem) {
    // (row groups, sub-slices): at most 4 blocks per warp per stage
    if (rg == 4) return launch_skinny<NT, 4, 1, T>(c, tm, tx, a, grid, smem);
    if (rg == 2) return subs == 2 ? launch_skinny<NT, 2, 2, T>(c, tm, tx, a, grid, smem)
                                  : launch_skinny<NT, 2, 1, T>(c, tm, tx, a, grid, smem);
    return subs == 4 ? launch_skinny<NT, 1, 4, T>(c, tm, tx, a, grid, smem)
         : subs == 2 ? launch_skinny<NT, 1, 2, T>(c, tm, tx, a, grid, smem)
                     : launch_skinny<NT, 1, 1, T>(c, tm, tx, a, grid, smem);
}

}  // namespace

namespace mgpu_k {

bool skinny_ok(const GemmOperand& A, const GemmOperand& B, int M, int N, int K) {
    return B.type == MGPU_Q4_0 && B.layout == MGPU_LAYOUT_NK && (A.type == MGPU_BF16 || A.type == MGPU_F16) &&
           M >= 1 && M <= 32 && N >= 1 && K % kSkSlice == 0 && B.ld == (int64_t)(K / 32) * 18 &&
           (reinterpret_cast<uintptr_t>(B.ptr) & 15) == 0 && (reinterpret_cast<uintptr_t>(A.ptr) & 15) == 0 &&
           (A.ld * 2) % 16 == 0;
}

cudaError_t gemm_q4_skinny(const LaunchCtx& c, const GemmOperand& A, const GemmOperand& B, const GemmOperand& C,
                           const void* bias, int bias_type, int M, int N, int K, const Epilogue& epi) {
    if (!skinny_ok(A, B, M, N, K)) return cudaErrorInvalidValue;
    const int NT = M <= 8 ? 1 : M <= 16 ? 2 : 4;
    const int SP = 8 * NT;
    // CTAs over the rows: one per SM, fewer when a CTA would get fewer than 16 rows
    const int G = max(1, min(c.sm_count, (N + 15) / 16));
    const int rows_per_cta = (N + G - 1) / G;
    // chunk: all of the CTA's rows when they fit in 64 (so each activation slice is staged once
    // per CTA), else 64-row chunks
    int RG = 1;
    while (RG < 4 && 16 * RG < rows_per_cta) RG <<= 1;
    const int TR = 16 * RG;
    const uint32_t x_offset = (uint32_t)((TR * kSkWRowBytes + 127) / 128 * 128);
    const uint32_t sub_bytes = x_offset + 2 * SP * kSkXPitch;  // a multiple of 128
    const size_t red_bytes = (size_t)(8 / RG) * TR * SP * sizeof(float);
    // sub-slices per stage: up to 4 blocks per warp, dividing K / 256, with at least 2 stages
    int subs = 4 / RG;
    auto stage_of = [&](int u) { return ((size_t)u * sub_bytes + 1023) / 1024 * 1024; };
    while (subs > 1 && ((K / kSkSlice) % subs != 0 || 2 * stage_of(subs) + red_bytes + 1024 > kSkSmemBudget))
        subs >>= 1;
    const uint32_t stage_bytes = (uint32_t)stage_of(subs);
    const int stages = (int)std::min<size_t>(kSkMaxStages, (kSkSmemBudget - 1024 - red_bytes) / stage_bytes);
    if (stages < 2) return cudaErrorInvalidValue;
    const size_t smem = 1024 + (size_t)stages * stage_bytes + red_bytes;

    CUtensorMap tm;
    // W as a 2-D array of 16-bit units: rows N, row pitch K/32 * 18 bytes; box = one 256-k slice
    // (72 units) x TR rows
    if (!make_tensor_map_u16(&tm, B.ptr, N, B.ld / 2, B.ld / 2, kSkWRowBytes / 2, TR)) return cudaErrorInvalidValue;
    // A as a 2-D array of 16-bit elements: M rows, K columns, pitch lda; box 136 x 8 NT
    CUtensorMap tx;
    if (!make_tensor_map_u16(&tx, A.ptr, M, K, A.ld, kSkXBox, SP)) return cudaErrorInvalidValue;
    SkinnyArgs a;
    a.A = A.ptr;
    a.lda = A.ld;
    a.C = const_cast<void*>(C.ptr);
    a.ldc = C.ld;
    a.c_type = C.type;
    a.bias = bias;
    a.bias_type = bias_type;
    a.epi = epi;
    a.S = M;
    a.N = N;
    a.K = K;
    a.stages = stages;
    a.sub_bytes = sub_bytes;
    a.stage_bytes = stage_bytes;
    a.x_offset = x_offset;
    a.status = c.status;
    const dim3 grid(G, (M + SP - 1) / SP);
    const bool bf16 = A.type == MGPU_BF16;
    switch (NT) {
        case 1: return bf16 ? dispatch_rg<1, __nv_bfloat16>(c, RG, subs, tm, tx, a, grid, smem) : dispatch_rg<1, __half>(c, RG, subs, tm, tx, a, grid, smem);
        case 2: return bf16 ? dispatch_rg<2, __nv_bfloat16>(c, RG, subs, tm, tx, a, grid, smem) : dispatch_rg<2, __half>(c, RG, subs, tm, tx, a, grid, smem);
        default: return bf16 ? dispatch_rg<4, __nv_bfloat16>(c, RG, subs, tm, tx, a, grid, smem) : dispatch_rg<4, __half>(c, RG, subs, tm, tx, a, grid, smem);
    }
}

}  // namespace mgpu_k
