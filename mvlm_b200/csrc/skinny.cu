// skinny.cu - skinny GEMM for batched decode (replaces dispatch_gemm_image / gemm_image,
// src/kernels/gemm.cl:157-200, when M is a handful of sequences and W is GGUF Q4_0).
//
// C[S][N] = A[S][K] . dequant(W[N][K])^T for S <= 32 concurrent sequences, A bf16 or fp16.
// The shape is the decode GEMV's with a few activation rows, so the kernel is built like it:
// each CTA owns an even share of W's rows and streams them once from HBM, while the weight
// decode happens in registers straight into tensor-core fragments.
//   * A producer thread stages the CTA's rows in 256-k slices (8 blocks = 144 bytes per row),
//     a stage holding 1..8 consecutive slices, with two TMA instructions per stage: one 3-D
//     box of the packed rows, viewed as [slice][row][72 16-bit units], so that each slice's
//     rows land at a 144-byte pitch (a fragment's 8 rows on distinct banks), and one 3-D box
//     of the activations, viewed as [128-element chunk][sequence][element] with 136-element
//     boxes, so that each sequence's chunk lands at a 272-byte pitch (rows past S, rows past N
//     and the 8 elements past a chunk read as zeros).  TMA issue costs ~50-75 ns per
//     instruction from the one producer thread; with one box per slice and operand it was the
//     bound of the K = 8192 shapes.  Weights are never written by the preceding kernel, so the
//     first stages' weights stream before griddepcontrol.wait; activations after it.
//   * A stage holds as many slices as give each warp up to 8 (row group, block) units (4 with
//     16 sequences), so that it has several independent chains per stage.
//   * Eight consumer warps split K: warp w takes block w of every 256-k sub-slice, for all the
//     chunk's 16-row groups, so the activation fragments it loads for a block serve every row
//     group.  The MMA is mma.sync.m16n8k16 with the weights as M (16 rows) and the sequences
//     as N (8 per tile), fp32 accumulation.  Its 16 k positions are taken in a permuted order
//     (k 2t, 2t+1 <-> block elements 4t, 4t+2; k 2t+8, 2t+9 <-> 4t+1, 4t+3; the second k16 step
//     the same + 16): the sum over k does not depend on the order, and in this one lane t's A
//     fragments are the nibbles of quant word t (bytes 4t..4t+3, which hold elements 4t..4t+3
//     low and 16+4t..19+4t high) in place, one mask-and-or per register:
//     nibble | 0x4300 (bf16 128 + q) or | 0x6400 (fp16 1024 + q), minus 136 / 1032 = q - 8
//     exactly.  The B fragments are the matching pairs of staged activations (one byte permute
//     per register).  A block's two MMAs start from zero, so their result is the exact
//     sum of (q - 8) x over the block, which is scaled by the block's fp16 d in fp32.
//   * After the last slice of a row chunk the warps' partial sums meet in shared memory, are
//     added in warp order (deterministic), and the CTA writes C (+ bias, epilogue) for its rows.
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
    uint32_t stage_bytes;  // weights [SUBS][TR][144 B], then activations [2 SUBS][8 NT][272 B], 1 KB aligned
    uint32_t x_offset;     // offset of the activations inside a stage (128-byte aligned)
    uint32_t tx_bytes;     // bytes the two copies of a stage deliver
    int shape;             // which (row groups, sub-slices) body runs (SkinnyShape)
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

// (q - 8) of the two 4-bit fields at bit SH of each 16-bit half of w, as a T pair (exact).
template <typename T, int SH>
__device__ __forceinline__ uint32_t nib_pair(uint32_t w, uint32_t sub2) {
    const uint32_t v = ((w >> SH) & 0x000F000Fu) | Magic<T>::kOr;
    uint32_t r;
    if constexpr (std::is_same<T, __nv_bfloat16>::value)
        asm("sub.rn.bf16x2 %0, %1, %2;" : "=r"(r) : "r"(v), "r"(sub2));
    else
        asm("sub.rn.f16x2 %0, %1, %2;" : "=r"(r) : "r"(v), "r"(sub2));
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

// The kernel's body for NT = 8-sequence tiles per CTA (S per CTA <= 8 NT), RG = 16-row groups
// per chunk, SUBS = 256-k sub-slices per stage.
template <int NT, int RG, int SUBS, typename T>
__device__ __forceinline__ void skinny_body(const CUtensorMap& tmW, const CUtensorMap& tmX, const SkinnyArgs& a) {
    constexpr int TR = 16 * RG;         // rows per chunk
    constexpr int SP = 8 * NT;          // sequences per CTA
    constexpr int RP = TR + 4;          // partial-sum row pitch: a warp's 32 writes on distinct banks
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
    float* red = reinterpret_cast<float*>(smem + (size_t)a.stages * a.stage_bytes);  // [8 warps][SP][RP]

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
            const uint32_t bytes = a.tx_bytes;
            // one copy per stage for each operand: W's box is [SUBS slices][TR rows][72 units],
            // the activations' [2 SUBS chunks of 128][8 NT sequences][136 elements]
            auto w_load = [&](int it, int s) {
                const int c = it / nslices, ks = it % nslices;
                tma_load_3d(smem + (size_t)s * a.stage_bytes, &tmW, 0, r0 + c * TR, ks * SUBS, &full_bar[s]);
            };
            auto x_load = [&](int it, int s) {
                const int ks = it % nslices;
                tma_load_3d(smem + (size_t)s * a.stage_bytes + a.x_offset, &tmX, 0, seq0, 2 * ks * SUBS, &full_bar[s]);
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

    // ---- consumers: warp w takes block w of every sub-slice, for every row group ----
    const int g = lane >> 2, t = lane & 3;
    const int bw = warp;                  // block within a sub-slice (0..7)
    const bool even_block = (bw & 1) == 0;  // quants at 2 mod 4: realign with a byte permute
    const uint32_t sub2 = pack_pair<T>(Magic<T>::kSub);
    // this lane's activation words inside a sub-slice: chunk bw / 4, sequence 8j + g, elements
    // 32 (bw % 4) + 4t .. + 3 (and + 16)
    const uint32_t x_lane = a.x_offset + (uint32_t)(bw >> 2) * (SP * kSkXPitch) + (uint32_t)g * kSkXPitch +
                            (uint32_t)(bw & 3) * 64 + 8u * t;
    // this lane's weight bytes inside a sub-slice: row g of a group, block bw (even: the aligned
    // word at 4t before the quant word; odd: the quant word t itself)
    const uint32_t w_lane = (uint32_t)g * kSkWRowBytes + (uint32_t)bw * 18 + (even_block ? 4u * t : 2u + 4u * t);
    const uint32_t d_lane = (uint32_t)g * kSkWRowBytes + (uint32_t)bw * 18;
    int s = 0;
    uint32_t ph = 0;
    for (int c = 0; c < nchunks; ++c) {
        float acc[RG][NT][4];
#pragma unroll
        for (int r = 0; r < RG; ++r)
#pragma unroll
            for (int j = 0; j < NT; ++j) acc[r][j][0] = acc[r][j][1] = acc[r][j][2] = acc[r][j][3] = 0.0f;
        for (int ks = 0; ks < nslices; ++ks) {
            if (!mbar_wait(&full_bar[s], ph, a.status)) return;
            const uint8_t* stg = smem + (size_t)s * a.stage_bytes;
#pragma unroll
            for (int u = 0; u < SUBS; ++u) {
                const uint8_t* wst = stg + (size_t)u * (TR * kSkWRowBytes);
                const uint8_t* xst = stg + (size_t)u * (2 * SP * kSkXPitch);
                // B fragments of block bw for every 8-sequence tile: k 2t, 2t+1 = elements
                // (4t, 4t+2), k 2t+8, 2t+9 = (4t+1, 4t+3); then the same + 16
                uint32_t bf[NT][4];
#pragma unroll
                for (int j = 0; j < NT; ++j) {
                    const uint8_t* xr = xst + x_lane + (size_t)(8 * j) * kSkXPitch;
                    const uint2 lo = *reinterpret_cast<const uint2*>(xr);
                    const uint2 hi = *reinterpret_cast<const uint2*>(xr + 32);
                    bf[j][0] = prmt(lo.x, lo.y, 0x5410u);
                    bf[j][1] = prmt(lo.x, lo.y, 0x7632u);
                    bf[j][2] = prmt(hi.x, hi.y, 0x5410u);
                    bf[j][3] = prmt(hi.x, hi.y, 0x7632u);
                }
#pragma unroll
                for (int r = 0; r < RG; ++r) {
                    const uint8_t* rw = wst + (size_t)(r * 16) * kSkWRowBytes;
                    uint32_t wg, wg8;
                    if (even_block) {
                        const uint32_t* p = reinterpret_cast<const uint32_t*>(rw + w_lane);
                        const uint32_t* p8 = reinterpret_cast<const uint32_t*>(rw + w_lane + 8 * kSkWRowBytes);
                        wg = prmt(p[0], p[1], 0x5432u);
                        wg8 = prmt(p8[0], p8[1], 0x5432u);
                    } else {
                        wg = *reinterpret_cast<const uint32_t*>(rw + w_lane);
                        wg8 = *reinterpret_cast<const uint32_t*>(rw + w_lane + 8 * kSkWRowBytes);
                    }
                    const float dg = __half2float(*reinterpret_cast<const __half*>(rw + d_lane));
                    const float dg8 = __half2float(*reinterpret_cast<const __half*>(rw + d_lane + 8 * kSkWRowBytes));
                    // A: rows g / g+8; first k16 step the low nibbles (elements 4t, 4t+2 at bit 0,
                    // 4t+1, 4t+3 at bit 8), second the high nibbles (bits 4 and 12)
                    const uint32_t a0[4] = {nib_pair<T, 0>(wg, sub2), nib_pair<T, 0>(wg8, sub2),
                                            nib_pair<T, 8>(wg, sub2), nib_pair<T, 8>(wg8, sub2)};
                    const uint32_t a1[4] = {nib_pair<T, 4>(wg, sub2), nib_pair<T, 4>(wg8, sub2),
                                            nib_pair<T, 12>(wg, sub2), nib_pair<T, 12>(wg8, sub2)};
#pragma unroll
                    for (int j = 0; j < NT; ++j) {
                        float d4[4] = {0.0f, 0.0f, 0.0f, 0.0f};
                        mma16816<T>(d4, a0, bf[j][0], bf[j][1]);
                        mma16816<T>(d4, a1, bf[j][2], bf[j][3]);
                        acc[r][j][0] = fmaf(dg, d4[0], acc[r][j][0]);
                        acc[r][j][1] = fmaf(dg, d4[1], acc[r][j][1]);
                        acc[r][j][2] = fmaf(dg8, d4[2], acc[r][j][2]);
                        acc[r][j][3] = fmaf(dg8, d4[3], acc[r][j][3]);
                    }
                }
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty_bar[s]);
            if (++s == a.stages) {
                s = 0;
                ph ^= 1u;
            }
        }
        // partial sums of this warp: rows 16r + g, 16r + g + 8, sequences 8j + 2t, 8j + 2t + 1
#pragma unroll
        for (int r = 0; r < RG; ++r)
#pragma unroll
            for (int j = 0; j < NT; ++j) {
                float* rp = red + ((size_t)warp * SP + 8 * j + 2 * t) * RP + r * 16 + g;
                rp[0] = acc[r][j][0];
                rp[RP] = acc[r][j][1];
                rp[8] = acc[r][j][2];
                rp[RP + 8] = acc[r][j][3];
            }
        __syncwarp();
        if (lane == 0) mbar_arrive(&red_bar);
        if (!mbar_wait(&red_bar, (uint32_t)c & 1u, a.status)) return;
        const int row0 = r0 + c * TR;
        const int nrows = min(TR, r1 - row0);
        const bool fused = epilogue_active(a.epi);
        for (int i = tid; i < ns * TR; i += 256) {
            const int sq = i / TR, r = i % TR;  // consecutive threads: consecutive rows
            if (r >= nrows) continue;
            float v = 0.0f;
#pragma unroll
            for (int w = 0; w < 8; ++w) v += red[((size_t)w * SP + sq) * RP + r];
            if (a.bias) v += bias_value(a.bias, a.bias_type, row0 + r);
            if (fused) v = epilogue_finish(a.epi, seq0 + sq, row0 + r, v);
            store_value(a.C, a.c_type, (size_t)(seq0 + sq) * a.ldc + row0 + r, v);
        }
        if (c + 1 < nchunks) {
            // the next chunk's partials overwrite these
            __syncwarp();
            if (lane == 0) mbar_arrive(&done_bar);
            if (!mbar_wait(&done_bar, (uint32_t)c & 1u, a.status)) return;
        }
    }
}

// The (row groups, sub-slices) pairs the planner uses.  One kernel function per (NT, T) holds
// them all and picks one at run time: a decode step's GEMMs of different shapes then launch the
// same function, and a dependent launch of a different function was measured ~1.4 us slower
// than one of the same function (the M = 1 decode step: 455 -> 388 us with one function).
enum SkinnyShape : int { kRg1S1, kRg1S2, kRg1S4, kRg1S8, kRg2S1, kRg2S2, kRg2S4, kRg3S1, kRg3S2, kRg4S1 };

template <int NT, typename T>
__global__ void __launch_bounds__(kSkThreads, 2)
    gemm_q4_skinny(const __grid_constant__ CUtensorMap tmW, const __grid_constant__ CUtensorMap tmX, SkinnyArgs a) {
    switch (a.shape) {
        case kRg4S1: skinny_body<NT, 4, 1, T>(tmW, tmX, a); break;
        case kRg3S1: skinny_body<NT, 3, 1, T>(tmW, tmX, a); break;
        case kRg2S1: skinny_body<NT, 2, 1, T>(tmW, tmX, a); break;
        case kRg2S2: skinny_body<NT, 2, 2, T>(tmW, tmX, a); break;
        case kRg1S1: skinny_body<NT, 1, 1, T>(tmW, tmX, a); break;
        case kRg1S2: skinny_body<NT, 1, 2, T>(tmW, tmX, a); break;
        case kRg1S4: skinny_body<NT, 1, 4, T>(tmW, tmX, a); break;
        default:
            // with one 8-sequence tile only (the registers of two CTAs per SM)
            if constexpr (NT == 1) {
                switch (a.shape) {
                    case kRg3S2: skinny_body<NT, 3, 2, T>(tmW, tmX, a); break;
                    case kRg2S4: skinny_body<NT, 2, 4, T>(tmW, tmX, a); break;
                    case kRg1S8: skinny_body<NT, 1, 8, T>(tmW, tmX, a); break;
                    default: break;
                }
            }
            break;
    }
}

template <int NT, typename T>
cudaError_t launch_skinny(const mgpu_k::LaunchCtx& c, const CUtensorMap& tm, const CUtensorMap& tx,
                          const SkinnyArgs& a, dim3 grid, size_t smem) {
    auto kern = gemm_q4_skinny<NT, T>;
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

// The shape id of a planner choice.
int skinny_shape(int NT, int rg, int subs) {
    switch (rg) {
        case 4: return kRg4S1;
        case 3: return NT == 1 && subs == 2 ? kRg3S2 : kRg3S1;
        case 2: return NT == 1 && subs == 4 ? kRg2S4 : subs == 2 ? kRg2S2 : kRg2S1;
        default: return NT == 1 && subs == 8 ? kRg1S8 : subs == 4 ? kRg1S4 : subs == 2 ? kRg1S2 : kRg1S1;
    }
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
    // up to 16 sequences per CTA; more take further CTAs over the same rows (grid.y), whose
    // second read of the packed rows is served by L2
    const int NT = M <= 8 ? 1 : 2;
    const int SP = 8 * NT;
    // CTAs over the rows: one per SM, fewer when a CTA would get fewer than 8 rows.  Layer
    // shapes then all launch one CTA per SM: consecutive launches of a decode step whose grid
    // sizes differ (148 and 128 CTAs at N = 2048 with 16-row shares) were measured ~1 us slower
    // each (S = 8 step: 751 -> 575 us with 148 CTAs for every shape).
    const int G = max(1, min(c.sm_count, (N + 7) / 8));
    const int rows_per_cta = (N + G - 1) / G;
    auto xoff_of = [&](int rg, int u) { return ((size_t)u * 16 * rg * kSkWRowBytes + 127) / 128 * 128; };
    auto red_of = [&](int rg) { return (size_t)8 * SP * (16 * rg + 4) * sizeof(float); };
    auto stage_of = [&](int rg, int u) {
        return (xoff_of(rg, u) + (size_t)2 * u * SP * kSkXPitch + 1023) / 1024 * 1024;
    };
    // rows per chunk (16 RG): the choice with the fewest padded rows, counting each chunk's
    // reduction as 8 rows of work, among those where the partial sums and two stages fit
    int RG = 0;
    long best = 0;
    for (int rg = 1; rg <= 4; ++rg) {
        if (2 * stage_of(rg, 1) + red_of(rg) + 1024 > kSkSmemBudget) continue;
        const long chunks = (rows_per_cta + 16 * rg - 1) / (16 * rg);
        const long cost = chunks * 16 * rg + 8 * chunks;
        if (RG == 0 || cost <= best) {
            RG = rg;
            best = cost;
        }
    }
    if (RG == 0) return cudaErrorInvalidValue;
    const int TR = 16 * RG;
    const size_t red_bytes = red_of(RG);
    // sub-slices per stage: up to 8 (row group, block) units per warp (4 with two tiles),
    // dividing K / 256, with at least 2 stages
    const int max_units = NT == 1 ? 8 : 4;
    int subs = RG == 4 ? 1 : RG == 3 ? max_units / 4 : max_units / RG;
    while (subs > 1 && ((K / kSkSlice) % subs != 0 || 2 * stage_of(RG, subs) + red_bytes + 1024 > kSkSmemBudget))
        subs >>= 1;
    const uint32_t stage_bytes = (uint32_t)stage_of(RG, subs);
    const uint32_t x_offset = (uint32_t)xoff_of(RG, subs);
    const int stages = (int)std::min<size_t>(kSkMaxStages, (kSkSmemBudget - 1024 - red_bytes) / stage_bytes);
    if (stages < 2) return cudaErrorInvalidValue;
    const size_t smem = 1024 + (size_t)stages * stage_bytes + red_bytes;

    CUtensorMap tm;
    // W as [K/256 slices][N rows][72 units]: unit pitch 2 bytes, row pitch K/32 * 18 bytes, slice
    // pitch 144 bytes; box {72, TR, subs}, rows past N read as zeros
    {
        const int64_t dims[3] = {kSkWRowBytes / 2, N, K / kSkSlice};
        const int64_t strides[2] = {B.ld, kSkWRowBytes};
        const int box[3] = {kSkWRowBytes / 2, TR, subs};
        if (!make_tensor_map_u16_3d(&tm, B.ptr, dims, strides, box)) return cudaErrorInvalidValue;
    }
    // A as [K/128 chunks][M rows][128 elements]: box {136, 8 NT, 2 subs}, whose 8 columns past a
    // chunk and rows past M read as zeros; each activation row lands at a 272-byte pitch
    CUtensorMap tx;
    {
        const int64_t dims[3] = {128, M, K / 128};
        const int64_t strides[2] = {A.ld * 2, 256};
        const int box[3] = {kSkXBox, SP, 2 * subs};
        if (!make_tensor_map_u16_3d(&tx, A.ptr, dims, strides, box)) return cudaErrorInvalidValue;
    }
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
    a.tx_bytes = (uint32_t)(subs * TR * kSkWRowBytes + 2 * subs * SP * kSkXPitch);
    a.stage_bytes = stage_bytes;
    a.x_offset = x_offset;
    a.status = c.status;
    const dim3 grid(G, (M + SP - 1) / SP);
    const bool bf16 = A.type == MGPU_BF16;
    a.shape = skinny_shape(NT, RG, subs);
    if (NT == 1)
        return bf16 ? launch_skinny<1, __nv_bfloat16>(c, tm, tx, a, grid, smem)
                    : launch_skinny<1, __half>(c, tm, tx, a, grid, smem);
    return bf16 ? launch_skinny<2, __nv_bfloat16>(c, tm, tx, a, grid, smem)
                : launch_skinny<2, __half>(c, tm, tx, a, grid, smem);
}

}  // namespace mgpu_k
