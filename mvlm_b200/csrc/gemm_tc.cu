// gemm_tc.cu - tcgen05 tensor-core GEMM for sm_100a (replaces gemm_naive / gemm_tiled /
// gemm_image, src/kernels/gemm.cl:26-200, and the GEMM math of patch_embed / vision_proj,
// src/kernels/vision.cl:118-197, :402-441).
//
// C[M,N] = A[M,K] * op(B) (+ bias[N]), fp16 or bf16 operands, fp32 accumulation in TMEM.
//
// One persistent CTA per SM walks output tiles of 128 x BN (BN = 256 or 128), K in steps
// of 64 (one 128-byte swizzle atom of 16-bit elements).  Warp roles:
//   warp 0      TMA producer: A tiles (and 16-bit B tiles) with cp.async.bulk.tensor, 128B
//               swizzle, into a ring of smem stages; OOB boxes are zero-filled, which pads
//               ragged M, N and K.
//   warp 1      allocates TMEM (2 x BN fp32 columns: a double-buffered accumulator) and one
//               elected lane issues tcgen05.mma (M=128, N=BN, K=16 per instruction) and
//               tcgen05.commit to release stages / publish finished accumulators.
//   warps 2-5   epilogue: tcgen05.ld 32 lanes x 32 columns per warp, + bias, convert,
//               store; overlaps the next tile's main loop through the second accumulator.
//   warps 6-13  (Q8_0 / Q4_0 B only) dequantisers: read the packed GGUF blocks of the B
//               tile straight from global memory, decode them exactly in fp32, round to the
//               operand type and write them into the stage in the same 128B-swizzled
//               K-major layout TMA would have produced, then fence.proxy.async + arrive.
// B layouts: NK (K-major, e.g. GGUF F16 tensors) and KN (MN-major: the reference kernels'
// B[K][N], read by tcgen05 with the B-transpose bit).  Every TMA load fills only the issuing CTA.
//
// CTA pairs (CG = 2): a (2,1,1) cluster computes a 256 x BN tile with tcgen05 cta_group::2.
// Each CTA stages its own 128 rows of A and BN / 2 rows of B (TMA or its own dequantisers);
// the even CTA's MMA warp issues M = 256 MMAs that read both CTAs' stages and accumulate into
// both CTAs' TMEM.  Stage and accumulator barriers live in the even CTA (the odd CTA's TMA
// loads count their bytes there, its dequantisers and epilogue arrive there); the MMA commits
// arrive on the same barrier offsets of both CTAs, releasing each CTA's stages and
// accumulators.  This halves the B operand bytes each tensor core reads per MMA.
#include <atomic>
#include <mutex>
#include <type_traits>

#include "common.cuh"
#include "kernels.h"

using namespace mgpu_dev;

namespace {

constexpr int BM = 128, BK = 64;
constexpr int kABytes = BM * BK * 2;  // 16 KB
constexpr int kSmemBudget = 200 * 1024;
// B operand modes: 16-bit via TMA (K-major / MN-major); GGUF blocks read with plain loads
// (any K % 32 == 0); GGUF blocks staged by TMA in 256-k groups (K % 256 == 0).
enum BMode { B_TMA_K = 0, B_TMA_MN = 1, B_Q8 = 2, B_Q4 = 3, B_Q8_TMA = 4, B_Q4_TMA = 5 };
__host__ __device__ constexpr bool is_quant_mode(int m) { return m >= B_Q8; }
__host__ __device__ constexpr bool is_packed_tma(int m) { return m >= B_Q8_TMA; }
__host__ __device__ constexpr bool is_q4_mode(int m) { return m == B_Q4 || m == B_Q4_TMA; }
// bytes of one 256-element group of a GGUF row (8 blocks)
__host__ __device__ constexpr int group_bytes(int m) { return is_q4_mode(m) ? 144 : 272; }
constexpr int kDqWarps = 8;

__host__ __device__ constexpr int gemm_threads(int bmode) { return 192 + (is_quant_mode(bmode) ? kDqWarps * 32 : 0); }
// MT = 128-row M sub-tiles per CTA tile.  With MT = 2 (TMA-staged quantised modes only) a CTA
// computes a 256 x BN tile as two tcgen05 accumulators that share each decoded B stage, which
// halves the decode work per FLOP (for M = 761 each weight is decoded 3 times instead of 6);
// the host picks MT per shape, since 256-row tiles leave SMs idle when there are few of them.
// CG = CTAs per tile: with CG = 2 a (2,1,1) cluster computes a 256 x BN tile with tcgen05
// cta_group::2 MMAs (M = 256), each CTA staging 128 rows of A and BN / 2 rows of B.  Each
// tensor core then reads half as many B bytes per MMA as with one CTA per tile, and the
// MMA's shared-memory operand reads are what bound the one-CTA kernel (measured: a 128 x 128
// x 16 MMA step takes ~70 ns there, with decode, A loads and everything else removed).
__host__ __device__ constexpr int stage_bytes(int bn, int mt = 1, int cg = 1) { return mt * kABytes + (bn / cg) * BK * 2; }
// packed-group ring (two slots) of the TMA-staged quantised modes
__host__ __device__ constexpr int packed_bytes(int bn, int bmode, int cg = 1) {
    return is_packed_tma(bmode) ? 2 * (bn / cg) * group_bytes(bmode) : 0;
}
constexpr int kSmemMaxDyn = 226 * 1024;  // dynamic shared memory available next to the static barriers
__host__ __device__ constexpr int num_stages(int bn, int bmode = B_TMA_K, int mt = 1, int cg = 1) {
    return is_packed_tma(bmode) ? (kSmemMaxDyn - 1024 - packed_bytes(bn, bmode, cg)) / stage_bytes(bn, mt, cg)
                                : kSmemBudget / stage_bytes(bn, mt, cg);
}
__host__ __device__ constexpr int smem_bytes(int bn, int bmode, int mt = 1, int cg = 1) {
    return num_stages(bn, bmode, mt, cg) * stage_bytes(bn, mt, cg) + packed_bytes(bn, bmode, cg) + 1024;
}

struct GemmArgs {
    int M, N, K, num_kb, tiles_m, tiles_n;
    void* C;
    int64_t ldc;
    int c_type;
    const void* bias;
    int bias_type;
    mgpu_k::Epilogue epi;  // activation / residual after the bias
    const uint8_t* Bq;   // packed GGUF rows (quantised modes)
    int64_t bq_row_bytes;
    const uint8_t* bq_end;
    int* status;
    // split-K: `splits` CTAs share a tile, each over kb_per_split k-blocks (a multiple of 4,
    // i.e. whole 256-k groups); fp32 partials [split][M][N], and the tile's ticket counts
    // arrivals so that the last one sums the partials in split order.
    int splits, kb_per_split;
    unsigned int* tickets;
    float* partials;
    // cluster split-K: csplit > 1 runs each tile as one cluster of csplit CTAs (CTA pairs in
    // pair mode), the i-th over k-blocks [i * kb_per_split, ..) (the last may be shorter); the
    // fp32 partials stay in shared memory and the cluster sums them over DSMEM (splits ==
    // csplit, tickets and partials unused).
    int csplit;
    // Tile order: 0 = m-fastest over all of M; g > 0 = bands of g m-blocks, m-fastest inside a
    // band, the bands one after the other, so that a band's A rows stay in L2 while every
    // n-block passes over them (large M, where A does not fit L2 beside B).
    int group_m;
};

// The (m-block, n-block) of tile index `tile` in the order above.
__device__ __forceinline__ void tile_coords(const GemmArgs& g, int tile, int& m_blk, int& n_blk) {
    if (g.group_m <= 0 || g.group_m >= g.tiles_m) {
        m_blk = tile % g.tiles_m;
        n_blk = tile / g.tiles_m;
        return;
    }
    const int per_band = g.group_m * g.tiles_n;
    const int band = tile / per_band;
    const int first_m = band * g.group_m;
    const int gm = min(g.group_m, g.tiles_m - first_m);  // the last band may be narrower
    const int r = tile - band * per_band;
    m_blk = first_m + r % gm;
    n_blk = r / gm;
}
__device__ __forceinline__ int tile_n_blk(const GemmArgs& g, int tile) {
    int m, n;
    tile_coords(g, tile, m, n);
    return n;
}

template <typename T>
__device__ __forceinline__ uint32_t pack2(float a, float b);
template <>
__device__ __forceinline__ uint32_t pack2<__nv_bfloat16>(float a, float b) {
    __nv_bfloat162 v = __floats2bfloat162_rn(a, b);
    return *reinterpret_cast<uint32_t*>(&v);
}
template <>
__device__ __forceinline__ uint32_t pack2<__half>(float a, float b) {
    __half2 v = __floats2half2_rn(a, b);
    return *reinterpret_cast<uint32_t*>(&v);
}

__device__ __forceinline__ float bias_at(const void* bias, int type, int n) {
    if (type == MGPU_F32) return reinterpret_cast<const float*>(bias)[n];
    if (type == MGPU_F16) return __half2float(reinterpret_cast<const __half*>(bias)[n]);
    return __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(bias)[n]);
}

__device__ __forceinline__ void store_out(void* C, int type, size_t idx, float v) {
    if (type == MGPU_F32) reinterpret_cast<float*>(C)[idx] = v;
    else if (type == MGPU_F16) reinterpret_cast<__half*>(C)[idx] = __float2half_rn(v);
    else reinterpret_cast<__nv_bfloat16*>(C)[idx] = __float2bfloat16_rn(v);
}

// Raw words of one packed block (Q4_0: 5 words / 18 bytes, Q8_0: 9 words / 34 bytes) from a
// 2-byte-aligned address: the aligned words that cover it plus the realignment selector.
template <int NW>
struct RawBlock {
    uint32_t w[NW];
    uint32_t par;  // 0 or 2: byte offset of the block inside w[0]
    bool valid;
};

template <int NW, int BB>
__device__ __forceinline__ void load_block(RawBlock<NW>& rb, const uint8_t* p, const uint8_t* end, bool valid) {
    rb.valid = valid;
    rb.par = 0;
    if (!valid) return;
    const uintptr_t a = reinterpret_cast<uintptr_t>(p);
    rb.par = (uint32_t)(a & 3u);
    const uint32_t* wp = reinterpret_cast<const uint32_t*>(a & ~(uintptr_t)3);
    if (reinterpret_cast<const uint8_t*>(wp + NW) <= end) {
#pragma unroll
        for (int i = 0; i < NW; ++i) rb.w[i] = __ldg(wp + i);
    } else {
        // Last block of the buffer: do not read the 2 bytes past its end.
        const uint16_t* hp = reinterpret_cast<const uint16_t*>(p);
        uint16_t h[2 * NW];
#pragma unroll
        for (int i = 0; i < 2 * NW; ++i) h[i] = (i < BB / 2) ? __ldg(hp + i) : (uint16_t)0;
#pragma unroll
        for (int i = 0; i < NW; ++i) rb.w[i] = (uint32_t)h[2 * i] | ((uint32_t)h[2 * i + 1] << 16);
        rb.par = 0;
    }
}

// Byte `byte_sel` of v placed at bits 8-15 of the float 2^23: the value 2^23 + 256 * byte.
// Then fma(that, d / 256, -(2^15 + z) * d) = (byte - z) * d exactly: d / 256 and (2^15 + z) * d
// (z = 128 or 8: 9 or 13 significant bits times d's 11) are exact in fp32, the fma rounds once,
// and (byte - z) * d needs at most 19 bits.
#define MAGIC_F(v, byte_sel) __uint_as_float(prmt((v), 0x4B000000u, 0x7504u | ((byte_sel) << 4)))

// Decode one block into 32 values of T (4 x 16 bytes) and store them to the four swizzled
// 16-byte chunks `dst[0..3]`.
template <int BMODE, typename T, int NW>
__device__ __forceinline__ void decode_store(const RawBlock<NW>& rb, uint4* const (&dst)[4]) {
    if (!rb.valid) {
#pragma unroll
        for (int j = 0; j < 4; ++j) *dst[j] = make_uint4(0, 0, 0, 0);
        return;
    }
    const uint32_t sel = rb.par ? 0x7654u : 0x5432u;
    const uint32_t dsel = rb.par ? 0x4432u : 0x4410u;
    const float d = __half2float(__ushort_as_half((unsigned short)prmt(rb.w[0], 0u, dsel)));
    const float2 d8 = make_float2(d * 0.00390625f, d * 0.00390625f);
    if constexpr (is_q4_mode(BMODE)) {
        const float2 off = make_float2(-32776.0f * d, -32776.0f * d);
        uint32_t lo[4], hi[4];
#pragma unroll
        for (int m = 0; m < 4; ++m) {
            const uint32_t q = prmt(rb.w[m], rb.w[m + 1], sel);
            lo[m] = q & 0x0F0F0F0Fu;
            hi[m] = (q >> 4) & 0x0F0F0F0Fu;
        }
        // chunk 0: lo of qs[0..7], chunk 1: lo of qs[8..15], chunk 2/3: hi of the same
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const uint32_t* src = (j < 2) ? lo : hi;
            const int w0 = (j & 1) * 2;
            uint32_t o[4];
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                const uint32_t v = src[w0 + h];
                const float2 a = __ffma2_rn(make_float2(MAGIC_F(v, 0), MAGIC_F(v, 1)), d8, off);
                const float2 b = __ffma2_rn(make_float2(MAGIC_F(v, 2), MAGIC_F(v, 3)), d8, off);
                o[2 * h] = pack2<T>(a.x, a.y);
                o[2 * h + 1] = pack2<T>(b.x, b.y);
            }
            *dst[j] = make_uint4(o[0], o[1], o[2], o[3]);
        }
    } else {
        const float2 off = make_float2(-32896.0f * d, -32896.0f * d);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            uint32_t o[4];
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                const int m = 2 * j + h;
                const uint32_t v = prmt(rb.w[m], rb.w[m + 1], sel) ^ 0x80808080u;
                const float2 a = __ffma2_rn(make_float2(MAGIC_F(v, 0), MAGIC_F(v, 1)), d8, off);
                const float2 b = __ffma2_rn(make_float2(MAGIC_F(v, 2), MAGIC_F(v, 3)), d8, off);
                o[2 * h] = pack2<T>(a.x, a.y);
                o[2 * h + 1] = pack2<T>(b.x, b.y);
            }
            *dst[j] = make_uint4(o[0], o[1], o[2], o[3]);
        }
    }
}

template <int BN, int BMODE, typename T, int MT, int CG>
__global__ void __launch_bounds__(gemm_threads(BMODE), 1)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB, GemmArgs g) {
    static_assert(MT == 1 || (MT == 2 && BN == 128 && CG == 1), "256-row tiles use 128-column B tiles");
    static_assert(CG == 1 || (CG == 2 && (BMODE == B_TMA_K || BMODE == B_TMA_MN || is_packed_tma(BMODE))),
                  "CTA pairs stage A and B by TMA");
    constexpr int BNC = BN / CG;                 // B rows (output columns) staged by this CTA
    constexpr int S = num_stages(BN, BMODE, MT, CG);
    constexpr int SB = stage_bytes(BN, MT, CG);
    constexpr int TBM = BM * MT * CG;            // rows of a tile
    constexpr int AB = MT * kABytes;             // A bytes per stage in this CTA
    constexpr uint32_t kTmemCols = 2 * MT * BN;  // double-buffered accumulators
    constexpr bool kQuant = is_quant_mode(BMODE);
    constexpr bool kPair = CG == 2;
    constexpr bool kBf16 = sizeof(T) == 2 && !std::is_same<T, __half>::value;
    constexpr uint32_t kIdesc = idesc_f16(kBf16, false, BMODE == B_TMA_MN, BM * CG, BN);

    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
    __shared__ __align__(8) uint64_t full_bar[S];
    __shared__ __align__(8) uint64_t empty_bar[S];
    __shared__ __align__(8) uint64_t tfull_bar[2];
    __shared__ __align__(8) uint64_t tempty_bar[2];
    __shared__ __align__(8) uint64_t drain_bar;
    __shared__ __align__(8) uint64_t pk_full[2];
    __shared__ __align__(8) uint64_t pk_empty[2];
    __shared__ uint32_t tmem_base_slot;
    __shared__ volatile int abort_flag;
    __shared__ volatile int split_last;

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int total_tiles = g.tiles_m * g.tiles_n;
    const int total_units = total_tiles * g.splits;  // unit = (split, tile): split-major
    // CTA pairs walk the units together: cluster index and count stand in for the block's.
    // With cluster split-K each cluster owns one unit: (K slice, tile).
    const int csplit = g.csplit;
    const uint32_t crank = (kPair || csplit > 1) ? cluster_ctarank() : 0u;
    const uint32_t rank = kPair ? (crank & 1u) : 0u;         // CTA within its pair
    const uint32_t ksplit = kPair ? (crank >> 1) : crank;    // K slice (cluster split-K)
    const uint32_t lead = crank - rank;                      // the pair's even CTA
    const int ufirst = csplit > 1 ? (int)ksplit * total_tiles + (int)blockIdx.x / (CG * csplit)
                                  : (kPair ? (int)(blockIdx.x >> 1) : (int)blockIdx.x);
    const int ustep = csplit > 1 ? total_units : (kPair ? (int)(gridDim.x >> 1) : (int)gridDim.x);
    auto kb_end = [&](int kb0) { return min(kb0 + g.kb_per_split, g.num_kb); };

    if (tid == 0) {
        for (int s = 0; s < S; ++s) {
            // the pair's stage is full when both CTAs' dequantisers have arrived (on the even CTA)
            mbar_init(&full_bar[s], 1 + CG * (is_packed_tma(BMODE) ? BNC / 32 : kQuant ? kDqWarps : 0));
            mbar_init(&empty_bar[s], 1);
        }
        for (int a = 0; a < 2; ++a) {
            mbar_init(&tfull_bar[a], 1);
            mbar_init(&tempty_bar[a], 4 * CG);
        }
        mbar_init(&drain_bar, 1);
        for (int p = 0; p < 2; ++p) {
            mbar_init(&pk_full[p], 1);
            mbar_init(&pk_empty[p], kDqWarps);
        }
        abort_flag = 0;
        fence_mbar_init();
        // Programmatic dependent launch: the next kernel of the stream may start its prologue
        // (and stage its own weights) on SMs this grid leaves free; it reads our output only
        // after its griddepcontrol.wait.
        asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    }
    if (warp == 0 && lane == 0) {
        prefetch_tensormap(&tmA);
        if (!kQuant || is_packed_tma(BMODE)) prefetch_tensormap(&tmB);
    }
    if (warp == 1) {
        if constexpr (kPair) {
            tmem_alloc_pair(&tmem_base_slot, kTmemCols);
            tmem_relinquish_pair();
        } else {
            tmem_alloc(&tmem_base_slot, kTmemCols);
            tmem_relinquish();
        }
    }
    tc_fence_before();
    __syncthreads();
    // the peer arrives on (and its TMA completes bytes on) this CTA's barriers: both CTAs'
    // barriers are initialised before either goes on
    if constexpr (kPair) cluster_sync_all();
    tc_fence_after();
    const uint32_t tmem_base = tmem_base_slot;
    // the pair's even CTA's barriers, in the cluster window (pair mode)
    const uint32_t full0_cl = kPair ? cluster_addr(&full_bar[0], lead) : 0u;
    const uint32_t tempty0_cl = kPair ? cluster_addr(&tempty_bar[0], lead) : 0u;
    const uint16_t pair_mask = (uint16_t)(3u << lead);

    if (warp == 0) {
        // ---------------------------------------------------------------- TMA producer
        if (lane == 0) {
            // A (and bias / C) may belong to the preceding kernel of the stream: wait for it.
            // Everything that reads A or writes C is ordered after this (the MMAs consume the
            // stages loaded here, the epilogue their accumulators).  Quantised B is staged by
            // the dequant warps without waiting: weights are never written by the previous
            // kernel.
            // Dense B of this CTA's first stages is staged before the wait too.
            // In pair mode every load of either CTA counts its bytes on the even CTA's barrier,
            // and only the even CTA announces them (for both CTAs).
            auto expect = [&](uint32_t s) {
                if (!kPair || rank == 0)
                    mbar_arrive_expect_tx(&full_bar[s], (uint32_t)(CG * (AB + (kQuant ? 0 : BNC * BK * 2))));
            };
            auto load = [&](uint8_t* dst, int x, int y, uint32_t s, const CUtensorMap* map) {
                if constexpr (kPair) tma_load_2d_pair(dst, map, x, y, full0_cl + 8u * s);
                else tma_load_2d(dst, map, x, y, &full_bar[s]);
            };
            auto load_a = [&](uint8_t* a_dst, int kb, int m_blk, uint32_t s) {
#pragma unroll
                for (int mt = 0; mt < MT; ++mt)
                    load(a_dst + mt * kABytes, kb * BK, m_blk * TBM + ((int)rank * MT + mt) * BM, s, &tmA);
            };
            auto load_b = [&](uint8_t* b_dst, int kb, int n_blk, uint32_t s) {
                const int n0 = n_blk * BN + (int)rank * BNC;
                if constexpr (BMODE == B_TMA_K) {
                    load(b_dst, kb * BK, n0, s, &tmB);
                } else if constexpr (BMODE == B_TMA_MN) {
#pragma unroll
                    for (int j = 0; j < BNC / 64; ++j) load(b_dst + j * 8192, n0 + j * 64, kb * BK, s, &tmB);
                }
            };
            uint32_t it = 0;
            int pre = 0;
            if constexpr (!kQuant) {
                if (ufirst < total_units) {
                    const int tile = ufirst % total_tiles, kb0 = (ufirst / total_tiles) * g.kb_per_split;
                    const int n_blk = tile_n_blk(g, tile);
                    pre = min(S, kb_end(kb0) - kb0);
                    for (int p = 0; p < pre; ++p) {
                        // fresh ring: every slot is free
                        expect((uint32_t)p);
                        load_b(smem + p * SB + AB, kb0 + p, n_blk, (uint32_t)p);
                    }
                }
            }
            asm volatile("griddepcontrol.wait;" ::: "memory");
            for (int unit = ufirst; unit < total_units && !abort_flag; unit += ustep) {
                const int tile = unit % total_tiles, kb0 = (unit / total_tiles) * g.kb_per_split;
                int m_blk, n_blk;
                tile_coords(g, tile, m_blk, n_blk);
                for (int kb = kb0; kb < kb_end(kb0); ++kb, ++it) {
                    const uint32_t s = it % S, ph = (it / S) & 1u;
                    uint8_t* a_dst = smem + s * SB;
                    uint8_t* b_dst = a_dst + AB;
                    if ((int)it < pre) {
                        // B already in flight: A only
                        load_a(a_dst, kb, m_blk, s);
                        continue;
                    }
                    if (!mbar_wait(&empty_bar[s], ph ^ 1u, g.status)) {
                        abort_flag = 1;
                        break;
                    }
                    expect(s);
                    load_a(a_dst, kb, m_blk, s);
                    load_b(b_dst, kb, n_blk, s);
                }
            }
        }
    } else if (warp == 1) {
        // ---------------------------------------------------------------- MMA issuer
        // (pair mode: the even CTA's lane 0 issues for both CTAs; the odd CTA's warp idles)
        if (lane == 0 && rank == 0) {
            uint32_t it = 0, tcount = 0;
            bool issued = false;
            for (int unit = ufirst; unit < total_units && !abort_flag; unit += ustep, ++tcount) {
                const int kb0 = (unit / total_tiles) * g.kb_per_split;
                const uint32_t acc = tcount & 1u, acc_ph = (tcount >> 1) & 1u;
                if (!mbar_wait(&tempty_bar[acc], acc_ph ^ 1u, g.status)) {
                    abort_flag = 1;
                    break;
                }
                tc_fence_after();
                const uint32_t d_tmem = tmem_base + acc * (MT * BN);
                for (int kb = kb0; kb < kb_end(kb0); ++kb, ++it) {
                    const uint32_t s = it % S, ph = (it / S) & 1u;
                    if (!mbar_wait(&full_bar[s], ph, g.status)) {
                        abort_flag = 1;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t a_addr = smem_u32(smem + s * SB);
                    const uint32_t b_addr = a_addr + AB;
#pragma unroll
                    for (int k = 0; k < BK / 16; ++k) {
                        uint64_t bdesc;
                        if constexpr (BMODE == B_TMA_MN)
                            bdesc = smem_desc(b_addr + k * 2048, 8192, 1024, kSwizzle128B);
                        else
                            bdesc = smem_desc(b_addr + k * 32, 16, 1024, kSwizzle128B);
#pragma unroll
                        for (int mt = 0; mt < MT; ++mt) {
                            const uint64_t adesc = smem_desc(a_addr + mt * kABytes + k * 32, 16, 1024, kSwizzle128B);
                            if constexpr (kPair)
                                umma_f16_pair(d_tmem, adesc, bdesc, kIdesc, (kb != kb0 || k != 0) ? 1u : 0u);
                            else
                                umma_f16(d_tmem + mt * BN, adesc, bdesc, kIdesc, (kb != kb0 || k != 0) ? 1u : 0u);
                        }
                    }
                    issued = true;
                    if constexpr (kPair) umma_commit_pair_both(&empty_bar[s], pair_mask);
                    else umma_commit(&empty_bar[s]);
                }
                if (abort_flag) break;
                if constexpr (kPair) umma_commit_pair_both(&tfull_bar[acc], pair_mask);
                else umma_commit(&tfull_bar[acc]);
            }
            if (issued) {
                // All MMAs retire before TMEM is released.
                if constexpr (kPair) umma_commit_pair(&drain_bar);
                else umma_commit(&drain_bar);
                mbar_wait(&drain_bar, 0, g.status);
            }
        }
    } else if (warp < 6) {
        // ---------------------------------------------------------------- epilogue
        const int q = warp & 3;  // TMEM lane quarter this warp may access
        uint32_t tcount = 0;
        const bool vec_ok = (g.ldc % 8 == 0) && ((reinterpret_cast<uintptr_t>(g.C) & 15) == 0);
        for (int unit = ufirst; unit < total_units; unit += ustep, ++tcount) {
            const int tile = unit % total_tiles, split = unit / total_tiles;
            int m_blk, n_blk;
            tile_coords(g, tile, m_blk, n_blk);
            const uint32_t acc = tcount & 1u, acc_ph = (tcount >> 1) & 1u;
            if (abort_flag || !mbar_wait(&tfull_bar[acc], acc_ph, g.status)) {
                abort_flag = 1;
                break;
            }
            tc_fence_after();
            // The bias of the tile's BN columns in registers, BPL per lane (lane l: columns
            // l * BPL ..), loaded once per tile and handed to every row with shuffles: each
            // 32-column unit's bias load otherwise waited a full round trip to L2 behind the
            // weight stream, one unit after another (measured: fc1 2048 x 8192 + bias + GELU at
            // M = 761, 51.0 -> 40.9 us).  (Holding the next unit's residual or multiplier in
            // registers as well cost the mainloop registers: the plain prefill GEMMs lost 14 %.)
            constexpr int BPL = BN / 32;
            const bool reg_bias = g.bias && g.splits == 1 && csplit == 1;
            float breg[BPL];
            if (reg_bias) {
                const int c0 = n_blk * BN + lane * BPL;
#pragma unroll
                for (int i = 0; i < BPL; ++i) breg[i] = c0 + i < g.N ? bias_at(g.bias, g.bias_type, c0 + i) : 0.0f;
            }
#pragma unroll 1
            for (int cm = 0; cm < MT * (BN / 32); ++cm) {
            const int mt = cm / (BN / 32), cc = cm % (BN / 32);
            const int row = m_blk * TBM + ((int)rank * MT + mt) * BM + q * 32 + lane;
            {
                float v[32];
                tmem_ld_32x32b_x32(tmem_base + ((uint32_t)(q * 32) << 16) + acc * (MT * BN) + mt * BN + cc * 32, v);
                const int n0 = n_blk * BN + cc * 32;
                if (csplit > 1) {
                    // cluster split-K: this CTA's fp32 partial into its shared memory (the ring
                    // is idle: the tile's MMAs have all completed), summed after the cluster sync
                    float* red = reinterpret_cast<float*>(smem) + (q * 32 + lane) * (BN + 4) + cc * 32;
#pragma unroll
                    for (int j = 0; j < 8; ++j)
                        reinterpret_cast<float4*>(red)[j] = make_float4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
                    continue;
                }
                if (g.splits > 1) {
                    // split-K: this CTA's fp32 partial of the tile
                    if (row < g.M && n0 < g.N) {
                        float* pr = g.partials + ((size_t)split * g.M + row) * g.N + n0;
                        if ((g.N & 3) == 0 && n0 + 32 <= g.N) {
#pragma unroll
                            for (int j = 0; j < 8; ++j)
                                reinterpret_cast<float4*>(pr)[j] = make_float4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
                        } else {
#pragma unroll
                            for (int i = 0; i < 32; ++i)
                                if (n0 + i < g.N) pr[i] = v[i];
                        }
                    }
                    continue;
                }
                if (reg_bias && n0 < g.N) {
                    // column cc * 32 + j of the tile is lane (cc * 32 + j) / BPL's value (j % BPL)
#pragma unroll
                    for (int j = 0; j < 32; ++j) v[j] += __shfl_sync(0xffffffffu, breg[j % BPL], cc * (32 / BPL) + j / BPL);
                } else if (g.bias && n0 < g.N) {
                    // 16-byte loads, the type chosen once per eight values (columns past N add 0)
#pragma unroll
                    for (int q8 = 0; q8 < 4; ++q8) {
                        float b[8];
                        load8(g.bias, g.bias_type, 0, 0, n0 + 8 * q8, g.N, b);
#pragma unroll
                        for (int i = 0; i < 8; ++i) v[8 * q8 + i] += b[i];
                    }
                }
                if (epilogue_active(g.epi) && row < g.M && n0 < g.N) epilogue_row32(g.epi, row, n0, g.N, v);
                if (row < g.M && n0 < g.N) {
                    const size_t base = (size_t)row * g.ldc + n0;
                    if (vec_ok && n0 + 32 <= g.N && g.c_type != MGPU_F32) {
                        uint4* dst = reinterpret_cast<uint4*>(reinterpret_cast<uint16_t*>(g.C) + base);
#pragma unroll
                        for (int j = 0; j < 4; ++j) {
                            uint32_t o[4];
#pragma unroll
                            for (int h = 0; h < 4; ++h)
                                o[h] = (g.c_type == MGPU_BF16) ? pack2<__nv_bfloat16>(v[8 * j + 2 * h], v[8 * j + 2 * h + 1])
                                                               : pack2<__half>(v[8 * j + 2 * h], v[8 * j + 2 * h + 1]);
                            dst[j] = make_uint4(o[0], o[1], o[2], o[3]);
                        }
                    } else if (vec_ok && n0 + 32 <= g.N) {
                        float4* dst = reinterpret_cast<float4*>(reinterpret_cast<float*>(g.C) + base);
#pragma unroll
                        for (int j = 0; j < 8; ++j) dst[j] = make_float4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
                    } else {
#pragma unroll
                        for (int i = 0; i < 32; ++i)
                            if (n0 + i < g.N) store_out(g.C, g.c_type, base + i, v[i]);
                    }
                }
            }
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) {
                if constexpr (kPair) mbar_arrive_cluster(tempty0_cl + 8u * acc);
                else mbar_arrive(&tempty_bar[acc]);
            }
            if (g.splits > 1 && csplit == 1) {
                // The last of the tile's splits to arrive sums the partials in split order
                // (deterministic) and writes C; it leaves the ticket at zero for the next call.
                __threadfence();
                named_barrier_sync(2, 128);
                if (warp == 2 && lane == 0) {
                    const unsigned int t = atomicAdd(&g.tickets[tile], 1u);
                    const int last = t == (unsigned int)(g.splits - 1);
                    if (last) g.tickets[tile] = 0u;
                    split_last = last;
                }
                named_barrier_sync(2, 128);
                if (split_last) {
                    // all 128 epilogue threads over the tile's rows x columns, 4 columns each
                    __threadfence();
                    const int et = (warp - 2) * 32 + lane;
                    const int row0 = m_blk * TBM, n_base = n_blk * BN;
                    const int rows = min(TBM, g.M - row0), cols = min(BN, g.N - n_base);
                    const int c4 = (cols + 3) / 4;
                    const bool vec = (g.N & 3) == 0;
                    for (int idx = et; idx < rows * c4; idx += 128) {
                        const int row = row0 + idx / c4, n = n_base + (idx % c4) * 4;
                        float sum[4] = {0.0f, 0.0f, 0.0f, 0.0f};
                        for (int sp = 0; sp < g.splits; ++sp) {
                            const float* src = g.partials + ((size_t)sp * g.M + row) * g.N + n;
                            if (vec) {
                                const float4 v4 = __ldcg(reinterpret_cast<const float4*>(src));
                                sum[0] += v4.x;
                                sum[1] += v4.y;
                                sum[2] += v4.z;
                                sum[3] += v4.w;
                            } else {
                                for (int i = 0; i < 4; ++i)
                                    if (n + i < n_base + cols) sum[i] += __ldcg(src + i);
                            }
                        }
                        for (int i = 0; i < 4; ++i) {
                            if (n + i >= n_base + cols) break;
                            float o = sum[i];
                            if (g.bias) o += bias_at(g.bias, g.bias_type, n + i);
                            o = epilogue_finish(g.epi, row, n + i, o);
                            store_out(g.C, g.c_type, (size_t)row * g.ldc + n + i, o);
                        }
                    }
                }
                named_barrier_sync(2, 128);
            }
        }
    } else if constexpr (is_packed_tma(BMODE)) {
        // ---------------------------------------------------------------- dequantisers (TMA-staged)
        // Groups of 256 k (8 GGUF blocks per row) arrive by TMA in a two-slot ring; thread
        // (row r, part h) decodes SPT of the group's four MMA k-stages of its row (stages
        // h * SPT ..; two blocks each), straight from shared memory into the swizzled B tiles.
        // 128 B rows per CTA: two stages per thread; 64 rows: one.
        static_assert(BNC == 128 || BNC == 64, "packed mode stages 64 or 128 B rows per CTA");
        constexpr int SPT = BNC / 64;      // k-stages per thread per group
        static_assert(SPT * (256 / BNC) == 4, "threads x stages cover the group's four k-stages");
        static_assert((BNC / 32) * (256 / BNC) == kDqWarps, "each k-stage is decoded by BNC / 32 warps");
        constexpr int GB = group_bytes(BMODE);
        constexpr int HB = GB * SPT / 4;   // bytes of the row this thread decodes
        constexpr int HW = HB / 4;         // as 32-bit words (Q8_0: 34 / 17, Q4_0: 18 / 9)
        constexpr int BB = is_q4_mode(BMODE) ? 18 : 34;
        constexpr int NW = is_q4_mode(BMODE) ? 5 : 9;
        const int dt = tid - 192;
        const int r = dt & (BNC - 1), h = dt / BNC;
        uint8_t* pk = smem + S * SB;
        const int groups = g.kb_per_split / 4;  // 256-k groups per unit
        const int my_units = total_units > ufirst ? (total_units - 1 - ufirst) / ustep + 1 : 0;
        // cluster split-K: one unit, whose K slice may be the shorter last one
        const int kb_first = (ufirst / total_tiles) * g.kb_per_split;
        const uint32_t n_groups = csplit > 1 ? (uint32_t)(my_units ? (kb_end(kb_first) - kb_first) / 4 : 0)
                                             : (uint32_t)my_units * (uint32_t)groups;
        auto issue_group = [&](uint32_t gi) {
            const int unit = ufirst + (int)(gi / groups) * ustep;
            const int tile = unit % total_tiles;
            const int grp = (unit / total_tiles) * groups + (int)(gi % groups);
            const uint32_t slot = gi & 1u;
            if (!mbar_wait(&pk_empty[slot], ((gi >> 1) & 1u) ^ 1u, g.status)) return false;
            mbar_arrive_expect_tx(&pk_full[slot], (uint32_t)(BNC * GB));
            // this CTA's B rows of the tile (pair mode: rows BNC * rank ..), into its own ring
            tma_load_2d(pk + slot * (BNC * GB), &tmB, grp * (GB / 2), tile_n_blk(g, tile) * BN + (int)rank * BNC,
                        &pk_full[slot]);
            return true;
        };
        if (dt == 0 && n_groups > 0 && !issue_group(0)) abort_flag = 1;
        for (uint32_t gi = 0; gi < n_groups && !abort_flag; ++gi) {
            if (dt == 0 && gi + 1 < n_groups && !issue_group(gi + 1)) { abort_flag = 1; break; }
            const uint32_t slot = gi & 1u;
            if (!mbar_wait(&pk_full[slot], (gi >> 1) & 1u, g.status)) { abort_flag = 1; break; }
            uint32_t w[HW];
            const uint8_t* src = pk + slot * (BNC * GB) + r * GB + h * HB;
            if constexpr (HB % 8 == 0) {
#pragma unroll
                for (int i = 0; i < HW / 2; ++i) {
                    const uint2 v = reinterpret_cast<const uint2*>(src)[i];
                    w[2 * i] = v.x;
                    w[2 * i + 1] = v.y;
                }
            } else {
#pragma unroll
                for (int i = 0; i < HW; ++i) w[i] = reinterpret_cast<const uint32_t*>(src)[i];
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&pk_empty[slot]);
#pragma unroll
            for (int jj = 0; jj < SPT; ++jj) {
                const uint32_t it = gi * 4 + SPT * h + jj;
                const uint32_t s = it % S, ph = (it / S) & 1u;
                if (!mbar_wait(&empty_bar[s], ph ^ 1u, g.status)) {
                    abort_flag = 1;
                    break;
                }
                uint8_t* row_base = smem + s * SB + AB + (r >> 3) * 1024 + (r & 7) * 128;
#pragma unroll
                for (int half = 0; half < 2; ++half) {
                    constexpr int dummy = 0;
                    (void)dummy;
                    const int bi = 2 * jj + half;  // block within this thread's half row
                    RawBlock<NW> rb;
                    rb.valid = true;
                    // block bi starts at byte BB * bi of the half row (compile-time word / parity)
#pragma unroll
                    for (int q = 0; q < NW; ++q) rb.w[q] = w[(BB * bi) / 4 + q];
                    rb.par = (uint32_t)((BB * bi) & 3);
                    uint4* dst[4];
#pragma unroll
                    for (int j = 0; j < 4; ++j) dst[j] = reinterpret_cast<uint4*>(row_base + (((half * 4 + j) ^ (r & 7)) << 4));
                    decode_store<BMODE, T, NW>(rb, dst);
                }
                fence_proxy_async_smem();
                __syncwarp();
                if (lane == 0) {
                    if constexpr (kPair) mbar_arrive_cluster(full0_cl + 8u * s);
                    else mbar_arrive(&full_bar[s]);
                }
            }
        }
    } else if constexpr (kQuant) {
        // ---------------------------------------------------------------- dequantisers
        // Stage `it` of this CTA is k-block (it % kb_per_split) of its (it / kb_per_split)-th
        // unit (a tile, or one split of it).  The
        // packed blocks of stage it+3 are loaded into registers before stage it is decoded,
        // so three stages of global-memory latency are in flight per thread.
        constexpr int BB = is_q4_mode(BMODE) ? 18 : 34;
        constexpr int NW = is_q4_mode(BMODE) ? 5 : 9;
        constexpr int UPT = (2 * BN) / (kDqWarps * 32);  // blocks (units) per thread per stage
        constexpr int NPRE = 3;
        const int dt = tid - 192;
        const int nbk = (g.K + 31) / 32;  // blocks per row
        const int my_units = total_units > (int)blockIdx.x ? (total_units - 1 - (int)blockIdx.x) / (int)gridDim.x + 1 : 0;
        const uint32_t n_stages = (uint32_t)my_units * (uint32_t)g.kb_per_split;
        RawBlock<NW> raw[NPRE][UPT];
        auto load_stage = [&](RawBlock<NW>(&dst)[UPT], uint32_t it) {
            const bool live = it < n_stages;
            const int unit = (int)blockIdx.x + (int)(it / g.kb_per_split) * (int)gridDim.x;
            const int tile = unit % total_tiles;
            const int kb = (unit / total_tiles) * g.kb_per_split + (int)(it % g.kb_per_split);
            const int n_blk = live ? tile_n_blk(g, tile) : 0;
#pragma unroll
            for (int v = 0; v < UPT; ++v) {
                const int u = dt + v * kDqWarps * 32;
                const int n = n_blk * BN + (u >> 1);
                const int kq = kb * 2 + (u & 1);
                const bool ok = live && n < g.N && kq < nbk;
                load_block<NW, BB>(dst[v], g.Bq + (size_t)n * g.bq_row_bytes + (size_t)kq * BB, g.bq_end, ok);
            }
        };
        auto decode_stage = [&](RawBlock<NW>(&src)[UPT], uint32_t it) -> bool {
            const uint32_t s = it % S, ph = (it / S) & 1u;
            if (!mbar_wait(&empty_bar[s], ph ^ 1u, g.status)) return false;
            uint8_t* b_dst = smem + s * SB + AB;
#pragma unroll
            for (int v = 0; v < UPT; ++v) {
                const int u = dt + v * kDqWarps * 32;
                const int r = u >> 1, half = u & 1;
                uint8_t* row_base = b_dst + (r >> 3) * 1024 + (r & 7) * 128;
                uint4* dst[4];
#pragma unroll
                for (int j = 0; j < 4; ++j) dst[j] = reinterpret_cast<uint4*>(row_base + (((half * 4 + j) ^ (r & 7)) << 4));
                decode_store<BMODE, T, NW>(src[v], dst);
            }
            fence_proxy_async_smem();
            __syncwarp();
            if (lane == 0) mbar_arrive(&full_bar[s]);
            return true;
        };
#pragma unroll
        for (int p = 0; p < NPRE; ++p) load_stage(raw[p], (uint32_t)p);
        for (uint32_t it = 0; it < n_stages && !abort_flag; it += NPRE) {
#pragma unroll
            for (int p = 0; p < NPRE; ++p) {
                if (it + p < n_stages) {
                    RawBlock<NW> cur[UPT];
#pragma unroll
                    for (int v = 0; v < UPT; ++v) cur[v] = raw[p][v];
                    load_stage(raw[p], it + p + NPRE);
                    if (!decode_stage(cur, it + p)) { abort_flag = 1; break; }
                }
            }
        }
    }

    tc_fence_before();
    __syncthreads();
    if (csplit > 1) {
        // Cluster split-K: every CTA's partial (its 128 rows x BN) is in its shared memory.
        // The csplit CTAs holding the same rows (same place in their pairs) sum them, each a
        // share of the rows, reading the others' over DSMEM in K-slice order (deterministic),
        // then add the bias, convert and store.
        cluster_sync_all();
        constexpr int RP = BN + 4;  // partial row pitch in floats
        constexpr int C4 = BN / 4;
        const int tile = ufirst % total_tiles;
        int m_blk, n_blk;
        tile_coords(g, tile, m_blk, n_blk);
        const int rows_per = (BM + csplit - 1) / csplit;
        const int r0 = (int)ksplit * rows_per, r1 = min(BM, r0 + rows_per);
        uint32_t src[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) src[i] = i < csplit ? cluster_addr(smem, (uint32_t)i * CG + rank) : 0u;
        const bool vec = (g.ldc % 4 == 0) && ((reinterpret_cast<uintptr_t>(g.C) & 15) == 0);
        for (int idx = tid; idx < (r1 - r0) * C4; idx += (int)blockDim.x) {
            const int lr = r0 + idx / C4, c = (idx % C4) * 4;
            const int row = m_blk * TBM + (int)rank * BM + lr, n = n_blk * BN + c;
            if (row >= g.M || n >= g.N) continue;
            const uint32_t off = (uint32_t)((lr * RP + c) * 4);
            float4 part[8];
#pragma unroll
            for (int i = 0; i < 8; ++i)
                if (i < csplit) part[i] = ld_cluster_f4(src[i] + off);
            float o[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll
            for (int i = 0; i < 8; ++i)
                if (i < csplit) {
                    o[0] += part[i].x;
                    o[1] += part[i].y;
                    o[2] += part[i].z;
                    o[3] += part[i].w;
                }
            if (g.bias) {
#pragma unroll
                for (int j = 0; j < 4; ++j)
                    if (n + j < g.N) o[j] += bias_at(g.bias, g.bias_type, n + j);
            }
            if (epilogue_active(g.epi)) {
#pragma unroll
                for (int j = 0; j < 4; ++j)
                    if (n + j < g.N) o[j] = epilogue_finish(g.epi, row, n + j, o[j]);
            }
            const size_t base = (size_t)row * g.ldc + n;
            if (vec && n + 4 <= g.N) {
                if (g.c_type == MGPU_F32) {
                    *reinterpret_cast<float4*>(reinterpret_cast<float*>(g.C) + base) = make_float4(o[0], o[1], o[2], o[3]);
                } else {
                    const uint2 w = g.c_type == MGPU_BF16
                                        ? make_uint2(pack2<__nv_bfloat16>(o[0], o[1]), pack2<__nv_bfloat16>(o[2], o[3]))
                                        : make_uint2(pack2<__half>(o[0], o[1]), pack2<__half>(o[2], o[3]));
                    *reinterpret_cast<uint2*>(reinterpret_cast<uint16_t*>(g.C) + base) = w;
                }
            } else {
                for (int j = 0; j < 4 && n + j < g.N; ++j) store_out(g.C, g.c_type, base + j, o[j]);
            }
        }
    }
    // pair mode / cluster split-K: no CTA releases its TMEM or shared memory (which the pair's
    // MMAs or the cluster's sums read) before all are done
    if (kPair || csplit > 1) cluster_sync_all();
    if (warp == 1) {
        tc_fence_after();
        if constexpr (kPair) tmem_dealloc_pair(tmem_base, kTmemCols);
        else tmem_dealloc(tmem_base, kTmemCols);
    }
}

// ------------------------------------------------------------------ host side --------
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn get_encode_fn() {
    static EncodeTiledFn fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &p, 12000, cudaEnableDefault, &q) ==
                cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiledFn>(p);
    });
    return fn;
}

// 2-D map over a 16-bit row-major matrix: inner dim `cols` (contiguous), outer `rows`,
// row pitch `ld` elements, box {box_cols, box_rows}, 128B swizzle.
bool make_map(CUtensorMap* m, const void* ptr, int64_t rows, int64_t cols, int64_t ld, int box_cols, int box_rows) {
    EncodeTiledFn enc = get_encode_fn();
    if (!enc) return false;
    cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
    cuuint64_t strides[1] = {(cuuint64_t)(ld * 2)};
    cuuint32_t box[2] = {(cuuint32_t)box_cols, (cuuint32_t)box_rows};
    cuuint32_t estr[2] = {1, 1};
    return enc(m, CU_TENSOR_MAP_DATA_TYPE_UINT16, 2, const_cast<void*>(ptr), dims, strides, box, estr,
               CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// 2-D map over 16-bit units without swizzle (packed GGUF rows): inner dim `cols`, outer
// `rows`, row pitch `ld` units, box {box_cols, box_rows}.
bool make_map_plain(CUtensorMap* m, const void* ptr, int64_t rows, int64_t cols, int64_t ld, int box_cols,
                    int box_rows) {
    EncodeTiledFn enc = get_encode_fn();
    if (!enc) return false;
    cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
    cuuint64_t strides[1] = {(cuuint64_t)(ld * 2)};
    cuuint32_t box[2] = {(cuuint32_t)box_cols, (cuuint32_t)box_rows};
    cuuint32_t estr[2] = {1, 1};
    return enc(m, CU_TENSOR_MAP_DATA_TYPE_UINT16, 2, const_cast<void*>(ptr), dims, strides, box, estr,
               CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

template <int BN, int BMODE, typename T, int MT = 1, int CG = 1>
cudaError_t launch_gemm(const mgpu_k::LaunchCtx& c, const CUtensorMap& ma, const CUtensorMap& mb, const GemmArgs& g) {
    auto kern = gemm_tc_kernel<BN, BMODE, T, MT, CG>;
    const int smem = smem_bytes(BN, BMODE, MT, CG);
    // The shared-memory opt-in is a per-device function attribute: set it once per device.
    static std::atomic<uint64_t> configured{0};
    int ordinal = 0;
    cudaError_t e = cudaGetDevice(&ordinal);
    if (e != cudaSuccess) return e;
    const uint64_t bit = ordinal < 64 ? (1ull << ordinal) : 0ull;
    if (!bit || !(configured.load(std::memory_order_acquire) & bit)) {
        e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
        if (e != cudaSuccess) return e;
        configured.fetch_or(bit, std::memory_order_acq_rel);
    }
    const int units = g.tiles_m * g.tiles_n * g.splits;
    cudaLaunchConfig_t cfg = {};
    cfg.blockDim = dim3(gemm_threads(BMODE));
    cfg.dynamicSmemBytes = smem;
    cfg.stream = c.stream;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    int grid = units < c.sm_count ? units : c.sm_count;
    if (g.csplit > 1) {
        // cluster split-K: one cluster of CG x csplit CTAs per tile, all tiles launched at once
        if (MT != 1 || g.csplit * CG > 8 || BM * (BN + 4) * 4 > smem - 1024) return cudaErrorInvalidValue;
        attr[1].id = cudaLaunchAttributeClusterDimension;
        attr[1].val.clusterDim.x = CG * g.csplit;
        attr[1].val.clusterDim.y = 1;
        attr[1].val.clusterDim.z = 1;
        cfg.numAttrs = 2;
        cfg.gridDim = dim3(g.tiles_m * g.tiles_n * CG * g.csplit);
        return cudaLaunchKernelEx(&cfg, kern, ma, mb, g);
    }
    if constexpr (CG == 2) {
        attr[1].id = cudaLaunchAttributeClusterDimension;
        attr[1].val.clusterDim.x = 2;
        attr[1].val.clusterDim.y = 1;
        attr[1].val.clusterDim.z = 1;
        cfg.numAttrs = 2;
        cfg.gridDim = dim3(2);
        // clusters that fit on the device at once (per device, for this instantiation)
        static std::atomic<int> cached[64];
        int clusters = ordinal < 64 ? cached[ordinal].load(std::memory_order_acquire) : 0;
        if (clusters <= 0) {
            if (cudaOccupancyMaxActiveClusters(&clusters, kern, &cfg) != cudaSuccess || clusters <= 0) {
                (void)cudaGetLastError();
                clusters = c.sm_count / 2;
            }
            if (ordinal < 64) cached[ordinal].store(clusters, std::memory_order_release);
        }
        grid = 2 * (units < clusters ? units : clusters);
    }
    cfg.gridDim = dim3(grid);
    return cudaLaunchKernelEx(&cfg, kern, ma, mb, g);
}

template <int BN, typename T>
cudaError_t launch_mode(const mgpu_k::LaunchCtx& c, int bmode, int mt, int cg, const CUtensorMap& ma, const CUtensorMap& mb,
                        const GemmArgs& g) {
    switch (bmode) {
        case B_TMA_K:
            return cg == 2 ? launch_gemm<BN, B_TMA_K, T, 1, 2>(c, ma, mb, g) : launch_gemm<BN, B_TMA_K, T>(c, ma, mb, g);
        case B_TMA_MN:
            return cg == 2 ? launch_gemm<BN, B_TMA_MN, T, 1, 2>(c, ma, mb, g) : launch_gemm<BN, B_TMA_MN, T>(c, ma, mb, g);
        case B_Q8: return launch_gemm<BN, B_Q8, T>(c, ma, mb, g);
        case B_Q4: return launch_gemm<BN, B_Q4, T>(c, ma, mb, g);
        case B_Q8_TMA:
            if (cg == 2) return launch_gemm<BN, B_Q8_TMA, T, 1, 2>(c, ma, mb, g);
            if constexpr (BN == 128)
                return mt == 2 ? launch_gemm<BN, B_Q8_TMA, T, 2>(c, ma, mb, g) : launch_gemm<BN, B_Q8_TMA, T, 1>(c, ma, mb, g);
            return cudaErrorInvalidValue;
        default:
            if (cg == 2) return launch_gemm<BN, B_Q4_TMA, T, 1, 2>(c, ma, mb, g);
            if constexpr (BN == 128)
                return mt == 2 ? launch_gemm<BN, B_Q4_TMA, T, 2>(c, ma, mb, g) : launch_gemm<BN, B_Q4_TMA, T, 1>(c, ma, mb, g);
            return cudaErrorInvalidValue;
    }
}

bool is16(int t) { return t == MGPU_F16 || t == MGPU_BF16; }

}  // namespace

namespace mgpu_k {

const char* gemm_check(const GemmOperand& A, const GemmOperand& B, const GemmOperand& C, int M, int N, int K) {
    if (M <= 0 || N <= 0 || K <= 0) return "M, N, K must be positive";
    if (!is16(A.type)) return "A must be fp16 or bf16";
    if (!(is16(C.type) || C.type == MGPU_F32)) return "C must be fp16, bf16 or fp32";
    if (C.ld < N) return "C row pitch smaller than N";
    if ((reinterpret_cast<uintptr_t>(A.ptr) & 15) || (A.ld * 2) % 16) return "A must be 16-byte aligned with a row pitch that is a multiple of 8 elements";
    if (A.ld < K) return "A row pitch smaller than K";
    if (B.type == MGPU_Q4_0 || B.type == MGPU_Q8_0) {
        if (B.layout != MGPU_LAYOUT_NK) return "quantised B must be in GGUF [N][K/32] layout";
        if (K % 32) return "quantised B needs K % 32 == 0";
        if (B.ld & 1) return "quantised row bytes must be even";
        return nullptr;
    }
    if (B.type != A.type) return "A and B must have the same 16-bit type";
    if ((reinterpret_cast<uintptr_t>(B.ptr) & 15) || (B.ld * 2) % 16) return "B must be 16-byte aligned with a row pitch that is a multiple of 8 elements";
    if (B.layout == MGPU_LAYOUT_NK && B.ld < K) return "B row pitch smaller than K";
    if (B.layout == MGPU_LAYOUT_KN && B.ld < N) return "B row pitch smaller than N";
    if (!get_encode_fn()) return "cuTensorMapEncodeTiled unavailable";
    return nullptr;
}

}  // namespace

namespace {
// Clusters of `csize` CTAs (one CTA per SM: every instantiation takes ~200 KB of shared
// memory) that the current device holds at once.  Clusters are placed within a GPC, so this
// is below sm_count / csize for csize > 2 (measured on B200: 74, 45, 33, 22, 15 for 2, 3, 4,
// 6, 8).  Queried once per device and size.
int cluster_capacity(int sm_count, int csize) {
    if (csize <= 1) return sm_count;
    static std::atomic<int> cache[64][9];
    int ordinal = 0;
    if (csize > 8 || cudaGetDevice(&ordinal) != cudaSuccess || ordinal >= 64) return sm_count / csize;
    int n = cache[ordinal][csize].load(std::memory_order_acquire);
    if (n > 0) return n;
    auto kern = gemm_tc_kernel<128, B_TMA_K, __nv_bfloat16, 1, 1>;
    const int smem = smem_bytes(128, B_TMA_K);
    n = 0;
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) == cudaSuccess) {
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3(csize);
        cfg.blockDim = dim3(gemm_threads(B_Q8_TMA));
        cfg.dynamicSmemBytes = smem;
        cudaLaunchAttribute attr[1];
        attr[0].id = cudaLaunchAttributeClusterDimension;
        attr[0].val.clusterDim.x = csize;
        attr[0].val.clusterDim.y = 1;
        attr[0].val.clusterDim.z = 1;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
        if (cudaOccupancyMaxActiveClusters(&n, kern, &cfg) != cudaSuccess) n = 0;
    }
    (void)cudaGetLastError();
    if (n <= 0) n = sm_count / csize / 2;  // conservative when the query fails
    cache[ordinal][csize].store(n, std::memory_order_release);
    return n;
}
}  // namespace

namespace mgpu_k {

GemmPlan plan_gemm(const LaunchCtx& c, const GemmOperand& A, const GemmOperand& B, int M, int N, int K) {
    (void)A;
    GemmPlan p;
    const bool quant = B.type == MGPU_Q8_0 || B.type == MGPU_Q4_0;
    // Packed rows can be staged by TMA in 256-k groups when every group starts on a 16-byte
    // boundary: K % 256 == 0, row pitch % 16 == 0 and a 16-byte aligned base.
    const bool packed_ok = quant && K % 256 == 0 && B.ld % 16 == 0 && (reinterpret_cast<uintptr_t>(B.ptr) & 15) == 0 &&
                           B.ld == (int64_t)(K / 32) * (B.type == MGPU_Q4_0 ? 18 : 34);
    if (B.type == MGPU_Q8_0) p.bmode = packed_ok ? B_Q8_TMA : B_Q8;
    else if (B.type == MGPU_Q4_0) p.bmode = packed_ok ? B_Q4_TMA : B_Q4;
    else p.bmode = (B.layout == MGPU_LAYOUT_NK) ? B_TMA_K : B_TMA_MN;

    // Pick the tiling by its estimated makespan in SM cycles: waves x 16-k steps x step cost +
    // a fixed cost per CTA (pipeline fill, epilogue; the persistent CTAs overlap a tile's
    // epilogue with the next tile).  A step's MMA cost on one SM is bounded by the tensor
    // core's shared-memory operand reads, ~64 bytes per cycle (4 KB of A per 128 rows, 32
    // bytes per B column this CTA holds), and by its rate (BN / 2 cycles per 128 rows of this
    // CTA); a quantised B also costs ~1 cycle per B row this CTA decodes, overlapped with the
    // MMAs.  Measured steps run ~1.7x that bound (pipeline latency) and the fixed cost is
    // ~6000 cycles for one CTA per tile, ~11000 for packed and ~14000 for dense pairs.  Candidates: one CTA per 128 x BN tile; one CTA per 256 x 128 tile (two
    // accumulators sharing each decoded B stage, packed quantised B only); a CTA pair per
    // 256 x BN tile (cta_group::2, A and B staged by TMA).  Dense pairs start and finish more
    // slowly (measured: SigLIP B = 1 shapes ~1 us slower as pairs, B = 8 shapes 10-50 % faster);
    // packed pairs won on every M = 761 prefill shape.
    struct Cand {
        int bn, mt, cg;
    };
    const bool packed = is_packed_tma(p.bmode);
    const Cand dense_c[4] = {{128, 1, 1}, {256, 1, 1}, {128, 1, 2}, {256, 1, 2}};
    const Cand packed_c[4] = {{128, 1, 1}, {128, 2, 1}, {128, 1, 2}, {256, 1, 2}};
    const Cand* cands = packed ? packed_c : dense_c;
    const int n_cands = quant && !packed ? 1 : 4;  // GGUF rows read with plain loads: 128 x 128
    const double steps = (double)((K + 15) / 16);
    double best = 0.0;
    p.BN = 128;
    p.mt = 1;
    p.cg = 1;
    // Cluster split-K (one CTA or pair per K slice, csplit of them per cluster, one tile per
    // cluster, partials summed over DSMEM) when the tiles leave SMs idle.  Clusters are not
    // persistent, so every wave of them pays the fill, drain and sums (~12000 cycles
    // measured); how many clusters fit at once is queried from the device.
    const int num_kb = (K + BK - 1) / BK;
    const int gran = packed ? 4 : 1;  // k-blocks per slice unit (packed B: whole 256-k groups)
    p.csplit = 1;
    for (int i = 0; i < n_cands; ++i) {
        const Cand& cd = cands[i];
        if (cd.cg == 2 && M <= BM) continue;  // a pair needs two 128-row blocks
        const long rows = 128L * cd.mt * cd.cg;
        const long tiles = ((M + rows - 1) / rows) * (long)((N + cd.bn - 1) / cd.bn);
        const long slots = cd.cg == 2 ? c.sm_count / 2 : c.sm_count;
        const double bytes = 4096.0 * cd.mt + 32.0 * (cd.bn / cd.cg);
        const double rate = cd.mt * cd.bn / 2.0;
        double step = bytes / 64.0 > rate ? bytes / 64.0 : rate;
        if (quant && (double)(cd.bn / cd.cg) > step) step = (double)(cd.bn / cd.cg);
        step *= 1.7;
        const double fixed = cd.cg == 1 ? 6000.0 : quant ? 11000.0 : 14000.0;
        const bool split_ok = cd.mt == 1 && M > 16 && (packed || !quant) &&
                              BM * (cd.bn + 4) * 4 <= smem_bytes(cd.bn, p.bmode, 1, cd.cg) - 1024;
        for (int cs = 1; cs <= 8 / cd.cg; ++cs) {
            double cost;
            if (cs == 1) {
                cost = (double)((tiles + slots - 1) / slots) * steps * step + fixed;
            } else {
                if (!split_ok) break;
                const int kbps = (num_kb / gran + cs - 1) / cs * gran;
                if ((cs - 1) * kbps >= num_kb) break;  // every slice gets some K
                const long cap = cluster_capacity(c.sm_count, cd.cg * cs);
                if (cap <= 0) break;
                cost = (double)((tiles + cap - 1) / cap) * (kbps * 4.0 * step + 12000.0);
            }
            if ((i == 0 && cs == 1) || cost < best) {
                best = cost;
                p.BN = cd.bn;
                p.mt = cd.mt;
                p.cg = cd.cg;
                p.csplit = cs;
            }
        }
    }
    p.tiles_m = (M + BM * p.mt * p.cg - 1) / (BM * p.mt * p.cg);
    p.tiles_n = (N + p.BN - 1) / p.BN;
    p.num_kb = num_kb;
    if (p.csplit > 1) {
        p.splits = p.csplit;
        p.kb_per_split = (num_kb / gran + p.csplit - 1) / p.csplit * gran;
        return p;
    }
    // Split K for skinny M (M <= 16, e.g. a decode batch of up to 16 sequences) when the tiles
    // fill at most half of the SMs: the largest split count that divides the 256-k groups
    // and keeps splits x tiles within the SMs; each split is at least one group.  (At
    // M = 32 and 128 the fp32 partials cost as much as the idle SMs, measured on the Phi-1.5
    // decode shapes.)
    p.splits = 1;
    const int tiles = p.tiles_m * p.tiles_n;
    if (p.cg == 1 && M <= 16 && K % 256 == 0 && tiles * 2 <= c.sm_count) {  // fp32 partials in global memory
        const int groups = p.num_kb / 4;
        for (int sp = min(groups, c.sm_count / tiles); sp >= 2; --sp)
            if (groups % sp == 0) {
                p.splits = sp;
                break;
            }
    }
    p.kb_per_split = p.num_kb / p.splits;
    return p;
}

size_t gemm_split_bytes(const LaunchCtx& c, const GemmOperand& A, const GemmOperand& B, int M, int N, int K) {
    if (skinny_ok(A, B, M, N, K)) return 0;
    const GemmPlan p = plan_gemm(c, A, B, M, N, K);
    return p.splits > 1 && p.csplit == 1 ? (size_t)p.splits * M * N * sizeof(float) : 0;
}

bool make_tensor_map_u16_3d(CUtensorMap* m, const void* ptr, const int64_t dims[3], const int64_t strides[2],
                            const int box[3]) {
    EncodeTiledFn enc = get_encode_fn();
    if (!enc) return false;
    cuuint64_t d[3] = {(cuuint64_t)dims[0], (cuuint64_t)dims[1], (cuuint64_t)dims[2]};
    cuuint64_t st[2] = {(cuuint64_t)strides[0], (cuuint64_t)strides[1]};
    cuuint32_t b[3] = {(cuuint32_t)box[0], (cuuint32_t)box[1], (cuuint32_t)box[2]};
    cuuint32_t estr[3] = {1, 1, 1};
    return enc(m, CU_TENSOR_MAP_DATA_TYPE_UINT16, 3, const_cast<void*>(ptr), d, st, b, estr,
               CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

cudaError_t gemm(const LaunchCtx& c, const GemmOperand& A, const GemmOperand& B, const GemmOperand& C,
                 const void* bias, int bias_type, int M, int N, int K, const GemmSplitScratch* split,
                 const Epilogue& epi) {
    if (gemm_check(A, B, C, M, N, K)) return cudaErrorInvalidValue;
    // A few sequences against Q4_0 weights (batched decode): the streaming skinny kernel.
    if (skinny_ok(A, B, M, N, K)) return gemm_q4_skinny(c, A, B, C, bias, bias_type, M, N, K, epi);
    GemmPlan p = plan_gemm(c, A, B, M, N, K);
    if (p.splits > 1 && p.csplit == 1 && (!split || !split->tickets || !split->partials ||
                         (size_t)p.splits * M * N > split->max_partials ||
                         (size_t)p.tiles_m * p.tiles_n > split->max_tickets)) {
        p.splits = 1;
        p.kb_per_split = p.num_kb;
    }
    const int bmode = p.bmode, BN = p.BN, mt = p.mt, cg = p.cg, tiles_m = p.tiles_m;

    GemmArgs g;
    g.M = M;
    g.N = N;
    g.K = K;
    g.num_kb = (K + BK - 1) / BK;
    g.tiles_m = tiles_m;
    g.tiles_n = (N + BN - 1) / BN;
    g.C = const_cast<void*>(C.ptr);
    g.ldc = C.ld;
    g.c_type = C.type;
    g.bias = bias;
    g.bias_type = bias_type;
    g.epi = epi;
    g.Bq = nullptr;
    g.bq_row_bytes = 0;
    g.bq_end = nullptr;
    g.status = c.status;
    g.splits = p.splits;
    g.kb_per_split = p.kb_per_split;
    g.tickets = p.splits > 1 && p.csplit == 1 ? split->tickets : nullptr;
    g.partials = p.splits > 1 && p.csplit == 1 ? split->partials : nullptr;
    g.csplit = p.csplit;
    // Tile order: when A is larger than ~3/4 of L2, bands of m-blocks whose A rows take about a
    // third of L2, so that every n-block passes over a band while it is L2-resident instead of
    // each n-block streaming all of A from HBM again (SigLIP at B = 64: A = 107-401 MB).
    {
        const size_t a_block = (size_t)BM * mt * cg * K * 2;  // A rows of one m-block, 16-bit
        const int band = (int)std::max<size_t>(1, (40ull << 20) / a_block);
        g.group_m = (size_t)tiles_m * a_block > (96ull << 20) && band < tiles_m ? band : 0;
    }

    CUtensorMap ma, mb;
    memset(&mb, 0, sizeof(mb));
    if (!make_map(&ma, A.ptr, M, K, A.ld, BK, BM)) return cudaErrorInvalidValue;
    if (bmode == B_TMA_K) {
        if (!make_map(&mb, B.ptr, N, K, B.ld, BK, BN / cg)) return cudaErrorInvalidValue;
    } else if (bmode == B_TMA_MN) {
        if (!make_map(&mb, B.ptr, K, N, B.ld, 64, BK)) return cudaErrorInvalidValue;
    } else {
        g.Bq = reinterpret_cast<const uint8_t*>(B.ptr);
        g.bq_row_bytes = B.ld;
        g.bq_end = g.Bq + (size_t)N * B.ld;
        if (is_packed_tma(bmode)) {
            // the packed rows as a 2-D array of 16-bit units: box = one 256-k group x the B rows
            // one CTA stages
            if (!make_map_plain(&mb, B.ptr, N, B.ld / 2, B.ld / 2, group_bytes(bmode) / 2, BN / cg))
                return cudaErrorInvalidValue;
        }
    }
    const bool bf16 = A.type == MGPU_BF16;
    if (BN == 256)
        return bf16 ? launch_mode<256, __nv_bfloat16>(c, bmode, mt, cg, ma, mb, g)
                    : launch_mode<256, __half>(c, bmode, mt, cg, ma, mb, g);
    return bf16 ? launch_mode<128, __nv_bfloat16>(c, bmode, mt, cg, ma, mb, g)
                : launch_mode<128, __half>(c, bmode, mt, cg, ma, mb, g);
}

}  // namespace mgpu_k
