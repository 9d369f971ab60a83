// gemv.cu - decode-phase GEMV kernels for sm_100a (replaces gemv, src/kernels/gemm.cl:219-270).
//
// gemv_q_stream: y = dequant(W) . x for GGUF Q4_0 / Q8_0 weights kept packed in their
//   [N][K/32] block layout.  Each CTA owns an even share of the rows.  One producer thread
//   streams the CTA's contiguous byte range from HBM into a 2..8-stage shared-memory ring with
//   cp.async.bulk (the 1-D TMA engine, 16-byte granular, no registers held in flight); 16
//   consumer warps decode the 18 / 34-byte blocks out of shared memory.  Each consumer thread
//   owns one 32-element block column for the whole launch; its 32 activations are turned
//   once into 16-bit fixed point (two byte planes), and every block's dot product is exact
//   integer dp4a arithmetic on the packed nibbles / int8s (no per-weight unpacking), scaled
//   once per block in fp32 by the fp16 d.  Row sums are reduced across lanes with a
//   transposing shuffle butterfly.  Up to two CTAs per SM; launched with programmatic dependent
//   launch: the producer starts streaming weights while the previous kernel drains, and the
//   consumers execute griddepcontrol.wait before reading x (which the previous kernel may
//   write).
// gemv_q_mma: the same product with the warp-level integer MMA (mma.sync m16n8k32, u8/s8
//   weights x s8 activation digits, exact s32 sums): two GGUF blocks of 16 rows per MMA pair,
//   rows staged at a padded pitch so fragment loads are conflict-free.  Fewer instructions per
//   block, but in a chain of dependent launches of mixed shapes it measures slower than the
//   dp4a kernel, so the launcher uses it for the K whose block count does not divide 256.
// gemv_nk: dense [N][K] rows (GGUF F32/F16/BF16 tensors): warp per row group, 16-byte loads.
// gemv_kn: dense [K][N] (the reference kernels' orientation): columns across lanes, K split
//   across CTAs; fp32 partials go to scratch and the last CTA of each column tile sums them
//   in split order, so the result is deterministic.
// gemv_q_generic: any K that is a multiple of 32 (row starts need not be 16-byte aligned).
#include <mutex>

#include "common.cuh"
#include "kernels.h"
#include "qdot.cuh"

using namespace mgpu_dev;

namespace {

constexpr int kConsumerThreads = 256;  // gemv_q_mma
constexpr int kGemvThreads = kConsumerThreads + 32;
// gemv_q_stream: 16 consumer warps + the producer warp.  Two such CTAs fit an SM (the current
// GEMV and, under programmatic dependent launch, the next one) at <= 56 registers a thread.
constexpr int kStreamThreads = 512;
constexpr int kStreamBlock = kStreamThreads + 32;
static_assert(kStreamThreads == kRmsThreads, "the fused RMSNorm must reduce like the standalone kernel");
constexpr int kGemvMaxStages = 8;  // ring depth is chosen per shape, up to this
constexpr int kGemvCtasPerSm = 2;                 // at most; see the launcher
constexpr uint32_t kGemvSmemBudget = 100 * 1024;  // per CTA: two CTAs share an SM
// The MMA kernel's budget: two such CTAs plus their 1 KB reservations stay within an SM's
// 228 KB, and a 16-row chunk of K = 8192 Q4_0 rows (74 KB) fits beside its activations.
constexpr uint32_t kGemvMmaSmemBudget = 110 * 1024;

// RMSNorm applied to x by gemv_q_stream's prologue (gemv_q_norm).
struct GemvNorm {
    const void* gamma;
    int gtype;
    float eps;
};

struct GemvQArgs {
    const uint8_t* W;
    const void* x;
    void* y;
    int N;
    int nb;             // blocks per row (K / 32); 32 <= nb <= 256, nb % 32 == 0
    uint32_t row_bytes; // nb * block bytes, a multiple of 16
    uint32_t stage_stride;
    int stages;            // ring depth, 2..kGemvMaxStages
    int chunks_per_flush;  // chunks whose row partials are buffered before one reduction
    int* status;
    const void* gamma;     // RMSNorm weight [K] of gtype applied to x first, or null
    int gtype;
    float eps;
};

template <int QT, int RPT, typename XT, typename YT>
__global__ void __launch_bounds__(kStreamBlock, kGemvCtasPerSm) gemv_q_stream(GemvQArgs a) {
    constexpr int BB = QTraits<QT>::kBlockBytes;
    constexpr int NW = QTraits<QT>::kWords;
    extern __shared__ __align__(1024) uint8_t smem[];
    __shared__ __align__(8) uint64_t full_bar[kGemvMaxStages];
    __shared__ __align__(8) uint64_t empty_bar[kGemvMaxStages];

    const int tid = threadIdx.x;
    const int warp = tid >> 5, lane = tid & 31;
    const int nb = a.nb;
    const int RP = kStreamThreads / nb;  // rows decoded per step
    const int TR = RP * RPT;               // rows per chunk
    const int G = gridDim.x;
    const int r0 = (int)((long long)a.N * blockIdx.x / G);
    const int r1 = (int)((long long)a.N * (blockIdx.x + 1) / G);
    const int nchunks = (r1 - r0 + TR - 1) / TR;

    if (tid == 0) {
        for (int s = 0; s < a.stages; ++s) {
            mbar_init(&full_bar[s], 1);
            mbar_init(&empty_bar[s], kStreamThreads / 32);
        }
        fence_mbar_init();
        // Dependent kernels may be scheduled now; they only read this kernel's output after
        // their own griddepcontrol.wait.
        asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    }
    __syncthreads();

    if (warp == kStreamThreads / 32) {
        // ---- producer: stream this CTA's rows chunk by chunk ----
        // Weights are never written by the preceding kernel, so streaming starts before
        // griddepcontrol.wait and overlaps the previous kernel's tail.
        if (lane == 0) {
            int c = 0, s = 0;
            uint32_t ph = 0;
            for (; c < nchunks; ++c) {
                if (!mbar_wait(&empty_bar[s], ph ^ 1u, a.status)) break;
                const int row = r0 + c * TR;
                const uint32_t bytes = (uint32_t)min(TR, r1 - row) * a.row_bytes;
                mbar_arrive_expect_tx(&full_bar[s], bytes);
                bulk_g2s(smem + (size_t)s * a.stage_stride, a.W + (size_t)row * a.row_bytes, bytes, &full_bar[s]);
                if (++s == a.stages) {
                    s = 0;
                    ph ^= 1u;
                }
            }
            if (c < nchunks) {
                // Timed out: let the copies already issued land before the CTA exits.
                for (int k = max(0, c - a.stages); k < c; ++k)
                    mbar_wait(&full_bar[k % a.stages], (uint32_t)(k / a.stages) & 1u, nullptr);
            }
        }
        return;
    }

    // ---- consumers ----
    // Bring x's lines into L2 before waiting (the CTAs of the grid share them out): the loads
    // after the wait then hit L2 instead of queueing for HBM behind the weight streams
    // (measured: 409 -> 396 us per 97-launch decode step).  A prefetch returns no data to the
    // thread, and L2 is the point of coherence, so lines the preceding kernel still writes
    // are read correctly after griddepcontrol.wait.
    {
        const int nlines = (nb * 32 * (int)sizeof(XT) + 127) / 128;
        for (int l = (int)blockIdx.x + tid * G; l < nlines; l += kStreamThreads * G)
            asm volatile("prefetch.global.L2 [%0];" ::"l"(reinterpret_cast<const char*>(a.x) + (size_t)l * 128));
    }
    // x (and y) may belong to the preceding kernel of the stream: wait for it to complete.
    asm volatile("griddepcontrol.wait;" ::: "memory");
    const int K = nb * 32;
    uint32_t* planes = reinterpret_cast<uint32_t*>(smem + (size_t)a.stages * a.stage_stride);
    float* bscale = reinterpret_cast<float*>(planes + kXPlanes * (K / 4));
    if (a.gamma)
        prepare_x_norm<XT>(reinterpret_cast<const XT*>(a.x), a.gamma, a.gtype, a.eps, K, planes, bscale,
                           bscale + nb, tid, kStreamThreads);  // (the row partials' space, not in use yet)
    else
        prepare_x<XT>(reinterpret_cast<const XT*>(a.x), K, planes, bscale, tid, kStreamThreads);
    named_barrier_sync(1, kStreamThreads);
    const int col = tid % nb;  // block column owned by this thread for the whole launch
    XFixed xf;
    load_xfixed(planes, bscale, K / 4, col, xf);
    const uint32_t par = (uint32_t)(tid * BB) & 3u;  // block starts at byte 0 or 2 of a word
    const uint32_t sel = par ? 0x7654u : 0x5432u;
    const uint32_t dsel = par ? 0x4432u : 0x4410u;
    const uint32_t toff = (uint32_t)(tid * BB) - par;
    const int wpr = nb >> 5;  // warps per row slot
    const int slot = tid / nb;
    float* part = bscale + nb;  // chunks_per_flush * TR * wpr floats
    YT* __restrict__ y = reinterpret_cast<YT*>(a.y);

    int s = 0;
    uint32_t ph = 0;
    for (int c = 0; c < nchunks; ++c) {
        if (!mbar_wait(&full_bar[s], ph, a.status)) return;
        const uint8_t* st = smem + (size_t)s * a.stage_stride + toff;
        float acc[RPT];
#pragma unroll
        for (int i = 0; i < RPT; ++i) {
            const uint32_t* wp = reinterpret_cast<const uint32_t*>(st + i * (kStreamThreads * BB));
            uint32_t w[NW];
#pragma unroll
            for (int q = 0; q < NW; ++q) w[q] = wp[q];
            acc[i] = q_block_dot<QT, NW>(w, sel, dsel, xf);
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty_bar[s]);
        if (++s == a.stages) {
            s = 0;
            ph ^= 1u;
        }

        // Per-warp row partials go to shared memory; rows are reduced across the warps of
        // their slot and written out once per flush (two barriers per flush, not per chunk).
        int ri;
        const float v = warp_reduce_rows<RPT>(acc, lane, ri);
        const int cf = c % a.chunks_per_flush;
        if ((lane & ((32 / RPT) - 1)) == 0) part[(cf * TR + slot + RP * ri) * wpr + (warp % wpr)] = v;
        if (cf == a.chunks_per_flush - 1 || c == nchunks - 1) {
            named_barrier_sync(1, kStreamThreads);
            const int row0 = r0 + (c - cf) * TR;
            const int nrows = min((cf + 1) * TR, r1 - row0);
            for (int r = tid; r < nrows; r += kStreamThreads) {
                float sum = 0.0f;
                for (int w = 0; w < wpr; ++w) sum += part[r * wpr + w];
                y[row0 + r] = from_f32<YT>(sum);
            }
            // the next flush rewrites the partials: wait for every reader (not after the last)
            if (c != nchunks - 1) named_barrier_sync(1, kStreamThreads);
        }
    }
}

// ---- integer tensor-core inner product (mma.sync m16n8k32) ---------------------------
// gemv_q_mma computes the same sums as gemv_q_stream with the warp-level integer MMA:
//   A (16 x 32, u8 for Q4_0 nibbles / s8 for Q8_0 quants) = weights of 16 rows,
//   B (32 x 8, s8) = activation digit planes, D (16 x 8, s32) = exact integer sums.
// Activations are 23-bit fixed point per 32-element block (x = X * 2^(e-22), as above) written
// as three balanced base-256 digits X = p0 + 256 p1 + 65536 p2 with every p in [-128, 127],
// so all of B is signed bytes.  One MMA pair covers two blocks (b = 2p, 2p+1) of 16 rows: in
// the "lo" MMA the k positions 0..15 are elements 0..15 of block 2p and 16..31 elements 0..15
// of block 2p+1; the "hi" MMA does elements 16..31.  B column n < 4 holds plane n of block 2p
// on k < 16 (zeros on k >= 16), column n >= 4 plane n-4 of block 2p+1 on k >= 16; plane 3 is
// zero.  Lane (g, t) of D then holds, for rows g and g+8, the plane sums of block
// 2p + (t >> 1): t even planes 0 and 1, t odd plane 2.  With the nibbles of a Q4_0 quant
// word split into lo (q & 0x0F0F0F0F) and hi ((q >> 4) & 0x0F0F0F0F), the A fragments come
// straight from the packed bytes.  The -8 of Q4_0 enters once per block as -8 sum X,
// added by the plane-2 lanes: sum X (q - 8) = sum X q - 8 sum X.
// Rows are staged with a pitch of row_bytes + 16, which puts the 8 rows a fragment load
// touches on distinct banks.
__device__ __forceinline__ void mma_s8(int (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1, bool u8a) {
    if (u8a)
        asm volatile(
            "mma.sync.aligned.m16n8k32.row.col.s32.u8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
            "{%0,%1,%2,%3};"
            : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
            : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
    else
        asm volatile(
            "mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
            "{%0,%1,%2,%3};"
            : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
            : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// Per-block activation record in shared memory (128 bytes): planes 0, 1, 2 and a zero plane,
// 32 bytes each, with the 8 words of a plane stored in the order 0,4,1,5,2,6,3,7 so that lane
// t's (word t, word t+4) pair is one 8-byte load.  Per-block auxiliaries (16 bytes, fp32):
// {2^(e-22), 0, 2^(e-22) * 65536, -8 sum X / 65536 (Q4_0; 0 for Q8_0)}, read by lane t at
// offset 8 * (t & 1): a lane's plane scale and the offset it adds before scaling.
constexpr int kXRecBytes = 128;
constexpr int kXAuxBytes = 16;

// ITERS = K / 1024 words per thread (256 threads), a compile-time count so that all of the
// thread's loads are issued before the first is used (one L2 round trip, not ITERS).
// (K of 3, 5, 6 or 7 x 1024 takes the runtime-bounded form: ITERS = 8, EXACT = false.)
template <typename XT, bool Q4, int ITERS, bool EXACT>
__device__ __forceinline__ void prepare_x_digits_n(const XT* __restrict__ x, int K, uint8_t* xrec, uint8_t* xaux,
                                                   int tid, int nthreads) {
    constexpr int kMaxIter = ITERS;
    const int iters = EXACT ? ITERS : (K / 4) / nthreads;
    float v[kMaxIter][4];
#pragma unroll
    for (int it = 0; it < kMaxIter; ++it) {
        if (it < iters) {
            const int w = it * nthreads + tid;
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
    for (int it = 0; it < kMaxIter; ++it) {
        if (it < iters) {
            const int w = it * nthreads + tid;
            const int blk = w >> 3, wi = w & 7;
            float amax = fmaxf(fmaxf(fabsf(v[it][0]), fabsf(v[it][1])), fmaxf(fabsf(v[it][2]), fabsf(v[it][3])));
#pragma unroll
            for (int off = 1; off < 8; off <<= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, off));
            int e = 0;
            frexpf(amax, &e);  // the block's |x| < 2^e
            const float up = __int_as_float((127 + 22 - e) << 23);  // 2^(22-e); |e| < 100 for finite x
            // X + 0x808080 = u0 + 256 u1 + 65536 u2 with u in [0, 255] (|X| <= 2^22), and
            // p_i = u_i - 128 = the byte u_i ^ 0x80 read as signed: the balanced digits.
            uint32_t u[4];
            int xs = 0;
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const int X = __float2int_rn(v[it][j] * up);  // |X| <= 2^22
                xs += X;
                u[j] = (uint32_t)(X + 0x808080);
            }
            const uint32_t lo01 = prmt(u[0], u[1], 0x6240u), lo23 = prmt(u[2], u[3], 0x6240u);  // bytes 0, 2
            const uint32_t hi01 = prmt(u[0], u[1], 0x7351u), hi23 = prmt(u[2], u[3], 0x7351u);  // bytes 1, 3
            const uint32_t w0 = prmt(lo01, lo23, 0x5410u) ^ 0x80808080u;  // byte 0 of each X
            const uint32_t w1 = prmt(hi01, hi23, 0x5410u) ^ 0x80808080u;  // byte 1
            const uint32_t w2 = prmt(lo01, lo23, 0x7632u) ^ 0x80808080u;  // byte 2
            uint8_t* rec = xrec + (size_t)blk * kXRecBytes;
            const int slot = wi < 4 ? 2 * wi : 2 * (wi - 4) + 1;
            reinterpret_cast<uint32_t*>(rec)[slot] = w0;
            reinterpret_cast<uint32_t*>(rec + 32)[slot] = w1;
            reinterpret_cast<uint32_t*>(rec + 64)[slot] = w2;
            reinterpret_cast<uint32_t*>(rec + 96)[slot] = 0u;
            if constexpr (Q4) {
#pragma unroll
                for (int off = 1; off < 8; off <<= 1) xs += __shfl_xor_sync(0xffffffffu, xs, off);
            }
            if (wi == 0) {
                const float sc = __int_as_float((127 + e - 22) << 23);  // 2^(e-22)
                uint32_t* aux = reinterpret_cast<uint32_t*>(xaux + (size_t)blk * kXAuxBytes);
                aux[0] = __float_as_uint(sc);
                aux[1] = 0u;
                aux[2] = __float_as_uint(sc * 65536.0f);
                // the Q4_0 offset, -8 sum X, applied once per block by the plane-2 lanes (in
                // units of their 65536 scale)
                aux[3] = __float_as_uint(Q4 ? (float)(-8 * (long long)xs) * (1.0f / 65536.0f) : 0.0f);
            }
        }
    }
}

template <typename XT, bool Q4>
__device__ __forceinline__ void prepare_x_digits(const XT* __restrict__ x, int K, uint8_t* xrec, uint8_t* xaux,
                                                 int tid, int nthreads) {
    switch (K >> 10) {
        case 1: prepare_x_digits_n<XT, Q4, 1, true>(x, K, xrec, xaux, tid, nthreads); break;
        case 2: prepare_x_digits_n<XT, Q4, 2, true>(x, K, xrec, xaux, tid, nthreads); break;
        case 4: prepare_x_digits_n<XT, Q4, 4, true>(x, K, xrec, xaux, tid, nthreads); break;
        case 8: prepare_x_digits_n<XT, Q4, 8, true>(x, K, xrec, xaux, tid, nthreads); break;
        default: prepare_x_digits_n<XT, Q4, 8, false>(x, K, xrec, xaux, tid, nthreads); break;
    }
}

struct GemvMmaArgs {
    const uint8_t* W;
    const void* x;
    void* y;
    int N;
    int nb;                // blocks per row (K / 32); nb % 32 == 0, nb <= 256
    uint32_t row_bytes;    // nb * block bytes, a multiple of 32
    uint32_t pitch;        // row_bytes + 16: shared-memory row pitch
    uint32_t stage_stride;
    int stages;            // ring depth, 2..kGemvMaxStages
    int chunks_per_flush;  // chunks whose row partials are buffered before one reduction
    int* status;
};

constexpr int kMmaWarps = kConsumerThreads / 32;  // 8: each takes 1/8 of K

// RG = 16-row groups per chunk.  Warp w of the consumers owns block pairs
// [w * nb / 16, (w + 1) * nb / 16) of every row; its row partials meet in shared memory.
template <int QT, int RG, typename XT, typename YT>
__global__ void __launch_bounds__(kGemvThreads, kGemvCtasPerSm) gemv_q_mma(GemvMmaArgs a) {
    constexpr bool kQ4 = QT == MGPU_Q4_0;
    constexpr int BB = QTraits<QT>::kBlockBytes;
    constexpr int TR = 16 * RG;  // rows per chunk
    extern __shared__ __align__(1024) uint8_t smem[];
    __shared__ __align__(8) uint64_t full_bar[kGemvMaxStages];
    __shared__ __align__(8) uint64_t empty_bar[kGemvMaxStages];

    const int tid = threadIdx.x;
    const int warp = tid >> 5, lane = tid & 31;
    const int nb = a.nb;
    const int G = gridDim.x;
    const int r0 = (int)((long long)a.N * blockIdx.x / G);
    const int r1 = (int)((long long)a.N * (blockIdx.x + 1) / G);
    const int nchunks = (r1 - r0 + TR - 1) / TR;

    if (tid == 0) {
        for (int s = 0; s < a.stages; ++s) {
            mbar_init(&full_bar[s], 1);
            mbar_init(&empty_bar[s], kMmaWarps);
        }
        fence_mbar_init();
        asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    }
    __syncthreads();

    if (warp == kMmaWarps) {
        // ---- producer warp: one bulk copy per row (into the padded pitch), 32 lanes issue ----
        int c = 0, s = 0;
        uint32_t ph = 0;
        for (; c < nchunks; ++c) {
            bool ok = true;
            if (lane == 0) ok = mbar_wait(&empty_bar[s], ph ^ 1u, a.status);
            ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
            if (!ok) break;
            const int row = r0 + c * TR;
            const int n = min(TR, r1 - row);
            if (lane == 0) mbar_arrive_expect_tx(&full_bar[s], (uint32_t)n * a.row_bytes);
            __syncwarp();
            uint8_t* dst = smem + (size_t)s * a.stage_stride;
            for (int i = lane; i < n; i += 32)
                bulk_g2s(dst + (size_t)i * a.pitch, a.W + (size_t)(row + i) * a.row_bytes, a.row_bytes, &full_bar[s]);
            if (++s == a.stages) {
                s = 0;
                ph ^= 1u;
            }
        }
        if (c < nchunks && lane == 0) {
            // Timed out: let the copies already issued land before the CTA exits.
            for (int k = max(0, c - a.stages); k < c; ++k)
                mbar_wait(&full_bar[k % a.stages], (uint32_t)(k / a.stages) & 1u, nullptr);
        }
        return;
    }

    // ---- consumers ----
    asm volatile("griddepcontrol.wait;" ::: "memory");
    const int K = nb * 32;
    uint8_t* xrec = smem + (size_t)a.stages * a.stage_stride;
    uint8_t* xaux = xrec + (size_t)nb * kXRecBytes;
    float* part = reinterpret_cast<float*>(xaux + (size_t)nb * kXAuxBytes);
    prepare_x_digits<XT, kQ4>(reinterpret_cast<const XT*>(a.x), K, xrec, xaux, tid, kConsumerThreads);
    named_barrier_sync(1, kConsumerThreads);

    const int g = lane >> 2, t = lane & 3;
    const int ppw = nb >> 4;  // block pairs per warp
    const int p_begin = warp * ppw;
    // lane constants: which B register carries the data, and the lane's block within a pair
    const uint32_t bsel_lo = (g < 4) ? 0xFFFFFFFFu : 0u;
    const int bhalf = t >> 1;
    const uint8_t* xb_lane = xrec + (g >> 2) * kXRecBytes + (g & 3) * 32 + 8 * t;
    const uint8_t* xa_lane = xaux + bhalf * kXAuxBytes + (t & 1) * 8;
    YT* __restrict__ y = reinterpret_cast<YT*>(a.y);

    int s = 0;
    uint32_t ph = 0;
    for (int c = 0; c < nchunks; ++c) {
        if (!mbar_wait(&full_bar[s], ph, a.status)) return;
        const uint8_t* st = smem + (size_t)s * a.stage_stride;
        float acc[RG][2];
#pragma unroll
        for (int r = 0; r < RG; ++r) acc[r][0] = acc[r][1] = 0.0f;
        // two block pairs per iteration (ppw is even: nb % 32 == 0), so that two independent
        // MMA chains are in flight per warp
#pragma unroll 1
        for (int pp = 0; pp < ppw; pp += 2) {
            uint32_t b0[2], b1[2], h0[2], h1[2];
            float xsl[2];
            float corr[2];
#pragma unroll
            for (int u = 0; u < 2; ++u) {
                const int pr = p_begin + pp + u;
                const uint2 bw = *reinterpret_cast<const uint2*>(xb_lane + (size_t)(2 * pr) * kXRecBytes);
                const uint2 ax = *reinterpret_cast<const uint2*>(xa_lane + (size_t)(2 * pr) * kXAuxBytes);
                xsl[u] = __uint_as_float(ax.x);
                corr[u] = __uint_as_float(ax.y);
                b0[u] = bw.x & bsel_lo;
                b1[u] = bw.x & ~bsel_lo;
                h0[u] = bw.y & bsel_lo;
                h1[u] = bw.y & ~bsel_lo;
            }
#pragma unroll
            for (int r = 0; r < RG; ++r) {
                const uint8_t* rg = st + (size_t)(r * 16 + g) * a.pitch;
                const uint8_t* rg8 = rg + (size_t)8 * a.pitch;
                int dl[2][4], dh[2][4];
                float dg[2], dg8[2];
#pragma unroll
                for (int u = 0; u < 2; ++u) {
                    const int pr = p_begin + pp + u;
                    uint32_t alo[4], ahi[4];
                    if constexpr (kQ4) {
                        // block 2pr at byte 36 pr (quants at +2: realign), block 2pr+1 at
                        // 36 pr + 18 (quants at +20: aligned)
                        const uint32_t* q0 = reinterpret_cast<const uint32_t*>(rg + 36 * pr + 4 * t);
                        const uint32_t* q8 = reinterpret_cast<const uint32_t*>(rg8 + 36 * pr + 4 * t);
                        const uint32_t u0 = prmt(q0[0], q0[1], 0x5432u), u1 = q0[5];
                        const uint32_t v0 = prmt(q8[0], q8[1], 0x5432u), v1 = q8[5];
                        alo[0] = u0 & 0x0F0F0F0Fu; ahi[0] = (u0 >> 4) & 0x0F0F0F0Fu;
                        alo[1] = v0 & 0x0F0F0F0Fu; ahi[1] = (v0 >> 4) & 0x0F0F0F0Fu;
                        alo[2] = u1 & 0x0F0F0F0Fu; ahi[2] = (u1 >> 4) & 0x0F0F0F0Fu;
                        alo[3] = v1 & 0x0F0F0F0Fu; ahi[3] = (v1 >> 4) & 0x0F0F0F0Fu;
                    } else {
                        // block 2pr at byte 68 pr (quants at +2 and +18: realign), block 2pr+1
                        // at 68 pr + 34 (quants at +36 and +52: aligned)
                        const uint32_t* q0 = reinterpret_cast<const uint32_t*>(rg + 68 * pr + 4 * t);
                        const uint32_t* q8 = reinterpret_cast<const uint32_t*>(rg8 + 68 * pr + 4 * t);
                        alo[0] = prmt(q0[0], q0[1], 0x5432u);
                        ahi[0] = prmt(q0[4], q0[5], 0x5432u);
                        alo[1] = prmt(q8[0], q8[1], 0x5432u);
                        ahi[1] = prmt(q8[4], q8[5], 0x5432u);
                        alo[2] = q0[9];
                        ahi[2] = q0[13];
                        alo[3] = q8[9];
                        ahi[3] = q8[13];
                    }
#pragma unroll
                    for (int i = 0; i < 4; ++i) dl[u][i] = dh[u][i] = 0;
                    mma_s8(dl[u], alo, b0[u], b1[u], kQ4);
                    mma_s8(dh[u], ahi, h0[u], h1[u], kQ4);
                    // this lane's block: 2pr + (t >> 1); its fp16 scale for rows g and g+8
                    const int boff = (2 * pr + bhalf) * BB;
                    dg[u] = __half2float(*reinterpret_cast<const __half*>(rg + boff)) * xsl[u];
                    dg8[u] = __half2float(*reinterpret_cast<const __half*>(rg8 + boff)) * xsl[u];
                }
#pragma unroll
                for (int u = 0; u < 2; ++u) {
                    const int vg = (dl[u][0] + dh[u][0]) + 256 * (dl[u][1] + dh[u][1]);
                    const int vg8 = (dl[u][2] + dh[u][2]) + 256 * (dl[u][3] + dh[u][3]);
                    acc[r][0] = fmaf(dg[u], (float)vg + corr[u], acc[r][0]);
                    acc[r][1] = fmaf(dg8[u], (float)vg8 + corr[u], acc[r][1]);
                }
            }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty_bar[s]);
        if (++s == a.stages) {
            s = 0;
            ph ^= 1u;
        }
        // sum the four lanes of a row, then the 8 warps through shared memory
        const int cf = c % a.chunks_per_flush;
#pragma unroll
        for (int r = 0; r < RG; ++r) {
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                float v = acc[r][h];
                v += __shfl_xor_sync(0xffffffffu, v, 1);
                v += __shfl_xor_sync(0xffffffffu, v, 2);
                if (t == 0) part[(cf * TR + r * 16 + g + 8 * h) * kMmaWarps + warp] = v;
            }
        }
        if (cf == a.chunks_per_flush - 1 || c == nchunks - 1) {
            named_barrier_sync(1, kConsumerThreads);
            const int row0 = r0 + (c - cf) * TR;
            const int nrows = min((cf + 1) * TR, r1 - row0);
            for (int r = tid; r < nrows; r += kConsumerThreads) {
                const float4* pv = reinterpret_cast<const float4*>(part + r * kMmaWarps);
                const float4 u = pv[0], w = pv[1];
                y[row0 + r] = from_f32<YT>(((u.x + u.y) + (u.z + u.w)) + ((w.x + w.y) + (w.z + w.w)));
            }
            named_barrier_sync(1, kConsumerThreads);
        }
    }
}

// Fallback for rows that are not 16-byte aligned or K outside [1024, 8192]: one warp per
// row, byte loads.
template <int QT, typename XT, typename YT>
__global__ void __launch_bounds__(256) gemv_q_generic(const uint8_t* __restrict__ W, const XT* __restrict__ x,
                                                      YT* __restrict__ y, int N, int nb, size_t row_bytes) {
    constexpr int BB = QTraits<QT>::kBlockBytes;
    const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    if (warp >= N) return;
    const uint8_t* row = W + (size_t)warp * row_bytes;
    float acc = 0.0f;
    for (int b = lane; b < nb; b += 32) {
        const uint8_t* p = row + (size_t)b * BB;
        const float d = __half2float(__ushort_as_half((unsigned short)(p[0] | (p[1] << 8))));
        float s = 0.0f;
        if constexpr (QT == MGPU_Q4_0) {
            for (int j = 0; j < 16; ++j) {
                const uint8_t q = p[2 + j];
                s = fmaf(to_f32<XT>(x[b * 32 + j]), (float)((int)(q & 0xF) - 8), s);
                s = fmaf(to_f32<XT>(x[b * 32 + j + 16]), (float)((int)(q >> 4) - 8), s);
            }
        } else {
            for (int j = 0; j < 32; ++j) s = fmaf(to_f32<XT>(x[b * 32 + j]), (float)(int8_t)p[2 + j], s);
        }
        acc = fmaf(d, s, acc);
    }
#pragma unroll
    for (int off = 16; off >= 1; off >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, off);
    if (lane == 0) y[warp] = from_f32<YT>(acc);
}

// ------------------------------------------------------------------ dense NK ---------
// Warp per ROWS rows; each lane streams 16-byte chunks along K.  K % (16 / sizeof(WT)) == 0
// and 16-byte aligned rows, otherwise scalar.
template <typename WT, typename XT, typename YT, int ROWS>
__global__ void __launch_bounds__(256) gemv_nk_dense(const WT* __restrict__ W, int64_t ldw,
                                                     const XT* __restrict__ x, YT* __restrict__ y, int N,
                                                     int K, int vec) {
    constexpr int EPV = 16 / sizeof(WT);  // elements per 16-byte vector
    const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    const int row0 = warp * ROWS;
    if (row0 >= N) return;
    float acc[ROWS];
#pragma unroll
    for (int r = 0; r < ROWS; ++r) acc[r] = 0.0f;
    if (vec) {
        const int nvec = K / EPV;
        for (int v = lane; v < nvec; v += 32) {
            float xv[EPV];
#pragma unroll
            for (int e = 0; e < EPV; ++e) xv[e] = to_f32<XT>(x[v * EPV + e]);
            uint4 wv[ROWS];
#pragma unroll
            for (int r = 0; r < ROWS; ++r)
                wv[r] = (row0 + r < N) ? __ldg(reinterpret_cast<const uint4*>(W + (size_t)(row0 + r) * ldw) + v)
                                       : make_uint4(0, 0, 0, 0);
#pragma unroll
            for (int r = 0; r < ROWS; ++r) {
                const WT* we = reinterpret_cast<const WT*>(&wv[r]);
#pragma unroll
                for (int e = 0; e < EPV; ++e) acc[r] = fmaf(xv[e], to_f32<WT>(we[e]), acc[r]);
            }
        }
    } else {
        for (int k = lane; k < K; k += 32) {
            const float xv = to_f32<XT>(x[k]);
#pragma unroll
            for (int r = 0; r < ROWS; ++r)
                if (row0 + r < N) acc[r] = fmaf(xv, to_f32<WT>(W[(size_t)(row0 + r) * ldw + k]), acc[r]);
        }
    }
#pragma unroll
    for (int r = 0; r < ROWS; ++r) {
#pragma unroll
        for (int off = 16; off >= 1; off >>= 1) acc[r] += __shfl_xor_sync(0xffffffffu, acc[r], off);
    }
    if (lane == 0) {
#pragma unroll
        for (int r = 0; r < ROWS; ++r)
            if (row0 + r < N) y[row0 + r] = from_f32<YT>(acc[r]);
    }
}

// ------------------------------------------------------------------ dense KN ---------
// CTA = 256 threads over a tile of 256 columns x kchunk rows of K; thread handles COLS
// consecutive columns of kchunk/8 rows.  Partials of split s go to partials[s][N]; the last
// CTA of a column tile (atomic ticket) sums splits 0..S-1 in order and resets the ticket.
// Launched with programmatic dependent launch: the weights are never written by the
// preceding kernel, so each thread issues its first rows' loads before griddepcontrol.wait;
// x, the partials and the tickets are touched only after it.
constexpr int kKnCols = 256;
template <typename WT, typename XT, typename YT, bool UNROLL>
__global__ void __launch_bounds__(256) gemv_kn_split(const WT* __restrict__ W, int64_t ldw,
                                                     const XT* __restrict__ x, YT* __restrict__ y, int N,
                                                     int K, int kchunk, float* __restrict__ partials,
                                                     unsigned int* __restrict__ counters) {
    constexpr int CPT = 8;  // columns per thread (contiguous)
    __shared__ float red[8][kKnCols];
    __shared__ unsigned int ticket;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int col_tile = blockIdx.x, split = blockIdx.y, splits = gridDim.y;
    const int n0 = col_tile * kKnCols + lane * CPT;
    const int k_begin = split * kchunk;
    const int k_end = min(K, k_begin + kchunk);
    float acc[CPT];
#pragma unroll
    for (int i = 0; i < CPT; ++i) acc[i] = 0.0f;
    const bool full_vec = (n0 + CPT <= N) && ((ldw * sizeof(WT)) % 16 == 0) &&
                          ((reinterpret_cast<uintptr_t>(W) & 15) == 0);
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    int k = k_begin + warp;
    bool waited = false;
    if (UNROLL && full_vec) {
        // four rows per step, all loads issued before any is used: four times the bytes in
        // flight per warp (measured faster for fp32 rows of N >= 4096, slower for N = 2048 and
        // for 16-bit rows; the launcher decides)
        constexpr int R = 4;
        constexpr int V = (int)(CPT * sizeof(WT) / 16);
        for (; k + 8 * (R - 1) < k_end; k += 8 * R) {
            WT wv[R][CPT];
            float xv[R];
#pragma unroll
            for (int r = 0; r < R; ++r) {
                const WT* wr = W + (size_t)(k + 8 * r) * ldw + n0;
#pragma unroll
                for (int v = 0; v < V; ++v)
                    reinterpret_cast<uint4*>(wv[r])[v] = __ldg(reinterpret_cast<const uint4*>(wr) + v);
            }
            if (!waited) {
                asm volatile("griddepcontrol.wait;" ::: "memory");
                waited = true;
            }
#pragma unroll
            for (int r = 0; r < R; ++r) xv[r] = to_f32<XT>(x[k + 8 * r]);
#pragma unroll
            for (int r = 0; r < R; ++r)
#pragma unroll
                for (int i = 0; i < CPT; ++i) acc[i] = fmaf(xv[r], to_f32<WT>(wv[r][i]), acc[i]);
        }
    }
    if (!waited) asm volatile("griddepcontrol.wait;" ::: "memory");
    for (; k < k_end; k += 8) {
        const float xv = to_f32<XT>(x[k]);
        const WT* wr = W + (size_t)k * ldw + n0;
        if (full_vec) {
            WT wv[CPT];
#pragma unroll
            for (int v = 0; v < (int)(CPT * sizeof(WT) / 16); ++v)
                reinterpret_cast<uint4*>(wv)[v] = __ldg(reinterpret_cast<const uint4*>(wr) + v);
#pragma unroll
            for (int i = 0; i < CPT; ++i) acc[i] = fmaf(xv, to_f32<WT>(wv[i]), acc[i]);
        } else {
#pragma unroll
            for (int i = 0; i < CPT; ++i)
                if (n0 + i < N) acc[i] = fmaf(xv, to_f32<WT>(wr[i]), acc[i]);
        }
    }
#pragma unroll
    for (int i = 0; i < CPT; ++i) red[warp][lane * CPT + i] = acc[i];
    __syncthreads();
    {
        const int n = col_tile * kKnCols + tid;
        float s = 0.0f;
#pragma unroll
        for (int w = 0; w < 8; ++w) s += red[w][tid];
        if (n < N) partials[(size_t)split * N + n] = s;
    }
    __threadfence();
    __syncthreads();
    if (tid == 0) ticket = atomicAdd(&counters[col_tile], 1u);
    __syncthreads();
    if (ticket != (unsigned)(splits - 1)) return;
    __threadfence();
    const int n = col_tile * kKnCols + tid;
    if (n < N) {
        float s = 0.0f;
        for (int sp = 0; sp < splits; ++sp) s += __ldcg(partials + (size_t)sp * N + n);
        y[n] = from_f32<YT>(s);
    }
    if (tid == 0) counters[col_tile] = 0u;
}

// ------------------------------------------------------------------ dispatch helpers --
template <template <typename, typename> class F, typename... Args>
cudaError_t dispatch_xy(int xtype, int ytype, Args&&... args) {
#define MGPU_Y(XT)                                                                          \
    switch (ytype) {                                                                        \
        case MGPU_F32: return F<XT, float>::run(args...);                                  \
        case MGPU_F16: return F<XT, __half>::run(args...);                                 \
        case MGPU_BF16: return F<XT, __nv_bfloat16>::run(args...);                         \
        default: return cudaErrorInvalidValue;                                             \
    }
    switch (xtype) {
        case MGPU_F32: MGPU_Y(float)
        case MGPU_F16: MGPU_Y(__half)
        case MGPU_BF16: MGPU_Y(__nv_bfloat16)
        default: return cudaErrorInvalidValue;
    }
#undef MGPU_Y
}

template <int QT>
struct GemvQLaunch {
    template <typename XT, typename YT>
    struct F {
        static cudaError_t run(const mgpu_k::LaunchCtx& c, const uint8_t* W, const void* x, void* y, int N,
                               int K, const GemvNorm* norm) {
            constexpr int BB = QTraits<QT>::kBlockBytes;
            const int nb = K / 32;
            const size_t row_bytes = (size_t)nb * BB;
            const bool fast = (nb % 32 == 0) && nb <= 256 && (row_bytes % 16 == 0) &&
                              ((reinterpret_cast<uintptr_t>(W) & 15) == 0) &&
                              ((reinterpret_cast<uintptr_t>(x) & 15) == 0);
            // the RMSNorm prologue is in the streaming dp4a kernel only
            if (norm && !(fast && (kStreamThreads % nb) == 0)) return cudaErrorNotSupported;
            if (!fast) {
                const int blocks = (N * 32 + 255) / 256;
                gemv_q_generic<QT, XT, YT><<<blocks, 256, 0, c.stream>>>(W, (const XT*)x, (YT*)y, N, nb, row_bytes);
                return cudaGetLastError();
            }
            // The dp4a kernel gives each thread one block column of a row slot, so it needs
            // nb to divide its 512 consumer threads (K = 1024, 2048, 4096, 8192 with nb <= 256).
            // Other K go to the MMA kernel when it can stage them.  (Timed inside a chain of
            // dependent GEMVs of different shapes, the dp4a kernel is the faster of the two on
            // every Phi-1.5 shape, so it takes all K it supports.)
            const bool dp4a_ok = (kStreamThreads % nb) == 0;
            if (!dp4a_ok) {
                const cudaError_t e = run_mma(c, W, x, y, N, K, true);
                if (e != cudaErrorNotSupported) return e;
            }
            if (!dp4a_ok) {
                const int blocks = (N * 32 + 255) / 256;
                gemv_q_generic<QT, XT, YT><<<blocks, 256, 0, c.stream>>>(W, (const XT*)x, (YT*)y, N, nb, row_bytes);
                return cudaGetLastError();
            }
            const int RP = kStreamThreads / nb;
            // Layer-sized GEMVs take one CTA per SM: a launch then leaves room on every SM for
            // one CTA of the next GEMV in the stream, which under programmatic dependent launch
            // becomes resident early and streams its weights while this one finishes.  Large
            // ones (more than kBigRows rows per SM, e.g. the lm_head) take two per SM: twice the
            // warps and bytes in flight matter more there than the overlap.
            constexpr int kBigRows = 64;
            const int per_sm = N > c.sm_count * kBigRows ? kGemvCtasPerSm : 1;
            const int G = max(1, min(c.sm_count * per_sm, (N + RP - 1) / RP));
            const int rows_per_cta = (N + G - 1) / G;
            // Rows per thread (4, 2, 1) and ring depth (2..8 stages).  Four rows per thread
            // (a 36 KB chunk of Q4_0 K = 2048 rows) whenever two stages of them fit: a decode
            // chain then launches one function for every shape, and a dependent launch of a
            // different function was measured to cost ~1.4 us more than one of the same
            // function (a 97-GEMV Phi-1.5 step mixing two row counts took 455.8 us, one row
            // count for all 385.8 us).  The ring then holds all of a layer-sized GEMV's rows, so
            // its weights stream in before griddepcontrol.wait returns.  Otherwise: a ring that
            // holds all of the CTA's rows with the widest chunk that computes at most 25 %
            // padding rows; then, for GEMVs too large to prefetch whole, a 4-stage ring of the
            // widest chunk that fits.  Row partials of up to kPartFloats are buffered between
            // flushes.
            constexpr int kPartFloats = 4096;
            constexpr int kMaxRpt = 4;
            const int wpr = nb / 32;
            const size_t x_bytes = (size_t)kXPlanes * (K / 4) * 4 + (size_t)nb * 4;
            auto stride = [&](int r) { return ((size_t)RP * r * row_bytes + 1023) / 1024 * 1024; };
            auto chunks_of = [&](int r) { return (rows_per_cta + RP * r - 1) / (RP * r); };
            auto part_floats = [&](int r) {
                const int cpf = max(1, min(chunks_of(r), kPartFloats / (RP * r * wpr)));
                return (size_t)max(cpf * RP * r * wpr, kStreamThreads / 32);  // (also the RMSNorm scratch)
            };
            auto depth = [&](int r, int cap) {
                const size_t fixed = x_bytes + 4 * part_floats(r);
                if (fixed + 2 * stride(r) > kGemvSmemBudget) return 0;
                return max(2, min(cap, min(chunks_of(r), (int)((kGemvSmemBudget - fixed) / stride(r)))));
            };
            int rpt = 0, stages = 0;
            if (const int d = depth(kMaxRpt, kGemvMaxStages)) {
                rpt = kMaxRpt;
                stages = d;
            }
            for (int r = kMaxRpt; r >= 1 && !rpt; r >>= 1) {
                const int d = depth(r, kGemvMaxStages);
                const int waste = chunks_of(r) * RP * r - rows_per_cta;
                if (d && d >= chunks_of(r) && 4 * waste <= rows_per_cta) {
                    rpt = r;
                    stages = d;
                }
            }
            for (int r = kMaxRpt; r >= 1 && !rpt; r >>= 1) {
                // a 4-stage ring, or at least 64 KB in flight per CTA (two CTAs per SM keep twice
                // that, well above what the HBM latency needs): Q8_0 rows then take two rows per
                // thread in 35 KB chunks rather than one (the row reduction per block halves;
                // the Q8_0 lm_head measured 22.7 us with one row per thread)
                const int d = depth(r, 4);
                if (d >= min(4, chunks_of(r)) || (d >= 2 && (size_t)d * stride(r) >= 64 * 1024)) {
                    rpt = r;
                    stages = d;
                }
            }
            for (int r = kMaxRpt; r >= 1 && !rpt; r >>= 1) {
                const int d = depth(r, 4);
                if (d) {
                    rpt = r;
                    stages = d;
                }
            }
            if (!rpt) {
                rpt = 1;
                stages = 2;
            }
            GemvQArgs a;
            a.W = W;
            a.x = x;
            a.y = y;
            a.N = N;
            a.nb = nb;
            a.row_bytes = (uint32_t)row_bytes;
            a.stage_stride = (uint32_t)stride(rpt);
            a.stages = stages;
            a.chunks_per_flush = max(1, min(chunks_of(rpt), kPartFloats / (RP * rpt * wpr)));
            a.status = c.status;
            a.gamma = norm ? norm->gamma : nullptr;
            a.gtype = norm ? norm->gtype : 0;
            a.eps = norm ? norm->eps : 0.0f;
            const size_t smem = (size_t)a.stages * a.stage_stride + x_bytes + 4 * part_floats(rpt);
            switch (rpt) {
                case 4: return launch<4, XT, YT>(c, a, G, smem);
                case 2: return launch<2, XT, YT>(c, a, G, smem);
                default: return launch<1, XT, YT>(c, a, G, smem);
            }
        }
        // Integer tensor-core path (gemv_q_mma).  Returns cudaErrorNotSupported, launching
        // nothing, when a 16-row chunk with its padded pitch does not fit the shared-memory
        // budget (Q8_0 rows of K = 8192) or, unless `any_shape`, when the shape is not one it
        // is the faster kernel for; the caller then takes the dp4a kernel.
        static cudaError_t run_mma(const mgpu_k::LaunchCtx& c, const uint8_t* W, const void* x, void* y, int N,
                                   int K, bool any_shape) {
            constexpr int BB = QTraits<QT>::kBlockBytes;
            const int nb = K / 32;
            const size_t row_bytes = (size_t)nb * BB;
            const size_t pitch = row_bytes + 16;
            constexpr int kBigRows = 64;
            const int per_sm = N > c.sm_count * kBigRows ? kGemvCtasPerSm : 1;
            const int G = max(1, min(c.sm_count * per_sm, (N + 15) / 16));
            const int rows_per_cta = (N + G - 1) / G;
            constexpr int kPartFloats = 4096;
            const size_t x_bytes = (size_t)nb * (kXRecBytes + kXAuxBytes);
            auto stride = [&](int rg) { return ((size_t)16 * rg * pitch + 1023) / 1024 * 1024; };
            auto chunks_of = [&](int rg) { return (rows_per_cta + 16 * rg - 1) / (16 * rg); };
            auto part_floats = [&](int rg) {
                const int cpf = max(1, min(chunks_of(rg), kPartFloats / (16 * rg * kMmaWarps)));
                return (size_t)cpf * 16 * rg * kMmaWarps;
            };
            // ring depth for chunks of rg row groups, at most `cap`; a CTA whose rows form one
            // chunk may use a single stage
            auto depth = [&](int rg, int cap) {
                const size_t fixed = x_bytes + 4 * part_floats(rg);
                const int dmin = chunks_of(rg) == 1 ? 1 : 2;
                if (fixed + dmin * stride(rg) > kGemvMmaSmemBudget) return 0;
                return max(dmin, min(cap, min(chunks_of(rg), (int)((kGemvMmaSmemBudget - fixed) / stride(rg)))));
            };
            // Same policy as the dp4a kernel: prefetch the CTA's whole share when a ring can
            // hold it (widest chunk with at most 25 % padding rows), else stream through a
            // 4-stage ring of the widest chunk that fits.
            int rg = 0, stages = 0;
            for (int r = 4; r >= 1 && !rg; r >>= 1) {
                const int d = depth(r, kGemvMaxStages);
                const int waste = chunks_of(r) * 16 * r - rows_per_cta;
                if (d && d >= chunks_of(r) && 4 * waste <= max(rows_per_cta, 16)) {
                    rg = r;
                    stages = d;
                }
            }
            for (int r = 4; r >= 1 && !rg; r >>= 1) {
                const int d = depth(r, 4);
                if (d >= min(4, chunks_of(r))) {
                    rg = r;
                    stages = d;
                }
            }
            for (int r = 4; r >= 1 && !rg; r >>= 1) {
                const int d = depth(r, 4);
                if (d) {
                    rg = r;
                    stages = d;
                }
            }
            if (!rg) return cudaErrorNotSupported;
            const bool prefetched = stages >= chunks_of(rg);
            if (!any_shape && !(prefetched && rows_per_cta >= 24)) return cudaErrorNotSupported;
            GemvMmaArgs a;
            a.W = W;
            a.x = x;
            a.y = y;
            a.N = N;
            a.nb = nb;
            a.row_bytes = (uint32_t)row_bytes;
            a.pitch = (uint32_t)pitch;
            a.stage_stride = (uint32_t)stride(rg);
            a.stages = stages;
            a.chunks_per_flush = (int)(part_floats(rg) / ((size_t)16 * rg * kMmaWarps));
            a.status = c.status;
            const size_t smem = (size_t)stages * a.stage_stride + x_bytes + 4 * part_floats(rg);
            switch (rg) {
                case 4: return launch_mma<4>(c, a, G, smem);
                case 2: return launch_mma<2>(c, a, G, smem);
                default: return launch_mma<1>(c, a, G, smem);
            }
        }
        template <int RG>
        static cudaError_t launch_mma(const mgpu_k::LaunchCtx& c, const GemvMmaArgs& a, int G, size_t smem) {
            auto kern = gemv_q_mma<QT, RG, XT, YT>;
            static thread_local uint64_t configured = 0;  // one bit per device ordinal
            int ordinal = 0;
            cudaGetDevice(&ordinal);
            if (!(configured & (1ull << (ordinal & 63)))) {
                cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                     (int)kGemvMmaSmemBudget);
                if (e != cudaSuccess) return e;
                e = cudaFuncSetAttribute(kern, cudaFuncAttributePreferredSharedMemoryCarveout,
                                         (int)cudaSharedmemCarveoutMaxShared);
                if (e != cudaSuccess) return e;
                configured |= 1ull << (ordinal & 63);
            }
            cudaLaunchConfig_t cfg = {};
            cfg.gridDim = dim3(G);
            cfg.blockDim = dim3(kGemvThreads);
            cfg.dynamicSmemBytes = smem;
            cfg.stream = c.stream;
            cudaLaunchAttribute attr[1];
            attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
            attr[0].val.programmaticStreamSerializationAllowed = 1;
            cfg.attrs = attr;
            cfg.numAttrs = 1;
            return cudaLaunchKernelEx(&cfg, kern, a);
        }
        template <int RPT, typename XT2, typename YT2>
        static cudaError_t launch(const mgpu_k::LaunchCtx& c, const GemvQArgs& a, int G, size_t smem) {
            auto kern = gemv_q_stream<QT, RPT, XT2, YT2>;
            // Every instantiation asks for the largest shared-memory carve-out, so that
            // back-to-back GEMVs of different shapes never force an L1 / shared-memory
            // reconfiguration between them (which would also stop their CTAs from
            // overlapping under programmatic dependent launch).
            static thread_local uint64_t configured = 0;  // one bit per device ordinal
            int ordinal = 0;
            cudaGetDevice(&ordinal);
            if (!(configured & (1ull << (ordinal & 63)))) {
                cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                     (int)kGemvSmemBudget);
                if (e != cudaSuccess) return e;
                e = cudaFuncSetAttribute(kern, cudaFuncAttributePreferredSharedMemoryCarveout,
                                         (int)cudaSharedmemCarveoutMaxShared);
                if (e != cudaSuccess) return e;
                configured |= 1ull << (ordinal & 63);
            }
            cudaLaunchConfig_t cfg = {};
            cfg.gridDim = dim3(G);
            cfg.blockDim = dim3(kStreamBlock);
            cfg.dynamicSmemBytes = smem;
            cfg.stream = c.stream;
            cudaLaunchAttribute attr[1];
            attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
            attr[0].val.programmaticStreamSerializationAllowed = 1;
            cfg.attrs = attr;
            cfg.numAttrs = 1;
            return cudaLaunchKernelEx(&cfg, kern, a);
        }
    };
};

template <typename WT>
struct GemvNkLaunch {
    template <typename XT, typename YT>
    struct F {
        static cudaError_t run(const mgpu_k::LaunchCtx& c, const void* W, int64_t ldw, const void* x, void* y,
                               int N, int K) {
            constexpr int ROWS = 4;
            constexpr int EPV = 16 / sizeof(WT);
            const int vec = (K % EPV == 0) && ((ldw * (int64_t)sizeof(WT)) % 16 == 0) &&
                            ((reinterpret_cast<uintptr_t>(W) & 15) == 0);
            const int warps = (N + ROWS - 1) / ROWS;
            const int blocks = (warps * 32 + 255) / 256;
            gemv_nk_dense<WT, XT, YT, ROWS><<<blocks, 256, 0, c.stream>>>((const WT*)W, ldw, (const XT*)x,
                                                                         (YT*)y, N, K, vec);
            return cudaGetLastError();
        }
    };
};

// gemv_kn_split with programmatic dependent launch (the kernel orders its reads of x and its
// scratch writes after griddepcontrol.wait).
template <typename WT, typename XT, typename YT>
cudaError_t launch_kn(cudaStream_t stream, dim3 grid, const WT* W, int64_t ldw, const XT* x, YT* y, int N, int K,
                      int kchunk, float* partials, unsigned int* counters) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = dim3(256);
    cfg.dynamicSmemBytes = 0;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    if (sizeof(WT) == 4 && N >= 4096)
        return cudaLaunchKernelEx(&cfg, gemv_kn_split<WT, XT, YT, true>, W, ldw, x, y, N, K, kchunk, partials,
                                  counters);
    return cudaLaunchKernelEx(&cfg, gemv_kn_split<WT, XT, YT, false>, W, ldw, x, y, N, K, kchunk, partials,
                              counters);
}

template <typename WT>
struct GemvKnLaunch {
    template <typename XT, typename YT>
    struct F {
        static cudaError_t run(const mgpu_k::LaunchCtx& c, const void* W, int64_t ldw, const void* x, void* y,
                               int N, int K, float* partials, unsigned int* counters) {
            int splits = 1;
            mgpu_k::gemv_kn_scratch_bytes(N, K, c.sm_count, &splits);
            const int kchunk = (K + splits - 1) / splits;
            dim3 grid((N + kKnCols - 1) / kKnCols, splits);
            return launch_kn<WT, XT, YT>(c.stream, grid, (const WT*)W, ldw, (const XT*)x, (YT*)y, N, K, kchunk,
                                         partials, counters);
        }
    };
};

// Fixed scratch of gemv_kn_noalloc: split-K tickets (kNoAllocTickets x u32) followed by the
// fp32 partials (kNoAllocPartials floats).  One copy per GPU that loads this library, kept
// until the process exits; every call shares it.
constexpr int kNoAllocTickets = 4096;            // column tiles of 256 -> N <= 1,048,576
constexpr size_t kNoAllocPartials = 256 * 1024;  // splits * N <= 262,144 (1 MiB)
constexpr size_t kNoAllocBytes = kNoAllocTickets * sizeof(unsigned int) + kNoAllocPartials * sizeof(float);
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocBytes];

}  // namespace

namespace mgpu_k {

cudaError_t gemv_q(const LaunchCtx& c, int qtype, const uint8_t* W, int xtype, const void* x, int ytype,
                   void* y, int N, int K) {
    if (N <= 0) return cudaSuccess;
    const GemvNorm* none = nullptr;
    if (qtype == MGPU_Q4_0)
        return dispatch_xy<GemvQLaunch<MGPU_Q4_0>::F>(xtype, ytype, c, W, x, y, N, K, none);
    if (qtype == MGPU_Q8_0)
        return dispatch_xy<GemvQLaunch<MGPU_Q8_0>::F>(xtype, ytype, c, W, x, y, N, K, none);
    return cudaErrorInvalidValue;
}

cudaError_t gemv_q_norm(const LaunchCtx& c, int qtype, const uint8_t* W, int xtype, const void* x, int gtype,
                        const void* gamma, float eps, int ytype, void* y, int N, int K) {
    if (N <= 0) return cudaSuccess;
    GemvNorm nrm{gamma, gtype, eps};
    const GemvNorm* p = &nrm;
    if (qtype == MGPU_Q4_0)
        return dispatch_xy<GemvQLaunch<MGPU_Q4_0>::F>(xtype, ytype, c, W, x, y, N, K, p);
    if (qtype == MGPU_Q8_0)
        return dispatch_xy<GemvQLaunch<MGPU_Q8_0>::F>(xtype, ytype, c, W, x, y, N, K, p);
    return cudaErrorInvalidValue;
}

cudaError_t gemv_nk(const LaunchCtx& c, int wtype, const void* W, int64_t ldw, int xtype, const void* x,
                    int ytype, void* y, int N, int K) {
    if (N <= 0) return cudaSuccess;
    switch (wtype) {
        case MGPU_F32: return dispatch_xy<GemvNkLaunch<float>::F>(xtype, ytype, c, W, ldw, x, y, N, K);
        case MGPU_F16: return dispatch_xy<GemvNkLaunch<__half>::F>(xtype, ytype, c, W, ldw, x, y, N, K);
        case MGPU_BF16: return dispatch_xy<GemvNkLaunch<__nv_bfloat16>::F>(xtype, ytype, c, W, ldw, x, y, N, K);
        default: return cudaErrorInvalidValue;
    }
}

size_t gemv_kn_noalloc_max_n() { return kNoAllocPartials; }

cudaError_t gemv_kn_noalloc(const LaunchCtx& c, int wtype, const void* W, int64_t ldw, int xtype, const void* x,
                            int ytype, void* y, int N, int K) {
    if (N <= 0 || (size_t)N > kNoAllocPartials || (N + kKnCols - 1) / kKnCols > kNoAllocTickets)
        return cudaErrorInvalidValue;
    // The array's device address, looked up once per device with that device current.  The
    // lookup also clears the tickets once (stream-ordered before this call's kernel); after
    // that every call leaves them zero, because the last CTA of each column tile resets its
    // ticket before it exits.  The cache would hold a stale address after cudaDeviceReset,
    // which unloads this library's device code: do not call this entry point after one.
    static void* addr[64] = {};
    static std::mutex mu;
    int ordinal = 0;
    cudaError_t e = cudaGetDevice(&ordinal);
    if (e != cudaSuccess) return e;
    if (ordinal < 0 || ordinal >= 64) return cudaErrorInvalidDevice;
    void* base = nullptr;
    {
        std::lock_guard<std::mutex> lock(mu);
        if (!addr[ordinal]) {
            void* a = nullptr;
            e = cudaGetSymbolAddress(&a, g_noalloc_scratch);
            if (e != cudaSuccess) return e;
            e = cudaMemsetAsync(a, 0, kNoAllocTickets * sizeof(unsigned int), c.stream);
            if (e != cudaSuccess) return e;
            addr[ordinal] = a;
        }
        base = addr[ordinal];
    }
    unsigned int* tickets = reinterpret_cast<unsigned int*>(base);
    float* partials = reinterpret_cast<float*>(reinterpret_cast<unsigned char*>(base) +
                                               kNoAllocTickets * sizeof(unsigned int));
    int splits = 1;
    gemv_kn_scratch_bytes(N, K, c.sm_count, &splits);
    splits = max(1, min(splits, (int)(kNoAllocPartials / (size_t)N)));
    const int col_tiles = (N + kKnCols - 1) / kKnCols;
    const int kchunk = (K + splits - 1) / splits;
    dim3 grid(col_tiles, splits);
#define MGPU_NA_LAUNCH(WT, XT, YT) \
    if (sizeof(WT) == 4 && N >= 4096)                                                                            \
        gemv_kn_split<WT, XT, YT, true><<<grid, 256, 0, c.stream>>>((const WT*)W, ldw, (const XT*)x, (YT*)y, N, K,     \
                                                                    kchunk, partials, tickets);                       \
    else                                                                                                            \
        gemv_kn_split<WT, XT, YT, false><<<grid, 256, 0, c.stream>>>((const WT*)W, ldw, (const XT*)x, (YT*)y, N, K,    \
                                                                     kchunk, partials, tickets)
#define MGPU_NA_Y(WT, XT)                                                 \
    switch (ytype) {                                                      \
        case MGPU_F32: MGPU_NA_LAUNCH(WT, XT, float); break;              \
        case MGPU_F16: MGPU_NA_LAUNCH(WT, XT, __half); break;             \
        case MGPU_BF16: MGPU_NA_LAUNCH(WT, XT, __nv_bfloat16); break;     \
        default: return cudaErrorInvalidValue;                            \
    }
#define MGPU_NA_X(WT)                                    \
    switch (xtype) {                                     \
        case MGPU_F32: MGPU_NA_Y(WT, float) break;       \
        case MGPU_F16: MGPU_NA_Y(WT, __half) break;      \
        case MGPU_BF16: MGPU_NA_Y(WT, __nv_bfloat16) break; \
        default: return cudaErrorInvalidValue;           \
    }
    switch (wtype) {
        case MGPU_F32: MGPU_NA_X(float) break;
        case MGPU_F16: MGPU_NA_X(__half) break;
        case MGPU_BF16: MGPU_NA_X(__nv_bfloat16) break;
        default: return cudaErrorInvalidValue;
    }
#undef MGPU_NA_X
#undef MGPU_NA_Y
#undef MGPU_NA_LAUNCH
    return cudaGetLastError();
}

size_t gemv_kn_scratch_bytes(int N, int K, int sm_count, int* splits_out) {
    // One wave: at most 4 CTAs per SM (the number resident at once), each with at least 64 rows
    // of K.  (Rounding the split count up instead left a second wave of a few CTAs: with
    // N = 8192, 608 CTAs for 592 slots.)
    const int col_tiles = (N + kKnCols - 1) / kKnCols;
    int splits = (4 * sm_count) / col_tiles;
    splits = max(1, min(splits, (K + 63) / 64));
    if (splits_out) *splits_out = splits;
    return (size_t)col_tiles * sizeof(unsigned int) + (size_t)splits * N * sizeof(float) + 256;
}

cudaError_t gemv_kn(const LaunchCtx& c, int wtype, const void* W, int64_t ldw, int xtype, const void* x,
                    int ytype, void* y, int N, int K, float* partials, unsigned int* counters) {
    if (N <= 0) return cudaSuccess;
    switch (wtype) {
        case MGPU_F32:
            return dispatch_xy<GemvKnLaunch<float>::F>(xtype, ytype, c, W, ldw, x, y, N, K, partials, counters);
        case MGPU_F16:
            return dispatch_xy<GemvKnLaunch<__half>::F>(xtype, ytype, c, W, ldw, x, y, N, K, partials, counters);
        case MGPU_BF16:
            return dispatch_xy<GemvKnLaunch<__nv_bfloat16>::F>(xtype, ytype, c, W, ldw, x, y, N, K, partials,
                                                              counters);
        default: return cudaErrorInvalidValue;
    }
}

}  // namespace mgpu_k
