// chain.cu - the GEMVs of a decode step in one persistent launch (sm_100a).
//
// moondream2_forward runs a decode token as a chain of dependent dispatch_gemv calls, each
// waiting for the previous one (src/models/moondream2.cpp:357-542: q/k/v, o, gate/up, down
// per layer, then the lm_head).  One launch per GEMV pays, at every link, the grid's drain
// and launch, the weights' first bytes arriving from HBM and the activation vector's trip
// through L2 — a few microseconds against 0.4-1.5 us of HBM time for a Phi-1.5 layer GEMV.
// gemv_chain_kernel runs a whole chain of Q4_0 / Q8_0 GEMVs in one cooperative launch, one
// CTA per SM:
//   - a producer thread streams the CTA's rows of every GEMV, one GEMV after the other, into
//     a shared-memory ring with cp.async.bulk (the 1-D TMA).  Weights never depend on the
//     chain's data, so the stream does not stop at the links: while the consumers wait for a
//     GEMV's input vector, the ring fills with that GEMV's rows;
//   - sixteen consumer warps decode with the exact integer dp4a inner products of qdot.cuh
//     (each thread one 32-element block column of the rows, activations in 16-bit fixed point);
//   - a GEMV whose input is the output of an earlier GEMV of the chain reads it straight from
//     that GEMV's y.  Every GEMV that a later one reads has a 64-bit counter of its own,
//     monotonic over all launches of the chain (never reset): a CTA that has stored its rows
//     of the GEMV meets its consumers at a barrier, and one thread adds 1 to the counter with a
//     release reduction.  Before a dependent GEMV one thread of each CTA polls that single
//     counter with acquire loads until all G CTAs of this launch have added to it, and a
//     barrier then lets the CTA's consumers read the vector: one poller per CTA, one line per
//     GEMV, and one round trip to L2 for the data once the count is seen.  (Per-thread polls of
//     the flags of each element's writer CTAs, tried first, cost several dependent round trips
//     per thread before the data load.)
// Launches of one chain must not overlap (the counters and the launch counter are the chain's
// own), and all its CTAs must be resident together: the launch is cooperative.
#include <cuda_runtime.h>

#include "common.cuh"
#include "kernels.h"
#include "qdot.cuh"

using namespace mgpu_dev;

namespace {

constexpr int kChainNC = 512;         // consumer threads per CTA: 16 warps
constexpr int kChainMaxSlots = 12;
constexpr int kChainMaxStages = 192;  // the stage table is copied to shared memory
constexpr int kChainF = 4;            // chunks whose rows are reduced together
constexpr int kChainMaxK = 8192;
constexpr size_t kChainPlaneBytes = (size_t)kXPlanes * (kChainMaxK / 4) * 4 + (size_t)(kChainMaxK / 32) * 4;
constexpr size_t kChainPartBytes = (size_t)2 * 128 * 4;  // 2 buffers of F * RPT * NC / 32 <= 128 floats
constexpr int kFlagStride = 8;  // u64 words between two stages' counters (64 bytes)

// A chunk is RPT rows per consumer thread: NC * RPT blocks, whatever K is (Q4_0 18432 bytes,
// Q8_0 17408).  Thread t decodes the block at byte t * BB of the chunk (+ i * NC * BB for its
// i-th row): row slot t / nb, block column t % nb.
template <int QT, int NC>
struct ChainGeom {
    static_assert(NC == 512, "the row reduction is written for 16 consumer warps");
    static constexpr int RPT = QT == MGPU_Q4_0 ? 2 : 1;
    static constexpr uint32_t kChunk = (uint32_t)NC * RPT * QTraits<QT>::kBlockBytes;
};

struct ChainArgs {
    const mgpu_k::ChainStage* stages;
    int n_stages;
    int slots;                    // ring depth
    unsigned int* sync;           // [0..1] launch counter (u64), [2] finish ticket, [3] poison
    unsigned long long* flags;    // per stage (stride kFlagStride): CTAs that finished it, over all launches
    unsigned long long* times;    // null, or [n_stages] stage end (ns, max over CTAs) + start (min)
    int* status;
};

__device__ __forceinline__ bool poisoned(const unsigned int* sync) {
    return *reinterpret_cast<const volatile unsigned int*>(sync + 3) != 0u;
}

// Mark the launch failed: the device status for the host, the chain's poison word for the
// other CTAs (their waits give up) and for later launches (which then refuse to run), and this
// CTA's abort flag.
__device__ __forceinline__ void chain_fail(const ChainArgs& a, volatile int* s_abort) {
    *s_abort = 1;
    atomicExch(a.status, (int)MGPU_ERR_DEVICE_TIMEOUT);
    atomicExch(a.sync + 3, 1u);
}

// mbarrier wait bounded by the deadline; gives up early when the CTA aborts.
__device__ __forceinline__ bool chain_mbar_wait(uint64_t* bar, uint32_t parity, const ChainArgs& a,
                                                volatile int* s_abort) {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = globaltimer();
    while (true) {
        if (mbar_try_wait(bar, parity)) return true;
        if (*s_abort) return false;
        if (globaltimer() - t0 > kWaitLimitNs) {
            chain_fail(a, s_abort);
            return false;
        }
    }
}

// Named barrier 1 over the consumers with an OR of `flag`: every consumer thread passes the
// same sequence of these barriers, and one that gives up arrives with flag = true, so all of
// them learn it at the same barrier and leave together.
template <int NC>
__device__ __forceinline__ bool barrier_or(bool flag) {
    uint32_t r;
    asm volatile(
        "{\n .reg .pred p, q;\n"
        " setp.ne.u32 p, %1, 0;\n"
        " bar.red.or.pred q, 1, %2, p;\n"
        " selp.u32 %0, 1, 0, q;\n}\n"
        : "=r"(r)
        : "r"(flag ? 1u : 0u), "r"(NC)
        : "memory");
    return r != 0;
}

__device__ __forceinline__ unsigned long long ld_acquire_u64(const unsigned long long* p) {
    unsigned long long v;
    asm volatile("ld.acquire.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ void red_release_add_u64(unsigned long long* p, unsigned long long v) {
    asm volatile("red.release.gpu.global.add.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}

// Wait until stage dep's counter reaches `target` (every CTA of this launch has stored its rows
// of it), polling with acquire loads; false when it gave up.  One thread per CTA calls this.
__device__ __forceinline__ bool wait_stage(const ChainArgs& a, int dep, unsigned long long target,
                                           volatile int* s_abort) {
    const unsigned long long* f = a.flags + (size_t)dep * kFlagStride;
    if (ld_acquire_u64(f) >= target) return true;
    const uint64_t t0 = globaltimer();
    uint32_t spins = 0;
    while (ld_acquire_u64(f) < target) {
        if ((++spins & 15u) == 0u) {
            if (*s_abort || poisoned(a.sync)) {
                *s_abort = 1;
                return false;
            }
            if (globaltimer() - t0 > kWaitLimitNs) {
                chain_fail(a, s_abort);
                return false;
            }
        }
    }
    return true;
}

// Word w (elements 4w .. 4w+3) of a stage's input as four floats, read at L2 (another CTA may
// have just written it; L1 could hold an older copy).
__device__ __forceinline__ float4 load_x_word(const void* x, int xtype, int w) {
    if (xtype == MGPU_F32) return __ldcg(reinterpret_cast<const float4*>(x) + w);
    const uint2 u = __ldcg(reinterpret_cast<const uint2*>(x) + w);
    float4 f;
    if (xtype == MGPU_BF16) {
        f.x = __uint_as_float(u.x << 16);
        f.y = __uint_as_float(u.x & 0xFFFF0000u);
        f.z = __uint_as_float(u.y << 16);
        f.w = __uint_as_float(u.y & 0xFFFF0000u);
    } else {
        const float2 lo = __half22float2(*reinterpret_cast<const __half2*>(&u.x));
        const float2 hi = __half22float2(*reinterpret_cast<const __half2*>(&u.y));
        f.x = lo.x; f.y = lo.y; f.z = hi.x; f.w = hi.y;
    }
    return f;
}

// The stage's input vector into fixed point (qdot.cuh's layout) in shared memory: every thread
// issues all its loads (at L2), then converts.  The caller has waited for the stage that wrote it.
template <int NC, int ITERS>
__device__ __forceinline__ void prepare_x_chain(const mgpu_k::ChainStage& st, uint32_t* planes, float* bscale,
                                                int tid) {
    const int words = st.K / 4;
    float4 v4[ITERS];
#pragma unroll
    for (int it = 0; it < ITERS; ++it) {
        const int w = it * NC + tid;
        if (w < words) v4[it] = load_x_word(st.x, st.xtype, w);
    }
    // every lane converts (the block exponent is agreed with shuffles over 8 lanes)
#pragma unroll
    for (int it = 0; it < ITERS; ++it) {
        const int w = it * NC + tid;
        if (w < words) {
            const float v[4] = {v4[it].x, v4[it].y, v4[it].z, v4[it].w};
            convert_x_word(v, w, words, planes, bscale, (tid & 7) == 0);
        }
    }
}

// y[row] in the stage's type.
__device__ __forceinline__ void store_row(const mgpu_k::ChainStage& st, int row, float v) {
    if (st.ytype == MGPU_F32) reinterpret_cast<float*>(st.y)[row] = v;
    else if (st.ytype == MGPU_F16) reinterpret_cast<__half*>(st.y)[row] = __float2half_rn(v);
    else reinterpret_cast<__nv_bfloat16*>(st.y)[row] = __float2bfloat16_rn(v);
}

template <int QT, int NC>
__global__ void __launch_bounds__(NC + 32, 1) gemv_chain_kernel(ChainArgs a) {
    constexpr int RPT = ChainGeom<QT, NC>::RPT;
    constexpr int kWarps = NC / 32;  // consumer warps; one more warp is the producer
    constexpr int BB = QTraits<QT>::kBlockBytes;
    constexpr int NW = QTraits<QT>::kWords;
    constexpr uint32_t kChunk = ChainGeom<QT, NC>::kChunk;
    constexpr int R = kChainF * RPT;            // rows per thread between two reductions
    constexpr int kPartFloats = R * (NC / 32);  // row partials of one reduction: rows x warps per row
    extern __shared__ __align__(1024) uint8_t smem[];
    __shared__ __align__(8) uint64_t full_bar[kChainMaxSlots];
    __shared__ __align__(8) uint64_t empty_bar[kChainMaxSlots];
    __shared__ unsigned long long s_epoch;
    __shared__ int s_abort_storage;
    __shared__ uint32_t s_refuse;
    volatile int* s_abort = &s_abort_storage;

    const int tid = threadIdx.x;
    const int warp = tid >> 5, lane = tid & 31;
    const int G = gridDim.x, b = blockIdx.x;
    const int S = a.slots;

    if (tid == 0) {
        for (int s = 0; s < S; ++s) {
            mbar_init(&full_bar[s], 1);
            mbar_init(&empty_bar[s], kWarps);
        }
        *s_abort = 0;
        // Launches so far: every CTA reads the counter here, before it takes its finish ticket,
        // and the last CTA to take one advances it.  A failed earlier launch may have left flags
        // behind: then nothing runs.
        s_epoch = *reinterpret_cast<const volatile unsigned long long*>(a.sync);
        s_refuse = poisoned(a.sync) ? 1u : 0u;
        if (s_refuse) atomicExch(a.status, (int)MGPU_ERR_DEVICE_TIMEOUT);
        fence_mbar_init();
        if (a.times) atomicMin(a.times + a.n_stages, (unsigned long long)globaltimer());
    }

    uint8_t* ring = smem;
    uint32_t* planes = reinterpret_cast<uint32_t*>(smem + (size_t)S * kChunk);
    float* bscale = reinterpret_cast<float*>(planes + kXPlanes * (kChainMaxK / 4));
    float* part = bscale + kChainMaxK / 32;  // two buffers of kPartFloats
    // the stage table, copied once (every link's record is then a shared-memory read), and this
    // CTA's rows [r0, r1) of every stage, worked out once
    mgpu_k::ChainStage* table = reinterpret_cast<mgpu_k::ChainStage*>(part + 2 * 128);
    int2* rows = reinterpret_cast<int2*>(table + a.n_stages);
    {
        const uint4* src = reinterpret_cast<const uint4*>(a.stages);
        uint4* dst = reinterpret_cast<uint4*>(table);
        const int n16 = a.n_stages * (int)(sizeof(mgpu_k::ChainStage) / 16);
        for (int i = tid; i < n16; i += NC + 32) dst[i] = __ldg(src + i);
        for (int i = tid; i < a.n_stages; i += NC + 32) {
            const long long N = __ldg(&a.stages[i].N);
            rows[i] = make_int2((int)(N * b / G), (int)(N * (b + 1) / G));
        }
    }
    __syncthreads();
    const bool refuse = s_refuse != 0u;
    // a stage's counter counts the CTAs that finished it over all launches: this launch's CTAs
    // have all finished it when it reaches (launches before this one + 1) * G
    const unsigned long long target = (s_epoch + 1ull) * (unsigned long long)G;

    if (warp == kWarps) {
        // ---------------- producer: every stage's rows of this CTA, in stage order ----------------
        if (lane == 0 && !refuse) {
            int g = 0, slot = 0;  // chunks issued so far; ring slot and phase of the next one
            uint32_t ph = 0;
            bool ok = true;
            for (int s = 0; s < a.n_stages && ok; ++s) {
                const mgpu_k::ChainStage& st = table[s];
                const int lg = __ffs(st.K >> 5) - 1;  // log2 of the blocks per row
                const int TR = (NC >> lg) * RPT;
                const int r0 = rows[s].x, r1 = rows[s].y;
                for (int row = r0; row < r1; row += TR) {
                    if (!chain_mbar_wait(&empty_bar[slot], ph ^ 1u, a, s_abort)) {
                        ok = false;
                        break;
                    }
                    const uint32_t bytes = (uint32_t)min(TR, r1 - row) * st.row_bytes;
                    mbar_arrive_expect_tx(&full_bar[slot], bytes);
                    bulk_g2s(ring + (size_t)slot * kChunk, st.W + (size_t)row * st.row_bytes, bytes, &full_bar[slot]);
                    ++g;
                    if (++slot == S) {
                        slot = 0;
                        ph ^= 1u;
                    }
                }
            }
            if (!ok) {
                // Let the copies already issued land before the CTA exits.
                for (int k = g - S > 0 ? g - S : 0; k < g; ++k)
                    mbar_wait(&full_bar[k % S], (uint32_t)((k / S) & 1), nullptr);
            }
        }
    } else if (!refuse) {
        // ---------------- consumers ----------------
        int slot = 0, pbuf = 0;
        uint32_t ph = 0;
        bool abort = false;
        for (int s = 0; s < a.n_stages; ++s) {
            const mgpu_k::ChainStage& st = table[s];
            const int K = st.K, nb = K >> 5, words = K >> 2;
            const int lg = __ffs(nb) - 1;  // nb = K / 32 is a power of two (32 .. 256)
            const int RP = NC >> lg, TR = RP * RPT;
            const int r0 = rows[s].x, r1 = rows[s].y;
            const int nch = (r1 - r0 + TR - 1) >> (__ffs(TR) - 1);

            // wait (one thread) for the stage that writes the input; the barrier also keeps the
            // previous stage's readers of the activation planes ahead of their rewrite
            {
                bool ok = true;
                if (st.dep >= 0 && tid == 0) ok = wait_stage(a, st.dep, target, s_abort);
                if (barrier_or<NC>(abort || !ok)) {
                    abort = true;
                    break;
                }
            }
            // the input vector, in fixed point, to shared memory
            if (K <= NC * 4) prepare_x_chain<NC, 1>(st, planes, bscale, tid);
            else if (K <= NC * 8) prepare_x_chain<NC, 2>(st, planes, bscale, tid);
            else prepare_x_chain<NC, kChainMaxK / (NC * 4)>(st, planes, bscale, tid);
            if (barrier_or<NC>(abort)) {
                abort = true;
                break;
            }
            const int col = tid & (nb - 1), rslot = tid >> lg, wpr = nb >> 5;
            XFixed xf;
            load_xfixed(planes, bscale, words, col, xf);
            const uint32_t par4 = (uint32_t)(tid * BB) & 3u;  // block starts at byte 0 or 2 of a word
            const uint32_t sel = par4 ? 0x7654u : 0x5432u;
            const uint32_t dsel = par4 ? 0x4432u : 0x4410u;
            const uint32_t toff = (uint32_t)(tid * BB) - par4;

            float acc[R];
#pragma unroll
            for (int i = 0; i < R; ++i) acc[i] = 0.0f;
            for (int c0 = 0; c0 < nch; c0 += kChainF) {
                // up to kChainF chunks, then one reduction of their rows
#pragma unroll
                for (int f = 0; f < kChainF; ++f) {
                    if (c0 + f < nch) {
                        if (!abort && !chain_mbar_wait(&full_bar[slot], ph, a, s_abort)) abort = true;
                        if (!abort) {
                            const uint8_t* stg = ring + (size_t)slot * kChunk + toff;
#pragma unroll
                            for (int i = 0; i < RPT; ++i) {
                                const uint32_t* wp = reinterpret_cast<const uint32_t*>(stg + i * (NC * BB));
                                uint32_t w[NW];
#pragma unroll
                                for (int q = 0; q < NW; ++q) w[q] = wp[q];
                                acc[f * RPT + i] = q_block_dot<QT, NW>(w, sel, dsel, xf);
                            }
                        }
                        __syncwarp();
                        if (lane == 0) mbar_arrive(&empty_bar[slot]);
                        if (++slot == S) {
                            slot = 0;
                            ph ^= 1u;
                        }
                    }
                }
                // reduce across the lanes, then across the warps of a row slot through shared
                // memory (double-buffered, so one barrier per reduction), and store the rows
                // (a group of one chunk, as the smallest GEMVs have, reduces only its RPT rows)
                int ri;
                float v;
                bool holder;
                if (c0 + 1 >= nch) {
                    float a1[RPT];
#pragma unroll
                    for (int i = 0; i < RPT; ++i) a1[i] = acc[i];
                    v = warp_reduce_rows<RPT>(a1, lane, ri);
                    holder = (lane & ((32 / RPT) - 1)) == 0;
                } else {
                    v = warp_reduce_rows<R>(acc, lane, ri);
                    holder = (lane & ((32 / R) - 1)) == 0;
                }
                float* pb = part + pbuf * kPartFloats;
                const int fc = ri / RPT, i = ri % RPT;
                if (holder) pb[(fc * TR + rslot + RP * i) * wpr + (warp % wpr)] = v;
                if (barrier_or<NC>(abort)) {
                    abort = true;
                    break;
                }
                const int row0 = r0 + c0 * TR;
                const int nrows = min(kChainF * TR, r1 - row0);
                if (tid < nrows) {
                    float sum = 0.0f;
                    for (int w = 0; w < wpr; ++w) sum += pb[tid * wpr + w];
                    store_row(st, row0 + tid, sum);
                }
                pbuf ^= 1;
            }
            if (abort) break;
            // Every CTA adds to the counter of a stage a later stage reads, rows or none, once
            // all its consumers have stored their rows (the barrier); the release reduction makes
            // those stores visible before the count.
            if (st.post) {
                if (barrier_or<NC>(abort)) break;
                if (tid == NC - 32) red_release_add_u64(a.flags + (size_t)s * kFlagStride, 1ull);
            }
            if (a.times && tid == 0 && nch > 0) atomicMax(a.times + s, (unsigned long long)globaltimer());
        }
    }
    __syncthreads();
    if (tid == 0) {
        __threadfence();
        const unsigned int t = atomicAdd(a.sync + 2, 1u);
        if (t == (unsigned)(G - 1)) {
            // the last CTA: every CTA has read the launch counter; advance it for the next launch
            a.sync[2] = 0u;
            __threadfence();
            atomicAdd(reinterpret_cast<unsigned long long*>(a.sync), 1ull);
        }
    }
}

template <int QT, int NC>
cudaError_t launch_chain(const mgpu_k::LaunchCtx& c, const mgpu_k::ChainStage* stages, int n, unsigned int* sync,
                         unsigned long long* flags, unsigned long long* times) {
    auto kern = gemv_chain_kernel<QT, NC>;
    constexpr uint32_t kChunk = ChainGeom<QT, NC>::kChunk;
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    int max_optin = 0;
    e = cudaDeviceGetAttribute(&max_optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
    if (e != cudaSuccess) return e;
    // the ring takes what the activation planes, the partials, the stage table and the
    // kernel's static shared memory (barriers, flags) leave
    cudaFuncAttributes fa;
    e = cudaFuncGetAttributes(&fa, kern);
    if (e != cudaSuccess) return e;
    const size_t table = (size_t)n * (sizeof(mgpu_k::ChainStage) + sizeof(int2));
    const size_t fixed = kChainPlaneBytes + kChainPartBytes + table + fa.sharedSizeBytes;
    if ((size_t)max_optin < fixed + 2 * kChunk) return cudaErrorInvalidConfiguration;
    int slots = (int)(((size_t)max_optin - fixed) / kChunk);
    slots = slots > kChainMaxSlots ? kChainMaxSlots : slots;
    const size_t smem = (size_t)slots * kChunk + kChainPlaneBytes + kChainPartBytes + table;
    e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    int per_sm = 0;
    e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, NC + 32, smem);
    if (e != cudaSuccess) return e;
    if (per_sm < 1) return cudaErrorInvalidConfiguration;
    ChainArgs args;
    args.stages = stages;
    args.n_stages = n;
    args.slots = slots;
    args.sync = sync;
    args.flags = flags;
    args.times = times;
    args.status = c.status;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(c.sm_count);
    cfg.blockDim = dim3(NC + 32);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = c.stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeCooperative;
    attr[0].val.cooperative = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kern, args);
}

}  // namespace

namespace mgpu_k {

bool chain_shape_ok(int K) { return K >= 1024 && K <= kChainMaxK && K % 1024 == 0 && (kChainNC % (K / 32)) == 0; }

int chain_max_links() { return kChainMaxStages; }

size_t chain_flag_bytes(int) { return (size_t)kChainMaxStages * kFlagStride * sizeof(unsigned long long); }

cudaError_t gemv_chain(const LaunchCtx& c, int qtype, const ChainStage* stages, int n, unsigned int* sync,
                       unsigned long long* flags, unsigned long long* times) {
    if (n <= 0) return cudaSuccess;
    if (n > kChainMaxStages) return cudaErrorInvalidValue;
    if (qtype == MGPU_Q4_0) return launch_chain<MGPU_Q4_0, kChainNC>(c, stages, n, sync, flags, times);
    if (qtype == MGPU_Q8_0) return launch_chain<MGPU_Q8_0, kChainNC>(c, stages, n, sync, flags, times);
    return cudaErrorInvalidValue;
}

}  // namespace mgpu_k
