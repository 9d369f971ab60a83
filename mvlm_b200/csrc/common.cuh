// common.cuh - sm_100a device helpers shared by the mvlm_b200 kernels: bounded mbarrier
// waits, bulk / tensor (TMA) copies (CTA-local destinations only), tcgen05 (TMEM + UMMA) wrappers and
// element conversions.  Every wait on a barrier is bounded by a %globaltimer deadline; on
// expiry the kernel records MGPU_ERR_DEVICE_TIMEOUT in the per-device status word and
// returns instead of spinning.
#pragma once
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/mgpu_cuda.h"
#include "kernels.h"

namespace mgpu_dev {

// Two seconds: every kernel in this library finishes in well under a millisecond, so a
// wait this long means a barrier will never complete.
constexpr uint64_t kWaitLimitNs = 2000000000ull;

__device__ __forceinline__ uint64_t globaltimer() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// ------------------------------------------------------------------ mbarrier --------
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}
__device__ __forceinline__ void fence_mbar_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.release.cta.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.release.cta.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
                 "r"(bytes)
                 : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n .reg .pred p;\n"
        " mbarrier.try_wait.parity.acquire.cta.shared::cta.b64 p, [%1], %2, %3;\n"
        " selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity), "r"(1000000u)
        : "memory");
    return ok != 0;
}
// Bounded wait for the phase with the given parity to complete.  Returns false (after
// recording the timeout) when the deadline passes.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, int* status,
                                          uint64_t limit_ns = kWaitLimitNs) {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = globaltimer();
    while (true) {
        if (mbar_try_wait(bar, parity)) return true;
        if (globaltimer() - t0 > limit_ns) {
            if (status) atomicExch(status, (int)MGPU_ERR_DEVICE_TIMEOUT);
            return false;
        }
    }
}

// ------------------------------------------------------------------ copies ----------
// 1-D bulk copy global -> shared, completion signalled on `bar` (complete_tx).  src, dst
// 16-byte aligned; bytes a multiple of 16.  The destination is this CTA's own shared memory.
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
            smem_u32(dst)),
        "l"(src), "r"(bytes), "r"(smem_u32(bar))
        : "memory");
}
// 2-D tensor-map (TMA) tile load into this CTA's shared memory.  x is the innermost coordinate.
__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int x, int y, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
            smem_u32(dst)),
        "l"(map), "r"(x), "r"(y), "r"(smem_u32(bar))
        : "memory");
}
// 3-D tensor-map (TMA) tile load into this CTA's shared memory.  x is the innermost coordinate.
__device__ __forceinline__ void tma_load_3d(void* dst, const CUtensorMap* map, int x, int y, int z, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], [%5];" ::"r"(
            smem_u32(dst)),
        "l"(map), "r"(x), "r"(y), "r"(z), "r"(smem_u32(bar))
        : "memory");
}
__device__ __forceinline__ void prefetch_tensormap(const CUtensorMap* map) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(map) : "memory");
}
// Make this thread's generic-proxy shared-memory writes visible to the async proxy
// (tcgen05.mma operand reads).
__device__ __forceinline__ void fence_proxy_async_smem() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
__device__ __forceinline__ void named_barrier_sync(int id, int threads) {
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}

// ------------------------------------------------------------------ tcgen05 ---------
__device__ __forceinline__ void tmem_alloc(uint32_t* dst_smem, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst_smem)),
                 "r"(ncols)
                 : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
__device__ __forceinline__ void tc_fence_before() {
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
// D(tmem) (+)= A(smem desc) * B(smem desc), kind::f16 (fp16 or bf16 operands, fp32 accum).
__device__ __forceinline__ void umma_f16(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                         uint32_t accumulate) {
    asm volatile(
        "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
        " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}\n" ::"r"(d_tmem),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
}
// Arrive on `bar` once all previously issued tcgen05.mma of this thread have completed.
__device__ __forceinline__ void umma_commit(uint64_t* bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                     smem_u32(bar))
                 : "memory");
}
// ------------------------------------------------------------------ CTA pairs -------
// Two CTAs of a (2,1,1) cluster share one 256-row tile through tcgen05 cta_group::2: the
// even CTA issues the MMAs, which read A and B from both CTAs' shared memory at the same
// offsets and write each CTA's 128 accumulator rows into that CTA's own TMEM.
__device__ __forceinline__ uint32_t cluster_ctarank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}
// Address of the same shared-memory object in CTA `rank` of the cluster.
__device__ __forceinline__ uint32_t cluster_addr(const void* p, uint32_t rank) {
    uint32_t d;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(d) : "r"(smem_u32(p)), "r"(rank));
    return d;
}
// Arrive on a barrier of a CTA of this cluster (default .release.cta semantics, as for a local
// arrive: the writer's preceding fence.proxy.async orders its shared-memory writes before the
// pair's MMAs that the arrival releases).
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t cl_addr) {
    asm volatile("mbarrier.arrive.shared::cluster.b64 _, [%0];" ::"r"(cl_addr) : "memory");
}
// Every thread of both CTAs of the cluster.
__device__ __forceinline__ void cluster_sync_all() {
    asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// Pair TMEM allocation: issued by the same warp of both CTAs, same destination offset.
__device__ __forceinline__ void tmem_alloc_pair(uint32_t* dst_smem, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst_smem)),
                 "r"(ncols)
                 : "memory");
}
__device__ __forceinline__ void tmem_relinquish_pair() {
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc_pair(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
// D (both CTAs' TMEM) (+)= A (both CTAs' smem, 128 rows each) * B (both CTAs' smem, N/2 rows each).
__device__ __forceinline__ void umma_f16_pair(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                              uint32_t accumulate) {
    asm volatile(
        "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
        " tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n}\n" ::"r"(d_tmem),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
}
// Arrive on this CTA's `bar` once the pair MMAs issued so far have completed.
__device__ __forceinline__ void umma_commit_pair(uint64_t* bar) {
    asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
                 : "memory");
}
// The same, arriving on `bar` at the same offset in both CTAs of the pair (`mask`: the pair's
// two bits of the cluster's CTA ranks).
__device__ __forceinline__ void umma_commit_pair_both(uint64_t* bar, uint16_t mask) {
    asm volatile(
        "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;" ::"r"(
            smem_u32(bar)),
        "h"(mask)
        : "memory");
}
// 16 bytes of another CTA's shared memory (an address from cluster_addr).
__device__ __forceinline__ float4 ld_cluster_f4(uint32_t cl_addr) {
    float4 v;
    asm volatile("ld.shared::cluster.v4.f32 {%0, %1, %2, %3}, [%4];"
                 : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
                 : "r"(cl_addr)
                 : "memory");
    return v;
}
// 2-D tensor-map load into this CTA's own shared memory whose completion (bytes) is counted on
// the barrier at cluster address `bar_cl` (the even CTA's barrier of the pair).
__device__ __forceinline__ void tma_load_2d_pair(void* dst, const CUtensorMap* map, int x, int y, uint32_t bar_cl) {
    asm volatile(
        "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], "
        "[%4];" ::"r"(smem_u32(dst)),
        "l"(map), "r"(x), "r"(y), "r"(bar_cl)
        : "memory");
}

// 32 lanes x 32 consecutive fp32 columns: thread i of the warp gets TMEM lane (base + i).
__device__ __forceinline__ void tmem_ld_32x32b_x32(uint32_t taddr, float (&v)[32]) {
    uint32_t r[32];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
        "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
        "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]),
          "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]),
          "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]),
          "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
    for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

// Shared-memory matrix descriptor (tcgen05 "matrix descriptor"): start address, leading
// and stride byte offsets (>> 4), version 1 at bits 46-47, swizzle mode at bits 61-63.
constexpr uint32_t kSwizzle128B = 2;
__device__ __forceinline__ uint64_t smem_desc(uint32_t saddr, uint32_t lbo_bytes, uint32_t sbo_bytes,
                                              uint32_t swizzle) {
    uint64_t d = 0;
    d |= (uint64_t)((saddr >> 4) & 0x3FFF);
    d |= (uint64_t)((lbo_bytes >> 4) & 0x3FFF) << 16;
    d |= (uint64_t)((sbo_bytes >> 4) & 0x3FFF) << 32;
    d |= (uint64_t)1 << 46;
    d |= (uint64_t)(swizzle & 7) << 61;
    return d;
}
// Instruction descriptor for kind::f16: fp32 accumulator (c_format 1 at bits 4-5), A/B
// format at bits 7-9 / 10-12 (0 = f16, 1 = bf16), major-ness at bits 15 / 16 (0 = K-major,
// 1 = MN-major), N >> 3 at bits 17-22, M >> 4 at bits 24-28.
__host__ __device__ constexpr uint32_t idesc_f16(bool bf16, bool a_mn_major, bool b_mn_major, int M, int N) {
    return (1u << 4) | ((bf16 ? 1u : 0u) << 7) | ((bf16 ? 1u : 0u) << 10) | ((a_mn_major ? 1u : 0u) << 15) |
           ((b_mn_major ? 1u : 0u) << 16) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

// ------------------------------------------------------------------ conversions -----
template <typename T> __device__ __forceinline__ float to_f32(T v);
template <> __device__ __forceinline__ float to_f32<float>(float v) { return v; }
template <> __device__ __forceinline__ float to_f32<__half>(__half v) { return __half2float(v); }
template <> __device__ __forceinline__ float to_f32<__nv_bfloat16>(__nv_bfloat16 v) { return __bfloat162float(v); }
template <typename T> __device__ __forceinline__ T from_f32(float v);
template <> __device__ __forceinline__ float from_f32<float>(float v) { return v; }
template <> __device__ __forceinline__ __half from_f32<__half>(float v) { return __float2half_rn(v); }
template <> __device__ __forceinline__ __nv_bfloat16 from_f32<__nv_bfloat16>(float v) { return __float2bfloat16_rn(v); }

// ------------------------------------------------------------------ fused epilogue --

// act(v) in fp32, every form written as v * sigmoid(z) = v / (1 + exp(-z)):
//   SILU             z = v: the reference's v / (1 + exp(-v)) (activations.cl:48-56);
//   GELU             z = 2 inner, inner = sqrt(2/pi) (v + 0.044715 v^3): the tanh approximation
//                    0.5 v (1 + tanh(inner)) = v sigmoid(2 inner);
//   GELU_AS_SHIPPED  z = -2 inner: the reference's gelu kernel reverses tanh's sign
//                    (activations.cl:94-106 compute 1 - 2 / (1 + exp(-2a)) = -tanh(a)), so it
//                    outputs 0.5 v (1 - tanh(inner)) = v sigmoid(-2 inner).
// No form subtracts two nearly equal numbers (a 1 + tanh(.) form cancels where tanh is near -1,
// which turns tanh's absolute error into the whole result in the tails), so the relative error
// stays a few fp32 ulps for every finite v.  1 + exp(-z) = inf (z < -88) gives v * 0 = -0 or 0.
__device__ __forceinline__ float activate(int act, float v) {
    float z;
    if (act == MGPU_ACT_SILU) {
        z = v;
    } else if (act == MGPU_ACT_GELU || act == MGPU_ACT_GELU_AS_SHIPPED) {
        const float inner = 0.7978845608f * fmaf(0.044715f * v, v * v, v);
        z = act == MGPU_ACT_GELU ? 2.0f * inner : -2.0f * inner;
    } else {
        return v;
    }
    return __fdividef(v, 1.0f + __expf(-z));
}

__device__ __forceinline__ float load_float(const void* p, int type, size_t i) {
    if (type == MGPU_F32) return reinterpret_cast<const float*>(p)[i];
    if (type == MGPU_F16) return __half2float(reinterpret_cast<const __half*>(p)[i]);
    return __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(p)[i]);
}

__device__ __forceinline__ float epilogue_finish(const mgpu_k::Epilogue& e, int row, int n, float v) {
    v = activate(e.act, v);
    if (e.mul) v *= load_float(e.mul, e.mul_type, (size_t)row * e.ldm + n);
    if (e.resid) v += load_float(e.resid, e.resid_type, (size_t)row * e.ldr + n);
    return v;
}
// Eight values of an [M][ld] operand at (row, n) .. (row, n + 7); columns at or past N read 0.
__device__ __forceinline__ void load8(const void* p, int type, int64_t ld, int row, int n, int N, float (&o)[8]) {
    const size_t base = (size_t)row * ld + n;
    if (type == MGPU_F32) {
        const float* q = reinterpret_cast<const float*>(p) + base;
        if (n + 8 <= N && (reinterpret_cast<uintptr_t>(q) & 15) == 0) {
            const float4 a = reinterpret_cast<const float4*>(q)[0], b = reinterpret_cast<const float4*>(q)[1];
            o[0] = a.x; o[1] = a.y; o[2] = a.z; o[3] = a.w; o[4] = b.x; o[5] = b.y; o[6] = b.z; o[7] = b.w;
        } else {
#pragma unroll
            for (int i = 0; i < 8; ++i) o[i] = n + i < N ? q[i] : 0.0f;
        }
        return;
    }
    const uint16_t* q = reinterpret_cast<const uint16_t*>(p) + base;
    uint32_t w[4];
    if (n + 8 <= N && (reinterpret_cast<uintptr_t>(q) & 15) == 0) {
        const uint4 t = *reinterpret_cast<const uint4*>(q);
        w[0] = t.x; w[1] = t.y; w[2] = t.z; w[3] = t.w;
    } else {
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const uint32_t lo = n + 2 * i < N ? q[2 * i] : 0u, hi = n + 2 * i + 1 < N ? q[2 * i + 1] : 0u;
            w[i] = lo | (hi << 16);
        }
    }
    if (type == MGPU_BF16) {
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            o[2 * i] = __uint_as_float(w[i] << 16);
            o[2 * i + 1] = __uint_as_float(w[i] & 0xFFFF0000u);
        }
    } else {
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&w[i]));
            o[2 * i] = f.x;
            o[2 * i + 1] = f.y;
        }
    }
}

// The epilogue over one thread's 32 consecutive columns of a row (the tile epilogue's unit):
// each choice (activation, operand types) is taken once per 32 values, and the operands are
// read 16 bytes at a time, so the unrolled code stays small and its loads few.
template <int ACT>
__device__ __forceinline__ void activate32(float (&v)[32]) {
#pragma unroll
    for (int i = 0; i < 32; ++i) v[i] = activate(ACT, v[i]);
}
__device__ __forceinline__ void epilogue_row32(const mgpu_k::Epilogue& e, int row, int n0, int N, float (&v)[32]) {
    switch (e.act) {
        case MGPU_ACT_GELU: activate32<MGPU_ACT_GELU>(v); break;
        case MGPU_ACT_SILU: activate32<MGPU_ACT_SILU>(v); break;
        case MGPU_ACT_GELU_AS_SHIPPED: activate32<MGPU_ACT_GELU_AS_SHIPPED>(v); break;
        default: break;
    }
    if (e.mul) {
#pragma unroll
        for (int g = 0; g < 4; ++g) {
            float m[8];
            load8(e.mul, e.mul_type, e.ldm, row, n0 + 8 * g, N, m);
#pragma unroll
            for (int i = 0; i < 8; ++i) v[8 * g + i] *= m[i];
        }
    }
    if (e.resid) {
#pragma unroll
        for (int g = 0; g < 4; ++g) {
            float r[8];
            load8(e.resid, e.resid_type, e.ldr, row, n0 + 8 * g, N, r);
#pragma unroll
            for (int i = 0; i < 8; ++i) v[8 * g + i] += r[i];
        }
    }
}

__device__ __forceinline__ bool epilogue_active(const mgpu_k::Epilogue& e) {
    return e.act != MGPU_ACT_NONE || e.resid || e.mul;
}

__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
    uint32_t d;
    asm("prmt.b32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(sel));
    return d;
}

}  // namespace mgpu_dev
