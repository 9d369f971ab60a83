// peer.cu - exchanges between the GPUs of one node over NVLink, through peer memory.
//
// The N-GPU decode step moves a few KB per token: every GPU's bf16 hidden state to every other
// GPU (an all-gather before the column-sharded lm_head) and each sequence's greedy
// (index, value) pair to the GPU that owns the sequence (an all-to-all after it).  A collective
// library call costs ~15 us per round trip at these sizes; here one small kernel per exchange
// stores this GPU's bytes straight into every peer's receive slots (plain stores to peer memory
// mapped through CUDA IPC; no multicast, no TMA), then publishes one flag per peer and waits for
// the peers' flags.
//
// Memory layout of a group (one allocation per GPU, shared with the peers by CUDA IPC):
//   [world slots of slot_bytes][world u64 flags][u64 epoch]
// Flag f on GPU g holds the number of the last exchange whose bytes GPU f has finished storing
// into GPU g's slot f.  Every GPU runs the same exchanges in the same order, so their epoch
// counters agree; flags only grow.  The writer's ordering: the CTA's stores, bar.sync, then per
// peer a system-scope fence and a release store of the flag.  The reader: an acquire load of
// each flag until it reaches this exchange's number (bounded by a %globaltimer limit, after
// which the kernel records MGPU_ERR_DEVICE_TIMEOUT and returns); the slots are read by later
// kernels of the stream, after this one has completed.
//
// Reuse: a peer may store its next exchange on a group into this GPU's slots as soon as its own
// previous exchange on the group completed, which does not wait for this GPU to have read them.
// In the decode step two groups alternate (the hidden states' all-gather, the pairs'
// all-to-all) and every GPU reads a group's slots before it joins the other group's exchange;
// a peer's next exchange on the first group comes after its exchange on the second, which
// completes only once this GPU has published its flag there, i.e. after it read the slots.
// A caller without such an intervening exchange must alternate two groups itself.
#include "common.cuh"
#include "kernels.h"

using namespace mgpu_dev;

namespace {

__device__ __forceinline__ void st_release_sys_u64(unsigned long long* p, unsigned long long v) {
    asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ unsigned long long ld_acquire_sys_u64(const unsigned long long* p) {
    unsigned long long v;
    asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}

__global__ void __launch_bounds__(256) peer_exchange_kernel(mgpu_k::PeerExchangeArgs a) {
    __shared__ unsigned long long s_epoch;
    const int tid = threadIdx.x;
    if (tid == 0) s_epoch = *a.epoch + 1;
    __syncthreads();
    const unsigned long long ep = s_epoch;
    // 16-byte stores when sizes and offsets allow, else 8-byte ones (e.g. 8-byte argmax pairs)
    const bool wide = a.bytes % 16 == 0 && a.slot_bytes % 16 == 0 && a.src_stride % 16 == 0;
    for (int p = 0; p < a.world; ++p) {
        const uint8_t* s = a.src + (a.src_stride ? (size_t)p * a.src_stride : 0);
        uint8_t* d = a.dst[p] + (size_t)a.rank * a.slot_bytes;
        if (wide) {
            for (size_t i = tid; i < a.bytes / 16; i += blockDim.x)
                reinterpret_cast<uint4*>(d)[i] = reinterpret_cast<const uint4*>(s)[i];
        } else {
            for (size_t i = tid; i < a.bytes / 8; i += blockDim.x)
                reinterpret_cast<uint2*>(d)[i] = reinterpret_cast<const uint2*>(s)[i];
        }
    }
    __syncthreads();
    if (tid < a.world) {
        // every store of the CTA is ordered before this thread's flag (bar.sync, then a
        // cumulative system-scope fence and release)
        __threadfence_system();
        st_release_sys_u64(a.dst_flag[tid] + a.rank, ep);
    }
    if (tid == 0) {
        const uint64_t t0 = globaltimer();
        bool ok = true;
        for (int p = 0; p < a.world && ok; ++p) {
            while (ld_acquire_sys_u64(a.my_flags + p) < ep) {
                if (globaltimer() - t0 > a.limit_ns) {
                    if (a.status) atomicExch(a.status, (int)MGPU_ERR_DEVICE_TIMEOUT);
                    ok = false;
                    break;
                }
            }
        }
        *a.epoch = ep;
    }
    __syncthreads();
}

}  // namespace

namespace mgpu_k {

cudaError_t peer_exchange(const LaunchCtx& c, const PeerExchangeArgs& a) {
    if (a.world < 1 || a.world > kMaxPeers || a.rank < 0 || a.rank >= a.world || a.bytes % 8 != 0 ||
        a.slot_bytes % 8 != 0 || a.bytes > a.slot_bytes)
        return cudaErrorInvalidValue;
    peer_exchange_kernel<<<1, 256, 0, c.stream>>>(a);
    return cudaGetLastError();
}

}  // namespace mgpu_k
