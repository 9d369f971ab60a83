// kernels.h - host-side launchers of the sm_100a kernels (internal to libmgpu).
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

namespace mgpu_k {

// What a GEMM epilogue applies after its bias: C = act(v) * mul[row][n] + residual[row][n]
// (mgpu_act; mul and residual are [M][ld] of f32 / f16 / bf16, or null).  Default: nothing.
struct Epilogue {
    int act = 0;
    const void* resid = nullptr;
    int resid_type = 0;
    int64_t ldr = 0;
    const void* mul = nullptr;
    int mul_type = 0;
    int64_t ldm = 0;
};

struct LaunchCtx {
    cudaStream_t stream;
    int sm_count;
    int* status;      // per-device status word (MGPU_ERR_DEVICE_TIMEOUT on a bounded-wait expiry)
    void* workspace;  // per-device scratch arena, zero-initialised once, kept zero by its users
    size_t workspace_bytes;
};

// ---------------------------------------------------------------- GEMV (gemv.cu) ----
// y[N] = W[N][K] (GGUF blocks of qtype) . x[K]
cudaError_t gemv_q(const LaunchCtx& c, int qtype, const uint8_t* W, int xtype, const void* x, int ytype,
                   void* y, int N, int K);
// y[N] = W[N][K] . x[K] for dense W (f32 / f16 / bf16), row pitch ldw elements
cudaError_t gemv_nk(const LaunchCtx& c, int wtype, const void* W, int64_t ldw, int xtype, const void* x,
                    int ytype, void* y, int N, int K);
// y[N] = x[K] . W[K][N] for dense W (reference orientation), row pitch ldw elements.  Split
// over K with fp32 partials in scratch and a last-CTA reduction in fixed order.
cudaError_t gemv_kn(const LaunchCtx& c, int wtype, const void* W, int64_t ldw, int xtype, const void* x,
                    int ytype, void* y, int N, int K, float* partials, unsigned int* counters);
size_t gemv_kn_scratch_bytes(int N, int K, int sm_count, int* splits_out);
// Same as gemv_kn, with its scratch in a fixed device array of this library (no allocation).
// N <= gemv_kn_noalloc_max_n(); otherwise cudaErrorInvalidValue before any launch.
cudaError_t gemv_kn_noalloc(const LaunchCtx& c, int wtype, const void* W, int64_t ldw, int xtype, const void* x,
                            int ytype, void* y, int N, int K);
size_t gemv_kn_noalloc_max_n();
// gemv_q with x replaced by RMSNorm(x) = x * rsqrt(mean(x^2) + eps) * gamma (rounded to x's type)
// in the kernel's prologue.  cudaErrorNotSupported (nothing launched) for shapes the streaming
// kernel does not take; the caller then normalises first (rms_norm) and runs gemv_q.
cudaError_t gemv_q_norm(const LaunchCtx& c, int qtype, const uint8_t* W, int xtype, const void* x, int gtype,
                        const void* gamma, float eps, int ytype, void* y, int N, int K);

// ------------------------------------------------------- GEMV chain (chain.cu) ------
// One GEMV of a chain, as the kernel reads it from device memory (64 bytes).
struct ChainStage {
    const uint8_t* W;    // GGUF Q4_0 / Q8_0 rows [N][row_bytes]
    const void* x;       // input [K] of xtype: an external vector, or a view of stage dep's y
    void* y;             // output [N] of ytype
    int N, K;
    uint32_t row_bytes;
    int xtype, ytype;
    int dep;             // the stage whose output x is (-1: x is ready when the chain starts)
    int reserved[2];     // keeps the record at 64 bytes (the kernel copies it 16 bytes at a time)
    int post;            // 1: a later stage reads this one's output (the CTAs post their flags)
    int pad;
};
// K the chain kernel takes: 1024 .. 8192, K / 32 dividing its 512 consumer threads.
bool chain_shape_ok(int K);
// Links one chain may hold (its stage table is copied to shared memory).
int chain_max_links();
// Bytes of the per-stage counters a chain owns (zeroed once; the kernel only counts them up).
size_t chain_flag_bytes(int sm_count);
// One cooperative launch (one CTA per SM) over the n stages (all of qtype) at `stages` (device
// memory).  sync: 4 zeroed words owned by the chain (launch counter (u64), finish ticket,
// poison); flags: chain_flag_bytes zeroed bytes owned by the chain.  times: null, or n + 1
// words: per-stage end time (max over CTAs, %globaltimer ns; start at 0) and the launch's start
// (min over CTAs; start at ~0).
cudaError_t gemv_chain(const LaunchCtx& c, int qtype, const ChainStage* stages, int n, unsigned int* sync,
                       unsigned long long* flags, unsigned long long* times);

// ---------------------------------------------------------------- misc (misc.cu) ----
cudaError_t dequant(const LaunchCtx& c, int qtype, const uint8_t* W, int otype, void* out, int64_t n);
cudaError_t quantize(const LaunchCtx& c, int qtype, const float* src, uint8_t* dst, int64_t n);
cudaError_t fill_uniform(const LaunchCtx& c, int otype, void* out, int64_t n, uint64_t seed, float lo, float hi);
cudaError_t fill_normal(const LaunchCtx& c, int otype, void* out, int64_t n, uint64_t seed, float sigma);
cudaError_t convert(const LaunchCtx& c, int itype, const void* in, int otype, void* out, int64_t n);
// One CTA waits on an mbarrier that never completes, bounded by limit_ns.
cudaError_t selftest_bounded_wait(const LaunchCtx& c, uint64_t limit_ns);
// out[0] = argmax index, out[1] = the value (fp32 bits), reference argmax semantics; n >= 1.
cudaError_t argmax(const LaunchCtx& c, int type, const void* logits, int n, int* out);
// The same for `rows` rows of n values, row r at element r * ld: pair r at out[2r], out[2r+1].
cudaError_t argmax_rows(const LaunchCtx& c, int type, const void* logits, int rows, int n, int64_t ld, int* out);
// out[r][:] = RMSNorm(in[r][:]) for rows r < rows of H values (in / out of `type`, w of wtype).
cudaError_t rms_norm(const LaunchCtx& c, int type, const void* in, void* out, int wtype, const void* w, int rows,
                     int H, float eps);
// The global first maximum of a row column-sharded over n_ranks, from the ranks' argmax pairs.
cudaError_t argmax_combine(const LaunchCtx& c, const int* pairs, int n_ranks, int n_total, int* out);
// patches[p][k] (k < kpad, zero for k >= C*ph*pw) from image [C][H][W]; same element type
cudaError_t im2col(const LaunchCtx& c, int type, const void* img, void* patches, int C, int H, int W, int ph,
                   int pw, int kpad);

// ---------------------------------------------------------------- GEMM (gemm_tc.cu) --
struct GemmOperand {
    const void* ptr;
    int type;     // MGPU_F16 / MGPU_BF16 / MGPU_Q4_0 / MGPU_Q8_0 / MGPU_F32 (C only)
    int layout;   // MGPU_LAYOUT_KN / MGPU_LAYOUT_NK (B only)
    int64_t ld;   // row pitch in elements (dense) or bytes (quantised rows)
};
// How gemm() runs a shape: B mode, tile, and split-K.
struct GemmPlan {
    int bmode, BN, mt, cg, csplit, tiles_m, tiles_n, num_kb, splits, kb_per_split;
};
GemmPlan plan_gemm(const LaunchCtx& c, const GemmOperand& A, const GemmOperand& B, int M, int N, int K);
// Split-K scratch: one ticket per output tile (zero between calls; the kernel leaves it so)
// and fp32 partials for splits x M x N.
struct GemmSplitScratch {
    unsigned int* tickets;
    size_t max_tickets;
    float* partials;
    size_t max_partials;  // floats
};
// Bytes of fp32 partials gemm() uses for this shape (0: it does not split K).
size_t gemm_split_bytes(const LaunchCtx& c, const GemmOperand& A, const GemmOperand& B, int M, int N, int K);
// C[M,N] = A[M,K] * op(B) (+ bias[N]); A row-major [M][lda].  `split` may be null (no
// split-K, whatever the plan says).
cudaError_t gemm(const LaunchCtx& c, const GemmOperand& A, const GemmOperand& B, const GemmOperand& C,
                 const void* bias, int bias_type, int M, int N, int K, const GemmSplitScratch* split,
                 const Epilogue& epi = Epilogue());
// Skinny GEMM for batched decode (skinny.cu): Q4_0 W [N][K/32] rows, bf16/fp16 A, M <= 32.
bool skinny_ok(const GemmOperand& A, const GemmOperand& B, int M, int N, int K);
cudaError_t gemm_q4_skinny(const LaunchCtx& c, const GemmOperand& A, const GemmOperand& B, const GemmOperand& C,
                           const void* bias, int bias_type, int M, int N, int K, const Epilogue& epi = Epilogue());
// A 3-D TMA map over 16-bit units without swizzle: extents dims[0] (contiguous), dims[1],
// dims[2]; byte strides of dims 1 and 2 (multiples of 16, in any order); box {box[0..2]}.
bool make_tensor_map_u16_3d(CUtensorMap* m, const void* ptr, const int64_t dims[3], const int64_t strides[2],
                            const int box[3]);
// Exchange over peer memory (peer.cu): this GPU's `bytes` (from src, or src + p * src_stride
// for peer p) into slot `rank` of every peer's receive region, then one flag per peer, then a
// bounded wait for every peer's flag of this exchange.
constexpr int kMaxPeers = 8;
struct PeerExchangeArgs {
    const uint8_t* src;
    size_t src_stride;  // 0: the same bytes to every peer (all-gather); else per-peer chunks (all-to-all)
    size_t bytes;       // per peer, a multiple of 8, <= slot_bytes (a multiple of 8)
    size_t slot_bytes;
    uint8_t* dst[kMaxPeers];                  // peer p's receive slots (this GPU's own for p == rank)
    unsigned long long* dst_flag[kMaxPeers];  // peer p's flags
    unsigned long long* my_flags;             // this GPU's flags (world entries)
    unsigned long long* epoch;                // this GPU's exchange counter
    int rank, world;
    uint64_t limit_ns;
    int* status;
};
cudaError_t peer_exchange(const LaunchCtx& c, const PeerExchangeArgs& a);
// Why a GEMM request cannot run (nullptr when it can).
const char* gemm_check(const GemmOperand& A, const GemmOperand& B, const GemmOperand& C, int M, int N, int K);

}  // namespace mgpu_k
