/*
 * mgpu_cuda.h - C ABI of the B200 (sm_100a) matmul path that replaces MVLM's OpenCL
 * GEMM/GEMV dispatch.  Plain pointers, sizes and opaque handles only.
 *
 * Each entry point cites the reference interface it stands in for (paths relative to the
 * drxddy/MVLM project root).  The C++ mirror with the reference's own names and types
 * (mgpu::dispatch_gemm_image, cl_mem, cl_event, ...) is include/mgpu_compute.hpp.
 *
 * Conventions (the reference's, src/engine/compute.cpp:12-17):
 *   - Functions returning a handle return NULL on error; the reason is in
 *     mgpu_last_error() / mgpu_last_error_string() (thread-local).  Nothing aborts.
 *   - Work is enqueued in order on the device's single stream (the reference's one in-order
 *     queue, src/engine/device.cpp:297-300); no call synchronises implicitly except
 *     mgpu_buf_read/write, mgpu_wait_event and mgpu_finish.
 *   - A device handle is used by one host thread at a time.
 *   - The GEMV and GEMM kernels overlap the kernel before them in the stream: they start
 *     reading their weight operand (W / B) before that kernel has finished, and read
 *     activations and write outputs only after it.  A weight buffer must therefore not be
 *     written by the GEMV or GEMM call enqueued directly before the call that reads it as
 *     weights (uploads, copies, conversions and any other enqueued work may precede it).
 */
#ifndef MGPU_CUDA_H
#define MGPU_CUDA_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Element / block types.  Values are ggml's GGMLType (src/models/gguf_loader.h:12-30);
 * BF16 carries ggml's value 30, which the reference's enum does not list. */
enum mgpu_type {
    MGPU_F32 = 0,
    MGPU_F16 = 1,
    MGPU_Q4_0 = 2,
    MGPU_Q8_0 = 8,
    MGPU_BF16 = 30
};

/* Storage order of a 2-D weight.
 * KN: B[K][N] row-major, the orientation the reference kernels read (gemm.cl:28,159,221).
 * NK: W[N][K] rows, GGUF-native (ne0 = K fastest); the only order for Q4_0/Q8_0. */
enum mgpu_layout {
    MGPU_LAYOUT_KN = 0,
    MGPU_LAYOUT_NK = 1
};

/* Error codes returned by mgpu_last_error(). */
enum mgpu_status {
    MGPU_OK = 0,
    MGPU_ERR_INVALID_ARG = 1,   /* null handle, bad shape / type / layout / alignment */
    MGPU_ERR_UNSUPPORTED = 2,   /* valid request this build does not implement */
    MGPU_ERR_CUDA = 3,          /* a CUDA runtime / driver call failed */
    MGPU_ERR_OUT_OF_MEMORY = 4,
    MGPU_ERR_DEVICE_TIMEOUT = 5 /* a kernel's bounded wait expired; its output is invalid */
};

typedef struct mgpu_device mgpu_device; /* replaces DeviceInfo (src/engine/device.h:13-55) */
typedef struct mgpu_buf mgpu_buf;       /* replaces cl_mem */
typedef struct mgpu_event mgpu_event;   /* replaces cl_event */
typedef void* mgpu_program;             /* replaces cl_program; accepted and ignored */

/* Binary-compatible with TensorInfo (src/models/gguf_loader.h:51-58), so a caller can pass
 * the reference loader's `const TensorInfo*` directly. */
typedef struct mgpu_tensor_info {
    char name[256];
    uint32_t n_dims;
    uint64_t dims[4];
    uint32_t type;
    uint64_t offset;
    size_t data_size;
} mgpu_tensor_info;

/* ---------------------------------------------------------------- errors ---------- */
int mgpu_last_error(void);
const char* mgpu_last_error_string(void);
void mgpu_clear_error(void);

/* ---------------------------------------------------------------- device ---------- */
/* init_device (src/engine/device.h:58): select CUDA device `ordinal`, create the in-order
 * stream and the per-device status word.  NULL on failure. */
mgpu_device* mgpu_init_device(int ordinal);
void mgpu_release_device(mgpu_device* dev);
int mgpu_device_ordinal(const mgpu_device* dev);
int mgpu_device_sm_count(const mgpu_device* dev);
size_t mgpu_device_l2_bytes(const mgpu_device* dev);
/* The cudaStream_t all dispatches are enqueued on.  mgpu_set_stream replaces it (the caller
 * keeps ownership of a stream it passes in; NULL restores the device's own stream). */
void* mgpu_device_stream(const mgpu_device* dev);
int mgpu_set_stream(mgpu_device* dev, void* cuda_stream);
/* 0: dispatches return NULL (no event recorded, like passing no event in OpenCL);
 * 1: dispatches return a completion event; 2 (default): a profiling event whose
 * mgpu_profile_end gives the launch's device time, like CL_QUEUE_PROFILING_ENABLE. */
int mgpu_set_event_mode(mgpu_device* dev, int mode);
/* clFinish: wait for all enqueued work, then report any kernel status (timeouts). */
int mgpu_finish(mgpu_device* dev);

/* ---------------------------------------------------------------- memory ---------- */
/* create_buffer (src/engine/memory.h:19): device allocation, optionally filled from host. */
mgpu_buf* mgpu_create_buffer(mgpu_device* dev, size_t bytes, const void* host_src);
/* create_weight_image (src/engine/memory.h:16, memory.cpp:28-79): fp16 weight of `rows` x
 * `cols` (the reference kernels read it as B[K=rows][N=cols]).  Stored KN with the row pitch
 * padded with zeros to a multiple of 8 elements (the reference pads to 4 for RGBA texels). */
mgpu_buf* mgpu_create_weight_image(mgpu_device* dev, int rows, int cols, const uint16_t* data);
/* Wrap caller-owned device memory (e.g. a torch tensor's data_ptr); not freed on release. */
mgpu_buf* mgpu_wrap_buffer(mgpu_device* dev, void* device_ptr, size_t bytes);
/* A sub-range view of a buffer (shares memory; released independently). */
mgpu_buf* mgpu_buf_view(mgpu_buf* buf, size_t offset, size_t bytes);
/* Tag a buffer's contents: element/block type, layout, logical rows x cols and row pitch in
 * elements (0 = dense).  Untagged buffers are MGPU_F16 / KN, which is what the reference's
 * cl_mem arguments hold. */
int mgpu_buf_set_format(mgpu_buf* buf, int type, int layout, int64_t rows, int64_t cols, int64_t ld);
void* mgpu_buf_device_ptr(const mgpu_buf* buf);
size_t mgpu_buf_bytes(const mgpu_buf* buf);
/* Blocking host<->device copies (clEnqueueWrite/ReadBuffer with blocking=CL_TRUE). */
int mgpu_buf_write(mgpu_buf* buf, size_t offset, const void* src, size_t bytes);
int mgpu_buf_read(const mgpu_buf* buf, size_t offset, void* dst, size_t bytes);
/* Stream-ordered copies (clEnqueueWrite/ReadBuffer with blocking=CL_FALSE); host memory
 * should be pinned (mgpu_host_alloc) for the copy to be asynchronous. */
int mgpu_buf_write_async(mgpu_buf* buf, size_t offset, const void* src, size_t bytes);
int mgpu_buf_read_async(const mgpu_buf* buf, size_t offset, void* dst, size_t bytes);
/* Stream-ordered device-to-device copy between two buffers of one device
 * (clEnqueueCopyBuffer, used by kv_cache_append, src/models/moondream2.cpp:302-314). */
int mgpu_buf_copy_async(mgpu_buf* dst, size_t dst_offset, const mgpu_buf* src, size_t src_offset, size_t bytes);
void* mgpu_host_alloc(size_t bytes);
void mgpu_host_free(void* p);
void mgpu_release_buffer(mgpu_buf* buf);

/* upload_weight_image / upload_weight_buffer (src/models/moondream2.cpp:62-95): copy a GGUF
 * tensor's packed bytes to the device unchanged (Q4_0 18-byte / Q8_0 34-byte blocks stay
 * packed) and tag it NK with rows = dims[1], cols = dims[0]. */
mgpu_buf* mgpu_upload_weight(mgpu_device* dev, const mgpu_tensor_info* tensor, const void* host_data);

/* ---------------------------------------------------------------- dispatch -------- */
/* src/engine/compute.h:16-18 gemm_naive, :21-23 gemm_tiled, :26-28 gemm_image:
 * C[M,N] = A[M,K] * B[K,N].  All three run the same tcgen05 GEMM; A, B fp16 or bf16 (same
 * type), B layout KN or NK, C fp16 / bf16 / fp32, fp32 accumulation.  Returns the event. */
mgpu_event* mgpu_dispatch_gemm_naive(const mgpu_device* dev, mgpu_program program, mgpu_buf* A,
                                     mgpu_buf* B, mgpu_buf* C, int M, int N, int K);
mgpu_event* mgpu_dispatch_gemm_tiled(const mgpu_device* dev, mgpu_program program, mgpu_buf* A,
                                     mgpu_buf* B, mgpu_buf* C, int M, int N, int K);
mgpu_event* mgpu_dispatch_gemm_image(const mgpu_device* dev, mgpu_program program, mgpu_buf* A,
                                     mgpu_buf* B_img, mgpu_buf* C, int M, int N, int K);
/* src/engine/compute.h:31-33 gemv: y[1,N] = x[1,K] * W[K,N].  x fp16/bf16/fp32; W any type
 * (f32/f16/bf16 in KN or NK, Q4_0/Q8_0 in NK); y fp16/bf16/fp32; fp32 accumulation. */
mgpu_event* mgpu_dispatch_gemv(const mgpu_device* dev, mgpu_program program, mgpu_buf* x,
                               mgpu_buf* W_img, mgpu_buf* y, int N, int K);
/* src/engine/compute.h:101-105 patch_embed: image [C,H,W] (fp16) -> patches
 * [(H/ph)*(W/pw), embed_dim] = im2col(image) * proj_weight[C*ph*pw, embed_dim] + bias. */
mgpu_event* mgpu_dispatch_patch_embed(const mgpu_device* dev, mgpu_program program, mgpu_buf* image,
                                      mgpu_buf* proj_weight, mgpu_buf* proj_bias, mgpu_buf* patches,
                                      int C, int H, int W, int patch_h, int patch_w, int embed_dim);
/* src/engine/compute.h:128-131 vision_proj: output[num_patches, llm_dim] =
 * visual_tokens[num_patches, vision_dim] * proj_weight + proj_bias (bias may be NULL). */
mgpu_event* mgpu_dispatch_vision_proj(const mgpu_device* dev, mgpu_program program,
                                      mgpu_buf* visual_tokens, mgpu_buf* proj_weight,
                                      mgpu_buf* proj_bias, mgpu_buf* output, int num_patches,
                                      int vision_dim, int llm_dim);

/* No counterpart in the reference.  The same GEMV as mgpu_dispatch_gemv for a dense W stored
 * [K][N] (f32 / f16 / bf16, the reference kernels' orientation), for callers that cannot let
 * this library allocate device memory: engines that hand the whole GPU memory to their own
 * pool at start-up (a cudaMalloc here would fail or fragment it), and decode loops that must
 * not stall (mgpu_dispatch_gemv grows its scratch with cudaMalloc/cudaFree the first time it
 * sees a larger shape, and cudaFree waits for the whole device).  The split-K scratch of this
 * entry point is a fixed array of 1 MiB + 16 KiB that every GPU which loads this library holds
 * until the process exits; N is limited to 262144 (larger N is rejected with
 * MGPU_ERR_INVALID_ARG before anything is enqueued).  No cudaMalloc or cudaFree is called and
 * no event is recorded (the return value is the status).  The first call on a device looks
 * up the array's address on that device, which can load this library's device code there;
 * make that first call before any stream capture.  All calls share the one array, so calls
 * whose kernels overlap on the GPU (several streams, or several host threads on one device)
 * race: serialise them on one stream. */
int mgpu_dispatch_gemv_noalloc(const mgpu_device* dev, mgpu_buf* x, mgpu_buf* W_img, mgpu_buf* y, int N, int K);

/* New (no reference counterpart: the reference has no quantised kernels, README.md:57).
 * y[1,N] = x[1,K] * dequant(W)^T with W packed GGUF blocks [N][K/32] of `type`. */
mgpu_event* mgpu_gemv_q(const mgpu_device* dev, mgpu_buf* x, mgpu_buf* W, mgpu_buf* y, int N, int K,
                        int type);
/* dispatch_rms_norm (src/engine/compute.h:38-40, compute.cpp:156-184 launching
 * layernorm.cl:41-146): output[r] = input[r] * rsqrt(mean(input[r]^2) + eps) * weight for
 * num_rows rows of hidden_size values, fp32 arithmetic.  input / output fp16 (the reference's
 * types), bf16 or fp32, both of one type; weight fp16 / bf16 / fp32.  Returns the event. */
mgpu_event* mgpu_dispatch_rms_norm(const mgpu_device* dev, mgpu_program program, mgpu_buf* input, mgpu_buf* output,
                                   mgpu_buf* weight, int num_rows, int hidden_size, float eps);
/* New: the RMSNorm in front of a decode projection fused into the quantised GEMV:
 * y = x' * dequant(W)^T with x' = RMSNorm(x) computed as mgpu_dispatch_rms_norm does and rounded
 * to x's type, which is what the reference's rms_norm writes and its next dispatch_gemv reads
 * (moondream2.cpp:359-367, :455-463).  One launch, the norm in the GEMV's activation prologue,
 * for 1024 <= K <= 8192 with K a power of two; other shapes normalise into the device's scratch
 * and then run the GEMV (two launches; run those once before a graph capture). */
mgpu_event* mgpu_gemv_q_rmsnorm(const mgpu_device* dev, mgpu_buf* x, mgpu_buf* norm_weight, float eps, mgpu_buf* W,
                                mgpu_buf* y, int N, int K, int type);
/* New: the GEMVs of a decode step in one launch.  Replaces a run of dependent dispatch_gemv
 * calls (src/models/moondream2.cpp:357-542 calls one per projection, waiting on each) when
 * the weights are GGUF Q4_0 / Q8_0.  A link is one GEMV y[1,N] = x[1,K] * dequant(W)^T with the
 * argument meaning of mgpu_gemv_q.  Its x is either a buffer that is ready when the chain
 * runs, or the output of an earlier link: a view of that link's y (same type, K values inside
 * its N), the chain's dataflow.  The chain gives the same results as running the links one
 * after another with mgpu_gemv_q.  mgpu_gemv_chain_create checks the links once and keeps
 * pointers to the buffers, which must outlive the chain: all links share one quant type;
 * 1024 <= K <= 8192 with K a power of two and at most 192 links (MGPU_ERR_UNSUPPORTED
 * otherwise: split the chain, or run those GEMVs with mgpu_gemv_q); every x aligned to 4
 * elements; y ranges disjoint from each other, from every W and from every x that is not an
 * earlier y; W not written while the chain runs.  It allocates a small stage table and a
 * 64-byte counter per SM; mgpu_gemv_chain_run allocates nothing and can be captured in a
 * graph.  Runs of one chain must not overlap on the GPU (one stream).  A run that hits a
 * bounded-wait expiry reports MGPU_ERR_DEVICE_TIMEOUT and leaves the chain refusing to run:
 * destroy and re-create it. */
typedef struct mgpu_gemv_chain mgpu_gemv_chain;
typedef struct mgpu_gemv_link {
    mgpu_buf* x; /* [K] f32 / f16 / bf16, or a view of an earlier link's y */
    mgpu_buf* W; /* GGUF Q4_0 / Q8_0 blocks [N][K/32] */
    mgpu_buf* y; /* [N] f32 / f16 / bf16 */
    int N;
    int K;
} mgpu_gemv_link;
mgpu_gemv_chain* mgpu_gemv_chain_create(const mgpu_device* dev, const mgpu_gemv_link* links, int n_links);
mgpu_event* mgpu_gemv_chain_run(mgpu_gemv_chain* chain);
/* One run with per-link timing (synchronous): end_us[i] = microseconds from the run's start
 * to the moment the last CTA finished link i (device %globaltimer, max over CTAs). */
int mgpu_gemv_chain_run_timed(mgpu_gemv_chain* chain, double* end_us);
int mgpu_gemv_chain_links(const mgpu_gemv_chain* chain);
void mgpu_gemv_chain_destroy(mgpu_gemv_chain* chain);
/* C[M,N] = A[M,K] * dequant(W)^T (+ bias[N] if non-NULL), W packed [N][K/32] blocks, A
 * fp16/bf16; the blocks are dequantised to A's type inside the GEMM's weight loads. */
mgpu_event* mgpu_gemm_q(const mgpu_device* dev, mgpu_buf* A, mgpu_buf* W, mgpu_buf* C, int M, int N,
                        int K, int type, mgpu_buf* bias);
/* General entry: C = A * op(B) + bias, every operand's type/layout taken from its tag. */
mgpu_event* mgpu_gemm(const mgpu_device* dev, mgpu_buf* A, mgpu_buf* B, mgpu_buf* C, int M, int N,
                      int K, mgpu_buf* bias);
/* Activation applied by mgpu_gemm_fused after the bias.
 * GELU: the tanh approximation 0.5x(1 + tanh(sqrt(2/pi)(x + 0.044715x^3))) that
 *   dispatch_gelu's declaration states (src/engine/compute.h:48-50).
 * SILU: x / (1 + exp(-x)), the reference's silu kernel (src/kernels/activations.cl:30-65).
 * GELU_AS_SHIPPED: what the reference's gelu kernel computes (activations.cl:78-117):
 *   0.5x(1 - tanh(...)), because its tanh identity has the sign reversed; use it only to
 *   reproduce that kernel's output. */
enum mgpu_act {
    MGPU_ACT_NONE = 0,
    MGPU_ACT_GELU = 1,
    MGPU_ACT_SILU = 2,
    MGPU_ACT_GELU_AS_SHIPPED = 3
};
/* C = act(A * op(B) + bias) + residual, in the GEMM's epilogue (one pass over C).  Replaces
 * dispatch_gemm_image (src/engine/compute.h:27-29) followed by dispatch_gelu / dispatch_silu
 * (compute.h:44-50) and the residual add (dispatch_residual_add, src/models/moondream2.cpp:297-300,
 * over dispatch_vector_add, compute.h:134) on its output, as moondream2_forward chains them
 * (moondream2.cpp:454, :497-512).  bias [N] and
 * residual [M][N] (its own type and row pitch, default N) may be NULL; residual may be C
 * itself (in-place `hidden += ...`).  The sum and the activation are computed in fp32 and C
 * is rounded once, where the reference rounds to fp16 after each kernel. */
mgpu_event* mgpu_gemm_fused(const mgpu_device* dev, mgpu_buf* A, mgpu_buf* B, mgpu_buf* C, int M, int N,
                            int K, mgpu_buf* bias, int act, mgpu_buf* residual);
/* out = silu(A * op(W_gate)) * up, elementwise, in the gate GEMM's epilogue.  Replaces the
 * gate projection's dispatch_gemm_image followed by dispatch_silu_gate_multiply
 * (src/engine/compute.h:57-60, activations.cl:219-265), as moondream2_forward chains them
 * (src/models/moondream2.cpp:465-495): the gate activations are never stored.  up is [M][N]
 * (f32 / f16 / bf16, own row pitch, default N), the up projection's output; out may be up
 * itself. */
mgpu_event* mgpu_gemm_silu_gate(const mgpu_device* dev, mgpu_buf* A, mgpu_buf* W_gate, mgpu_buf* up,
                                mgpu_buf* out, int M, int N, int K);
/* out[n] = dequant(W)[n] for n elements (out fp32, fp16 or bf16 per its tag). */
mgpu_event* mgpu_dequant(const mgpu_device* dev, mgpu_buf* W, mgpu_buf* out, int64_t n, int type);

/* Replaces argmax_logits (src/models/moondream2.cpp:551-591), which reads the fp16 logits back
 * and scans them on the host.  Same result: the first index whose value is greater than every
 * earlier one, starting from (-1e30, index 0), with values read as there (exponent field zero
 * -> 0, all ones (Inf/NaN) -> +-1e30 by sign; bf16 / fp32 logits by the same rule on their own
 * fields).  Computed on the device by one CTA; `out` (>= 8 bytes) receives the int32 index and
 * the fp32 value, so shards of column-sharded logits combine by (larger value, smaller index). */
mgpu_event* mgpu_argmax(const mgpu_device* dev, mgpu_buf* logits, int n, mgpu_buf* out);
/* New: mgpu_argmax for a batch of `rows` rows of n logits, row r starting at element r * ld
 * (ld >= n), e.g. each sequence of a batched decode against one lm_head column shard.  `out`
 * (>= 8 * rows bytes) receives the rows' {int32 index, fp32 value} pairs in row order.  One CTA
 * per row, one launch. */
mgpu_event* mgpu_argmax_rows(const mgpu_device* dev, mgpu_buf* logits, int rows, int n, int64_t ld, mgpu_buf* out);
/* argmax_logits itself: waits for the stream and returns the index, or -1 on error. */
int mgpu_argmax_logits(const mgpu_device* dev, mgpu_buf* logits, int vocab_size);
/* New (the reference decodes on one device): the greedy token of logits column-sharded over
 * n_ranks GPUs, from the ranks' mgpu_argmax results gathered in rank order (`pairs`: n_ranks x
 * {int32 index within the shard, fp32 value}; rank r owns columns [r*(n/R) + min(r, n%R), ..)
 * of the n_total, the first n % R ranks one more).  `out` (>= 8 bytes) receives the global
 * index and its value: the larger value wins and equal values go to the lower rank, so the
 * result is argmax_logits' first maximum over the whole row.  One thread, one launch. */
mgpu_event* mgpu_argmax_combine(const mgpu_device* dev, mgpu_buf* pairs, int n_ranks, int n_total, mgpu_buf* out);

/* ---------------------------------------------------------------- peer groups ----- */
/* New (the reference runs on one device): small exchanges between the GPUs of one node over
 * NVLink, without a collective library, for the column-sharded lm_head of a batched decode
 * (each GPU's hidden state to every GPU; each sequence's argmax pair to the GPU that owns it).
 * A group holds, on each GPU, world receive slots of slot_bytes plus one flag per GPU, in one
 * allocation that the other GPUs map through CUDA IPC.  Every GPU of a group must run the same
 * exchanges in the same order; an exchange is one kernel on the device's stream that stores
 * into the peers' slots, publishes its flags and waits (bounded, default 2 s; on expiry the
 * device status reports MGPU_ERR_DEVICE_TIMEOUT) for the peers' flags.  Exchanges can be
 * captured into graphs.  Set-up, once per group:
 *   g = mgpu_peer_group_create(dev, rank, world, slot_bytes);
 *   mgpu_peer_group_handle(g, mine);                  64 bytes, to send to every rank
 *   mgpu_peer_group_connect(g, all);                  world x 64 bytes in rank order
 * (or mgpu_peer_group_connect_ptrs with the peers' slot addresses when the groups live in one
 * process).  The slots of this GPU are mgpu_peer_group_slots(g) (world x slot_bytes; slot r
 * holds rank r's bytes); they stay valid until the next exchange on the group. */
typedef struct mgpu_peer_group mgpu_peer_group;
mgpu_peer_group* mgpu_peer_group_create(mgpu_device* dev, int rank, int world, size_t slot_bytes);
int mgpu_peer_group_handle(const mgpu_peer_group* g, void* out64);
int mgpu_peer_group_connect(mgpu_peer_group* g, const void* handles);
int mgpu_peer_group_connect_ptrs(mgpu_peer_group* g, void* const* peer_slots);
void* mgpu_peer_group_local_ptr(const mgpu_peer_group* g);
mgpu_buf* mgpu_peer_group_slots(mgpu_peer_group* g);
int mgpu_peer_group_set_wait_limit(mgpu_peer_group* g, uint64_t limit_ns);
/* src (bytes, a multiple of 8, <= slot_bytes; src 16-byte aligned) into slot `rank` of every
 * GPU.  slot_bytes is rounded up to a multiple of 8 at creation. */
mgpu_event* mgpu_peer_allgather(mgpu_peer_group* g, const mgpu_buf* src, size_t bytes);
/* bytes [p * bytes_per_peer, (p + 1) * bytes_per_peer) of src into slot `rank` of GPU p. */
mgpu_event* mgpu_peer_alltoall(mgpu_peer_group* g, const mgpu_buf* src, size_t bytes_per_peer);
void mgpu_peer_group_destroy(mgpu_peer_group* g);

/* ---------------------------------------------------------------- events ---------- */
int mgpu_wait_event(mgpu_event* ev);                 /* clWaitForEvents(1, &ev) */
void mgpu_release_event(mgpu_event* ev);             /* clReleaseEvent */
double mgpu_profile_end(mgpu_event* ev);             /* profile_end (src/engine/profiler.h:16): ms */
float mgpu_event_elapsed_ms(mgpu_event* start, mgpu_event* end);
/* Record a marker event on the device stream now (also inside a graph capture, where it
 * becomes a node of the graph); mgpu_event_elapsed_ms(a, b) gives the device time between
 * two markers.  Release with mgpu_release_event. */
mgpu_event* mgpu_record_event(mgpu_device* dev);

/* ---------------------------------------------------------------- graphs ---------- */
/* CUDA-graph capture of a dispatch sequence on the device's stream (no reference
 * counterpart: the reference planned Qualcomm recordable queues, README.md:121-129, and
 * waits on the host after every op).  Between begin and end, dispatches are recorded, not
 * run; they must not grow the device's scratch (run each one once before capturing).
 * Dispatches return NULL while capturing. */
int mgpu_capture_begin(mgpu_device* dev);
typedef struct mgpu_graph mgpu_graph;
mgpu_graph* mgpu_capture_end(mgpu_device* dev);
int mgpu_graph_launch(mgpu_graph* graph);
void mgpu_graph_release(mgpu_graph* graph);

/* Failure-detection self test: launches one CTA that waits on an mbarrier nobody arrives
 * on, with a wait limit of `limit_ns`.  The wait expires, the kernel records
 * MGPU_ERR_DEVICE_TIMEOUT in the device status word and exits; the next mgpu_finish then
 * reports MGPU_ERR_DEVICE_TIMEOUT.  Returns the launch status. */
int mgpu_selftest_bounded_wait(mgpu_device* dev, uint64_t limit_ns);

/* ---------------------------------------------------------------- ggml table ------ */
size_t mgpu_ggml_type_size(int type);       /* ggml_type_size (gguf_loader.h:79) */
int mgpu_ggml_type_block_size(int type);    /* ggml_type_block_size (gguf_loader.h:82) */

/* ---------------------------------------------------------------- synthetic data --- */
/* Device-side seeded generators used by the benchmark (no reference counterpart): the
 * SplitMix64 stream of element i is seeded with seed + i, so results do not depend on the
 * launch shape. */
int mgpu_fill_uniform(const mgpu_device* dev, mgpu_buf* out, int64_t n, uint64_t seed, float lo,
                      float hi);
int mgpu_fill_normal(const mgpu_device* dev, mgpu_buf* out, int64_t n, uint64_t seed, float sigma);
/* fp32 -> GGUF Q4_0 / Q8_0 blocks on the device (ggml reference quantiser). */
int mgpu_quantize(const mgpu_device* dev, mgpu_buf* src_f32, mgpu_buf* dst_blocks, int64_t n, int type);
/* Element-type conversion of n values between two buffers (f32/f16/bf16). */
int mgpu_convert(const mgpu_device* dev, mgpu_buf* src, mgpu_buf* dst, int64_t n);

#ifdef __cplusplus
}
#endif
#endif /* MGPU_CUDA_H */
