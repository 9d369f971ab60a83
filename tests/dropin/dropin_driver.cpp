// dropin_driver.cpp - runs the reference's own moondream2_forward on the B200 path (test harness).
//
// Built by oracle/Makefile (when the MVLM checkout is present) together with:
//   - the reference's headers moondream2.h / device.h / memory.h / compute.h, unmodified, with
//     include/cl_compat in place of the OpenCL SDK;
//   - moondream2_forward.inc: the reference's src/models/moondream2.cpp from "Buffer Allocation"
//     to the end of moondream2_forward (moondream2_alloc_buffers, dispatch_residual_add,
//     kv_cache_append, moondream2_forward), extracted at build time, unmodified;
//   - mvlm_b200/engine/engine_cuda.cpp, the engine API of the matmul path on libmgpu.
// The compute.h operations that are not on the matmul path get stand-ins here, through host
// copies: the embedding row copy, RoPE at position 0 (the first decode step, where the rotation
// angle is 0: the identity), single-query softmax attention over the cache, and the residual add
// and SiLU-gated product as the reference's kernels compute them (activations.cl:219-299).
#include <cmath>
#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <ctime>
#include <vector>

#include "../../include/mgpu_cuda.h"
#include "compute.h"
#include "moondream2.h"

namespace {

mgpu_buf* B(cl_mem m) { return reinterpret_cast<mgpu_buf*>(m); }

// set when moondream2_forward asks a stand-in for something it does not cover
int g_uncovered = 0;

float half_to_float(uint16_t h) {
    const uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
    const uint32_t e = (h >> 10) & 0x1Fu, m = h & 0x3FFu;
    uint32_t bits;
    if (e == 0) {
        if (m == 0) {
            bits = sign;
        } else {  // subnormal: normalise
            int sh = 0;
            uint32_t mm = m;
            while (!(mm & 0x400u)) {
                mm <<= 1;
                ++sh;
            }
            bits = sign | ((uint32_t)(113 - sh) << 23) | ((mm & 0x3FFu) << 13);
        }
    } else if (e == 31) {
        bits = sign | 0x7F800000u | (m << 13);
    } else {
        bits = sign | ((e + 112) << 23) | (m << 13);
    }
    float f;
    memcpy(&f, &bits, 4);
    return f;
}

// fp32 -> fp16, round to nearest even (what vstore_half and (half) casts do)
uint16_t float_to_half(float f) {
    uint32_t x;
    memcpy(&x, &f, 4);
    const uint32_t sign = (x >> 16) & 0x8000u;
    const uint32_t ax = x & 0x7FFFFFFFu;
    if (ax >= 0x7F800000u) return (uint16_t)(sign | 0x7C00u | (ax > 0x7F800000u ? 0x200u : 0u));
    if (ax >= 0x477FF000u) return (uint16_t)(sign | 0x7C00u);  // rounds to infinity
    if (ax < 0x38800000u) {                                    // fp16 subnormal or zero
        if (ax < 0x33000000u) return (uint16_t)sign;
        const uint32_t e = ax >> 23, m = (ax & 0x7FFFFFu) | 0x800000u;
        const uint32_t shift = 126 - e;  // to 10 fraction bits of a subnormal
        uint32_t r = m >> shift;
        const uint32_t rem = m & ((1u << shift) - 1), half = 1u << (shift - 1);
        if (rem > half || (rem == half && (r & 1u))) ++r;
        return (uint16_t)(sign | r);
    }
    uint32_t r = ((ax >> 13) - (112u << 10));
    const uint32_t rem = ax & 0x1FFFu;
    if (rem > 0x1000u || (rem == 0x1000u && (r & 1u))) ++r;
    return (uint16_t)(sign | r);
}

std::vector<uint16_t> read_half(cl_mem m, size_t n) {
    std::vector<uint16_t> v(n);
    mgpu_buf_read(B(m), 0, v.data(), n * 2);
    return v;
}

}  // namespace

namespace mgpu {

// ---- compute.h operations off the matmul path ----
cl_event dispatch_embedding_lookup(const DeviceInfo*, cl_program, cl_mem embed_table, cl_mem token_ids, cl_mem output,
                                   int seq_len, int embed_dim) {
    std::vector<int> ids(seq_len);
    mgpu_buf_read(B(token_ids), 0, ids.data(), ids.size() * sizeof(int));
    const size_t row = (size_t)embed_dim * 2;
    for (int i = 0; i < seq_len; ++i) mgpu_buf_copy_async(B(output), i * row, B(embed_table), ids[i] * row, row);
    return nullptr;
}

cl_event dispatch_rope_apply(const DeviceInfo*, cl_program, cl_mem, cl_mem, cl_mem, int seq_len, int, int,
                             int offset) {
    if (offset != 0 || seq_len != 1) {
        fprintf(stderr, "dropin: RoPE stand-in covers position 0 only\n");
        g_uncovered = 1;
    }
    return nullptr;  // rotation by angle 0
}

// One query against the cache: per head softmax(q . k_j / sqrt(head_dim)) over the cache_len
// positions, then the weighted sum of v_j; fp32 arithmetic, fp16 store.  (moondream2_forward
// appends every layer's K and V to the one cache, so layer l of the first token sees l positions.)
cl_event dispatch_attention_decode(const DeviceInfo* dev, cl_program, cl_mem Q, cl_mem K_cache, cl_mem V_cache,
                                   cl_mem output, int cache_len, int num_heads, int head_dim) {
    mgpu_finish(reinterpret_cast<mgpu_device*>(dev->context));
    const size_t row = (size_t)num_heads * head_dim;
    std::vector<uint16_t> q = read_half(Q, row), k = read_half(K_cache, row * cache_len),
                          v = read_half(V_cache, row * cache_len), out(row);
    const float scale = 1.0f / sqrtf((float)head_dim);
    std::vector<float> p(cache_len);
    for (int h = 0; h < num_heads; ++h) {
        float mx = -INFINITY;
        for (int j = 0; j < cache_len; ++j) {
            float dot = 0.0f;
            for (int d = 0; d < head_dim; ++d)
                dot += half_to_float(q[h * head_dim + d]) * half_to_float(k[j * row + h * head_dim + d]);
            p[j] = dot * scale;
            mx = fmaxf(mx, p[j]);
        }
        float sum = 0.0f;
        for (int j = 0; j < cache_len; ++j) sum += (p[j] = expf(p[j] - mx));
        for (int d = 0; d < head_dim; ++d) {
            float acc = 0.0f;
            for (int j = 0; j < cache_len; ++j) acc += p[j] / sum * half_to_float(v[j * row + h * head_dim + d]);
            out[h * head_dim + d] = float_to_half(acc);
        }
    }
    mgpu_buf_write(B(output), 0, out.data(), row * 2);
    return nullptr;
}

cl_event dispatch_attention_prefill(const DeviceInfo*, cl_program, cl_mem, cl_mem, cl_mem, cl_mem, int, int, int) {
    fprintf(stderr, "dropin: no prefill attention stand-in\n");
    g_uncovered = 1;
    return nullptr;
}

// vector_add (activations.cl:271-299): fp32 sum of two fp16 vectors, stored fp16
cl_event dispatch_vector_add(const DeviceInfo* dev, cl_program, cl_mem a, cl_mem b, cl_mem output, int n) {
    mgpu_finish(reinterpret_cast<mgpu_device*>(dev->context));
    std::vector<uint16_t> va = read_half(a, n), vb = read_half(b, n), out(n);
    for (int i = 0; i < n; ++i) out[i] = float_to_half(half_to_float(va[i]) + half_to_float(vb[i]));
    mgpu_buf_write(B(output), 0, out.data(), (size_t)n * 2);
    return nullptr;
}

// silu_gate_multiply (activations.cl:219-265): gate * (1 / (1 + exp(-gate))) * up, stored fp16
cl_event dispatch_silu_gate_multiply(const DeviceInfo* dev, cl_program, cl_mem gate, cl_mem up, cl_mem output, int n) {
    mgpu_finish(reinterpret_cast<mgpu_device*>(dev->context));
    std::vector<uint16_t> g = read_half(gate, n), u = read_half(up, n), out(n);
    for (int i = 0; i < n; ++i) {
        const float gf = half_to_float(g[i]);
        out[i] = float_to_half(gf * (1.0f / (1.0f + expf(-gf))) * half_to_float(u[i]));
    }
    mgpu_buf_write(B(output), 0, out.data(), (size_t)n * 2);
    return nullptr;
}

// The reference's code, compiled as it is (see the file comment).
#include "moondream2_forward.inc"

}  // namespace mgpu

namespace {

cl_mem upload(const mgpu::DeviceInfo* dev, const void* data, size_t bytes) {
    return mgpu::create_buffer(dev, bytes, CL_MEM_READ_ONLY | CL_MEM_COPY_HOST_PTR, const_cast<void*>(data));
}

cl_mem upload_q(const mgpu::DeviceInfo* dev, const uint8_t* data, int qtype, int N, int K) {
    const size_t bytes = (size_t)N * (K / 32) * (qtype == MGPU_Q4_0 ? 18 : 34);
    cl_mem m = upload(dev, data, bytes);
    if (m) mgpu_buf_set_format(B(m), qtype, MGPU_LAYOUT_NK, N, K, 0);
    return m;
}

}  // namespace

// One decode token through moondream2_forward with the given weights.  proj: per layer q, k, v,
// o, gate, up, down ([N][K/32] blocks of qtype; q/k/v/o dim x dim, gate/up intermediate x dim,
// down dim x intermediate); norms: per layer input and post norm weights (fp16 [dim]); embed:
// fp16 [vocab][dim]; lm_head: [vocab][dim/32] blocks.  logits_out: vocab fp16.  Returns 0 on
// success.
extern "C" int dropin_forward_decode(int dim, int intermediate, int layers, int vocab, int heads, int qtype,
                                     const uint8_t* const* proj, const uint16_t* const* norms, const uint16_t* embed,
                                     const uint16_t* final_norm, const uint8_t* lm_head, int token,
                                     uint16_t* logits_out) {
    using namespace mgpu;
    DeviceInfo dev;
    if (!init_device(&dev)) return 1;
    Moondream2Model model{};
    Moondream2Config& cfg = model.config;
    cfg.llm_dim = dim;
    cfg.llm_intermediate = intermediate;
    cfg.llm_layers = layers;
    cfg.vocab_size = vocab;
    cfg.llm_heads = heads;
    cfg.head_dim = dim / heads;
    cfg.max_seq_len = 8;
    if (!moondream2_alloc_buffers(&model, &dev)) return 2;
    model.gemm_program = model.norm_program = model.activation_program = build_program_from_source(&dev, "", 0, "");
    model.rope_program = model.embedding_program = model.attention_program = model.gemm_program;
    Moondream2Weights& w = model.gpu_weights;
    w.num_layers = layers;
    w.layers = new TransformerLayerWeights[layers];
    for (int l = 0; l < layers; ++l) {
        TransformerLayerWeights& lw = w.layers[l];
        const uint8_t* const* p = proj + 7 * l;
        lw.q_proj_weight = upload_q(&dev, p[0], qtype, dim, dim);
        lw.k_proj_weight = upload_q(&dev, p[1], qtype, dim, dim);
        lw.v_proj_weight = upload_q(&dev, p[2], qtype, dim, dim);
        lw.o_proj_weight = upload_q(&dev, p[3], qtype, dim, dim);
        lw.gate_proj_weight = upload_q(&dev, p[4], qtype, intermediate, dim);
        lw.up_proj_weight = upload_q(&dev, p[5], qtype, intermediate, dim);
        lw.down_proj_weight = upload_q(&dev, p[6], qtype, dim, intermediate);
        lw.input_norm_weight = upload(&dev, norms[2 * l], (size_t)dim * 2);
        lw.post_norm_weight = upload(&dev, norms[2 * l + 1], (size_t)dim * 2);
    }
    w.token_embed = upload(&dev, embed, (size_t)vocab * dim * 2);
    w.final_norm_weight = upload(&dev, final_norm, (size_t)dim * 2);
    w.lm_head_weight = upload_q(&dev, lm_head, qtype, vocab, dim);
    model.initialized = true;

    cl_mem logits = moondream2_forward(&model, &dev, &token, 1);
    int rc = !logits ? 3 : mgpu_buf_read(B(logits), 0, logits_out, (size_t)vocab * 2) == MGPU_OK ? 0 : 4;
    if (g_uncovered) rc = 5;
    std::vector<cl_mem> all = {logits, w.token_embed, w.final_norm_weight, w.lm_head_weight, model.kv_cache.k_cache,
                               model.kv_cache.v_cache, model.scratch_a, model.scratch_b, model.scratch_q,
                               model.scratch_k, model.scratch_v, model.scratch_attn, model.scratch_gate,
                               model.scratch_up};
    for (int l = 0; l < layers; ++l) {
        const TransformerLayerWeights& lw = w.layers[l];
        for (cl_mem m : {lw.q_proj_weight, lw.k_proj_weight, lw.v_proj_weight, lw.o_proj_weight, lw.gate_proj_weight,
                         lw.up_proj_weight, lw.down_proj_weight, lw.input_norm_weight, lw.post_norm_weight})
            all.push_back(m);
    }
    for (cl_mem m : all)
        if (m) clReleaseMemObject(m);
    delete[] w.layers;
    destroy_device(&dev);
    return rc;
}
