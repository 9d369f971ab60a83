"""The engine drop-in, end to end: the reference's own moondream2_forward (src/models/
moondream2.cpp, extracted unmodified at build time with moondream2_alloc_buffers,
dispatch_residual_add and kv_cache_append) compiled with the reference's headers against
include/cl_compat, linked to libmgpu through mvlm_b200/engine/engine_cuda.cpp, runs one decode
token of a small Phi-style model on the GPU: embedding, per layer RMSNorm -> q/k/v GEMVs ->
attention -> o GEMV -> residual -> RMSNorm -> gate/up GEMVs -> SiLU-gated product -> down GEMV
-> residual, final RMSNorm, lm_head GEMV.  The GEMVs and norms are this library's kernels
(Q4_0 / Q8_0 weights); the ops off the matmul path are the harness's stand-ins
(tests/dropin/dropin_driver.cpp).  The logits are compared with the oracle applying the same
chain with the reference's fp16 stores in between."""
import ctypes
import os

import numpy as np
import pytest

import mvlm_b200 as mg
import oracle as O
from tests.numerics import TOL_16, assert_close

pytestmark = pytest.mark.gpu

LIB = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "oracle", "_ref",
                   "libref_dropin.so")


def _oracle_forward(qt, dim, inter, layers, heads, proj, norms, embed, final_norm, lm_head, token, eps=1e-5):
    f16 = lambda a: O.f16_to_f32(O.f16(a))  # noqa: E731  (a store in fp16)
    gemv = lambda x, W, N, K: f16(O.gemm_q(np.ascontiguousarray(x, np.float32), W, 1, N, K, qt))  # noqa: E731
    h = O.f16_to_f32(embed.reshape(-1, dim)[token])
    kc, vc = [], []  # the one cache every layer appends to, as moondream2_forward does
    hd = dim // heads
    for l in range(layers):
        q, k, v, o, g, u, d = proj[7 * l: 7 * l + 7]
        xn = O.rms_norm(h, O.f16_to_f32(norms[2 * l]), 1, dim, eps, O.F16)
        qq, kk, vv = gemv(xn, q, dim, dim), gemv(xn, k, dim, dim), gemv(xn, v, dim, dim)
        kc.append(kk.reshape(heads, hd))
        vc.append(vv.reshape(heads, hd))
        K, V = np.stack(kc, 1), np.stack(vc, 1)  # [heads][positions][hd]
        s = np.einsum("hd,hjd->hj", qq.reshape(heads, hd), K) / np.float32(np.sqrt(hd))
        p = np.exp(s - s.max(axis=1, keepdims=True))
        attn = f16(np.einsum("hj,hjd->hd", p / p.sum(axis=1, keepdims=True), V).reshape(-1))
        h = f16(h + gemv(attn, o, dim, dim))  # residual add (vector_add), fp16 store
        xn = O.rms_norm(h, O.f16_to_f32(norms[2 * l + 1]), 1, dim, eps, O.F16)
        gate, up = gemv(xn, g, inter, dim), gemv(xn, u, inter, dim)
        m = O.unfused_silu_gate(gate, up, O.F16)
        h = f16(h + gemv(m, d, dim, inter))
    xn = O.rms_norm(h, O.f16_to_f32(final_norm), 1, dim, eps, O.F16)
    return gemv(xn, lm_head, embed.size // dim, dim)


@pytest.mark.parametrize("qt", [O.Q4_0, O.Q8_0])
def test_reference_forward_runs_on_the_b200_path(qt):
    if not os.path.exists(LIB):
        pytest.skip("oracle/_ref/libref_dropin.so was not built (needs the reference checkout at build time)")
    L = ctypes.CDLL(LIB)
    fn = L.dropin_forward_decode
    fn.restype = ctypes.c_int
    dim, inter, layers, vocab, heads, token = 1024, 2048, 2, 2000, 16, 7
    rng_seed = 0x4D564C4D + qt
    shapes = [(dim, dim)] * 4 + [(inter, dim), (inter, dim), (dim, inter)]  # (N, K)
    proj = [O.quantize(O.normal(N * K, rng_seed + 10 * l + i, 0.03), qt)
            for l in range(layers) for i, (N, K) in enumerate(shapes)]
    norms = [O.f16(1.0 + O.normal(dim, rng_seed + 100 + i, 0.1)) for i in range(2 * layers)]
    embed = O.f16(O.normal(vocab * dim, rng_seed + 200, 1.0))
    final_norm = O.f16(1.0 + O.normal(dim, rng_seed + 300, 0.1))
    lm_head = O.quantize(O.normal(vocab * dim, rng_seed + 400, 0.03), qt)
    P = (ctypes.c_void_p * len(proj))(*[p.ctypes.data for p in proj])
    Nn = (ctypes.c_void_p * len(norms))(*[n.ctypes.data for n in norms])
    out = np.zeros(vocab, np.uint16)
    rc = fn(dim, inter, layers, vocab, heads, qt, P, Nn, ctypes.c_void_p(embed.ctypes.data),
            ctypes.c_void_p(final_norm.ctypes.data), ctypes.c_void_p(lm_head.ctypes.data), token,
            ctypes.c_void_p(out.ctypes.data))
    assert rc == 0, rc
    ref = _oracle_forward(qt, dim, inter, layers, heads, proj, norms, embed, final_norm, lm_head, token)
    assert_close(O.f16_to_f32(out), ref, TOL_16, f"moondream2_forward q{qt}")
    assert int(np.argmax(O.f16_to_f32(out))) == int(np.argmax(ref))
