"""GPU parity of the tcgen05 GEMM (replaces gemm_naive / gemm_tiled / gemm_image,
src/kernels/gemm.cl:26-200, and the GEMM math of patch_embed / vision_proj,
src/kernels/vision.cl:118-197, :402-441) against the CPU oracle, through the C ABI."""
import numpy as np
import pytest

import mvlm_b200 as mg
import oracle as O
from tests.numerics import TOL_16, TOL_F32, assert_close

pytestmark = pytest.mark.gpu

DISPATCH = [mg.dispatch_gemm_naive, mg.dispatch_gemm_tiled, mg.dispatch_gemm_image]


def _f16_pair(M, N, K, seed, sa=1.0, sb=1.0):
    A = O.f16(O.uniform(M * K, seed) * np.float32(sa))
    B = O.f16(O.uniform(K * N, seed + 1) * np.float32(sb))
    return A, B


@pytest.mark.parametrize("M,N,K", [(1, 1, 1), (3, 5, 7), (17, 33, 45), (128, 256, 64), (129, 72, 40),
                                   (200, 300, 100), (255, 129, 257), (761, 2048, 2048)])
@pytest.mark.parametrize("fn", DISPATCH, ids=["naive", "tiled", "image"])
def test_dispatch_gemm_reference_semantics(dev, fn, M, N, K):
    # fp16 A[M,K], fp16 B[K,N], fp16 C: the reference kernels' types and B orientation
    A, B = _f16_pair(M, N, K, 100 + M + N + K)
    ref = O.gemm_naive_f32(O.f16_to_f32(A), O.f16_to_f32(B), M, N, K, threads=True)
    dA = dev.array(A, mg.F16)
    dB = dev.create_weight_image(K, N, B) if fn is mg.dispatch_gemm_image else dev.array(B, mg.F16)
    dC = dev.empty(M * N, mg.F16)
    fn(dev, None, dA, dB, dC, M, N, K).wait()
    C = O.f16_to_f32(dC.read(np.uint16))
    assert_close(C, ref, TOL_16, f"{fn.__name__} {M}x{N}x{K}")
    if M * N * K <= 200 * 300 * 100:
        # the oracle's fp16 output is bit-identical to the reference gemm.cl (tests/test_oracle.py)
        assert_close(C, O.f16_to_f32(O.gemm_naive_f16(A, B, M, N, K)), TOL_16)


@pytest.mark.parametrize("qt", [O.Q8_0, O.Q4_0])
@pytest.mark.parametrize("K,N", [(2048, 6144), (2048, 2048), (2048, 8192), (8192, 2048)])
def test_prefill_quantised_phi(dev, qt, K, N):
    # Phi-1.5 prefill: M=761, bf16 activations ~N(0,1), weights ~N(0,0.02) in GGUF blocks
    M = 761
    A = O.bf16(O.normal(M * K, 0x4D564C4D + K, 1.0))
    W = O.quantize(O.normal(N * K, 0x4D564C4E + N, 0.02), qt)
    ref = O.gemm_q(O.bf16_to_f32(A), W, M, N, K, qt, threads=True)
    dC = dev.empty(M * N, mg.F32)
    mg.gemm_q(dev, dev.array(A, mg.BF16), dev.array(W, qt, mg.LAYOUT_NK), dC, M, N, K, qt).wait()
    assert_close(dC.read(np.float32), ref, TOL_16, f"prefill q{qt} {K}x{N}")


@pytest.mark.parametrize("qt", [O.Q8_0, O.Q4_0])
@pytest.mark.parametrize("M,N,K", [(8, 2048, 2048), (32, 6144, 2048), (128, 2048, 8192), (5, 100, 96),
                                   (130, 300, 160), (600, 5000, 512)])
def test_quantised_ragged_and_batched(dev, qt, M, N, K):
    A = O.bf16(O.normal(M * K, M + N, 1.0))
    W = O.quantize(O.normal(N * K, K, 0.02), qt)
    ref = O.gemm_q(O.bf16_to_f32(A), W, M, N, K, qt, threads=True)
    for ct in (mg.F32, mg.BF16):
        dC = dev.empty(M * N, ct)
        mg.gemm_q(dev, dev.array(A, mg.BF16), dev.array(W, qt, mg.LAYOUT_NK), dC, M, N, K, qt).wait()
        C = dC.read(mg.NP_DTYPE[ct])
        C = O.bf16_to_f32(C) if ct == mg.BF16 else C
        assert_close(C, ref, TOL_16, f"q{qt} {M}x{N}x{K} c{ct}")


@pytest.mark.parametrize("qt,M,N,K", [(O.Q4_0, 128, 2040, 8192), (O.Q8_0, 128, 6144, 2048),
                                      (O.Q8_0, 761, 2048, 2048), (O.Q4_0, 300, 1000, 8192)])
def test_cluster_split_k(dev, qt, M, N, K):
    # Shapes whose tiles leave SMs idle run as clusters that split K and sum the fp32 partials
    # over distributed shared memory (one CTA or CTA pair per K slice).  Bias, ragged N and
    # both output types; the sum is in slice order, so two calls give identical bits.
    A = O.bf16(O.normal(M * K, 3 * M + N, 1.0))
    W = O.quantize(O.normal(N * K, K + 1, 0.02), qt)
    bias = O.normal(N, 99, 0.5)
    ref = O.gemm_q(O.bf16_to_f32(A), W, M, N, K, qt, threads=True).reshape(M, N) + bias
    dA, dW, dB = dev.array(A, mg.BF16), dev.array(W, qt, mg.LAYOUT_NK), dev.array(bias, mg.F32)
    for ct in (mg.F32, mg.BF16):
        outs = []
        for _ in range(2):
            dC = dev.empty(M * N, ct)
            mg.gemm_q(dev, dA, dW, dC, M, N, K, qt, dB).wait()
            outs.append(dC.read(mg.NP_DTYPE[ct]))
        assert np.array_equal(outs[0], outs[1]), f"split-K sums not deterministic q{qt} {M}x{N}x{K}"
        C = O.bf16_to_f32(outs[0]) if ct == mg.BF16 else outs[0]
        assert_close(C, ref.reshape(-1), TOL_16, f"split-K q{qt} {M}x{N}x{K} c{ct}")


@pytest.mark.parametrize("K,N", [(1152, 3456), (1152, 1152), (1152, 4304), (4304, 1152)])
def test_siglip_layer_fp16(dev, K, N):
    # SigLIP per-layer GEMMs at B=1 (M=729): fp16 activations ~N(0,1), fp16 weights ~N(0,0.02)
    M = 729
    A = O.f16(O.normal(M * K, 7 + K, 1.0))
    B = O.f16(O.normal(K * N, 8 + N, 0.02))
    ref = O.gemm_naive_f32(O.f16_to_f32(A), O.f16_to_f32(B), M, N, K, threads=True)
    dC = dev.empty(M * N, mg.F16)
    mg.dispatch_gemm_image(dev, None, dev.array(A, mg.F16), dev.create_weight_image(K, N, B), dC, M, N, K).wait()
    assert_close(O.f16_to_f32(dC.read(np.uint16)), ref, TOL_16, f"siglip {K}x{N}")


@pytest.mark.parametrize("wt", [mg.F16, mg.BF16])
def test_gguf_native_nk_weights(dev, wt):
    # GGUF F16 tensors are W[N][K]; the GEMM reads them K-major without a transpose copy
    M, N, K = 300, 1000, 576
    conv, back = (O.f16, O.f16_to_f32) if wt == mg.F16 else (O.bf16, O.bf16_to_f32)
    A = conv(O.normal(M * K, 1, 1.0))
    W = conv(O.normal(N * K, 2, 0.02))
    ref = O.gemm_nk(back(A), W, wt, M, N, K)
    dC = dev.empty(M * N, mg.F32)
    mg.gemm(dev, dev.array(A, wt), dev.array(W, wt, mg.LAYOUT_NK), dC, M, N, K).wait()
    assert_close(dC.read(np.float32), ref, TOL_16)


def test_vision_proj_mlp_with_bias(dev):
    # projection MLP 2304 -> 8192 -> 2048 (the GELU between them is not on this path)
    M = 729
    for K, N, seed in ((2304, 8192, 11), (8192, 2048, 12)):
        X = O.f16(O.normal(M * K, seed, 1.0))
        W = O.f16(O.normal(K * N, seed + 1, 0.02))
        bias = O.f16(O.normal(N, seed + 2, 0.5))
        ref = O.add_bias(O.gemm_naive_f32(O.f16_to_f32(X), O.f16_to_f32(W), M, N, K, threads=True),
                         O.f16_to_f32(bias), M, N)
        out = dev.empty(M * N, mg.F16)
        mg.dispatch_vision_proj(dev, None, dev.array(X, mg.F16), dev.create_weight_image(K, N, W),
                                dev.array(bias, mg.F16), out, M, K, N).wait()
        assert_close(O.f16_to_f32(out.read(np.uint16)), ref, TOL_16, f"vision_proj {K}->{N}")


def test_patch_embed(dev):
    # SigLIP patch embedding: 3 x 378 x 378 image, 14 x 14 patches -> [729, 1152] + bias
    C, H, W, ph, pw, E = 3, 378, 378, 14, 14, 1152
    img = O.f16(O.normal(C * H * W, 21, 1.0))
    Wt = O.f16(O.normal(C * ph * pw * E, 22, 0.02))
    bias = O.f16(O.normal(E, 23, 0.5))
    patches = O.im2col(O.f16_to_f32(img), C, H, W, ph, pw)
    P, K = (H // ph) * (W // pw), C * ph * pw
    ref = O.add_bias(O.gemm_naive_f32(patches, O.f16_to_f32(Wt), P, E, K, threads=True), O.f16_to_f32(bias), P, E)
    out = dev.empty(P * E, mg.F16)
    mg.dispatch_patch_embed(dev, None, dev.array(img, mg.F16), dev.create_weight_image(K, E, Wt),
                            dev.array(bias, mg.F16), out, C, H, W, ph, pw, E).wait()
    assert_close(O.f16_to_f32(out.read(np.uint16)), ref, TOL_16, "patch_embed")


def test_gemm_rejects_bad_arguments(dev):
    A, B, C = dev.empty(64, mg.F16), dev.empty(64, mg.F16), dev.empty(64, mg.F32)
    with pytest.raises(mg.MgpuError):
        mg.dispatch_gemm_naive(dev, None, A, B, C, 0, 8, 8)
    with pytest.raises(mg.MgpuError):
        mg.dispatch_gemm_naive(dev, None, A, B, C, 16, 16, 16)  # buffers too small
    Bb = dev.empty(64, mg.BF16)
    with pytest.raises(mg.MgpuError):
        mg.dispatch_gemm_naive(dev, None, A, Bb, C, 8, 8, 8)  # mixed fp16 / bf16 operands
    dev.finish()


@pytest.mark.parametrize("at", [mg.BF16, mg.F16])
@pytest.mark.parametrize("M,N,K", [(1, 100, 256), (3, 2048, 2048), (8, 6144, 2048), (13, 1000, 512),
                                   (8, 2048, 8192), (16, 8192, 2048), (24, 1000, 1024), (5, 51200, 2048),
                                   (40, 2048, 8192), (128, 4096, 2048), (32, 51200, 2048)])
def test_skinny_q4_batched_decode(dev, at, M, N, K):
    # batched decode: M sequences against GGUF Q4_0 weights (the streaming skinny kernel).
    # Its MMAs take the exact (q - 8) and the 16-bit activations and scale each block's sum by d
    # in fp32, so an fp32 output stays within the fp32 tolerance (M <= 32; larger M takes the
    # tcgen05 GEMM, whose B tiles are (q - 8) d rounded to 16 bits)
    A = O.normal(M * K, 3 * M + K, 1.0)
    A16 = O.bf16(A) if at == mg.BF16 else O.f16(A)
    A32 = O.bf16_to_f32(A16) if at == mg.BF16 else O.f16_to_f32(A16)
    W = O.quantize(O.normal(N * K, N + 11, 0.02), O.Q4_0)
    bias = O.normal(N, N + 5, 0.1)
    ref = O.gemm_q(A32, W, M, N, K, O.Q4_0, threads=True).reshape(M, N) + bias[None, :]
    for ct in (mg.F32, mg.BF16, mg.F16):
        dC = dev.empty(M * N, ct)
        mg.gemm_q(dev, dev.array(A16, at), dev.array(W, O.Q4_0, mg.LAYOUT_NK), dC, M, N, K, O.Q4_0,
                  bias=dev.array(bias, mg.F32)).wait()
        C = dC.read(mg.NP_DTYPE[ct])
        C = O.bf16_to_f32(C) if ct == mg.BF16 else O.f16_to_f32(C) if ct == mg.F16 else C
        tol = TOL_F32 if ct == mg.F32 and M <= 32 else TOL_16
        assert_close(C, ref.reshape(-1), tol, f"skinny {M}x{N}x{K} a{at} c{ct}")
