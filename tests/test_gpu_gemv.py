"""GPU parity of the decode GEMV (replaces gemv, src/kernels/gemm.cl:219-270) against the CPU
oracle, through the C ABI.  Sizes are the Phi-1.5 decode shapes of the benchmark config plus
ragged / misaligned edge cases."""
import numpy as np
import pytest

import mvlm_b200 as mg
import oracle as O
from tests.numerics import TOL_16, TOL_F32, assert_close

pytestmark = pytest.mark.gpu

PHI_SHAPES = [(2048, 6144), (2048, 2048), (2048, 8192), (8192, 2048), (2048, 51200)]  # K x N


def _q_weights(N, K, t, seed):
    return O.quantize(O.normal(N * K, seed, 0.02), t)


@pytest.mark.parametrize("qt", [O.Q4_0, O.Q8_0])
@pytest.mark.parametrize("K,N", PHI_SHAPES)
def test_gemv_q_phi_shapes_fp32(dev, qt, K, N):
    x = O.normal(K, 0x4D564C4D + N, 1.0)
    W = _q_weights(N, K, qt, 0x4D564C4E + K)
    ref = O.gemm_q(x, W, 1, N, K, qt, threads=True)
    dx, dW, dy = dev.array(x, mg.F32), dev.array(W, qt, mg.LAYOUT_NK), dev.empty(N, mg.F32)
    ev = mg.gemv_q(dev, dx, dW, dy, N, K, qt)
    ev.wait()
    assert_close(dy.read(np.float32), ref, TOL_F32, f"gemv q{qt} {K}x{N}")


@pytest.mark.parametrize("xt,yt", [(mg.F16, mg.F32), (mg.BF16, mg.F32), (mg.F32, mg.F16), (mg.F32, mg.BF16),
                                   (mg.F16, mg.F16)])
@pytest.mark.parametrize("qt", [O.Q4_0, O.Q8_0])
def test_gemv_q_io_types(dev, qt, xt, yt):
    K, N = 2048, 3000
    xf = O.normal(K, 17, 1.0)
    x16 = O.f16(xf) if xt == mg.F16 else O.bf16(xf) if xt == mg.BF16 else xf
    xr = O.f16_to_f32(x16) if xt == mg.F16 else O.bf16_to_f32(x16) if xt == mg.BF16 else xf
    W = _q_weights(N, K, qt, 18)
    ref = O.gemm_q(xr, W, 1, N, K, qt, threads=True)
    dy = dev.empty(N, yt)
    mg.gemv_q(dev, dev.array(x16, xt), dev.array(W, qt, mg.LAYOUT_NK), dy, N, K, qt).wait()
    y = dy.read(mg.NP_DTYPE[yt])
    y = O.f16_to_f32(y) if yt == mg.F16 else O.bf16_to_f32(y) if yt == mg.BF16 else y
    assert_close(y, ref, TOL_F32 if yt == mg.F32 else TOL_16)


@pytest.mark.parametrize("K,N", [(32, 1), (96, 7), (1152, 33), (4096, 5), (16384, 64), (1024, 1), (2048, 3),
                                 (8192, 300), (3072, 500), (5120, 129), (7168, 40), (6144, 4000)])
@pytest.mark.parametrize("qt", [O.Q4_0, O.Q8_0])
def test_gemv_q_ragged(dev, qt, K, N):
    x = O.uniform(K, K + N)
    W = _q_weights(N, K, qt, 7 * K + N)
    ref = O.gemm_q(x, W, 1, N, K, qt)
    dy = dev.empty(N, mg.F32)
    mg.gemv_q(dev, dev.array(x, mg.F32), dev.array(W, qt, mg.LAYOUT_NK), dy, N, K, qt).wait()
    assert_close(dy.read(np.float32), ref, TOL_F32, f"ragged {K}x{N}")


@pytest.mark.parametrize("qt", [O.Q4_0, O.Q8_0])
def test_gemv_q_misaligned_rows(dev, qt):
    # weights starting 2 bytes into an allocation: rows are not 16-byte aligned -> generic kernel
    K, N = 2048, 129
    x = O.uniform(K, 5)
    W = _q_weights(N, K, qt, 6)
    ref = O.gemm_q(x, W, 1, N, K, qt)
    big = dev.create_buffer(W.size + 16, None)
    big.write(W, offset=2)
    view = big.view(2, W.size).set_format(qt, mg.LAYOUT_NK)
    dy = dev.empty(N, mg.F32)
    mg.gemv_q(dev, dev.array(x, mg.F32), view, dy, N, K, qt).wait()
    assert_close(dy.read(np.float32), ref, TOL_F32)


@pytest.mark.parametrize("wt", [mg.F32, mg.F16, mg.BF16])
@pytest.mark.parametrize("K,N", [(2048, 2048), (1152, 100), (100, 37)])
def test_gemv_dense_nk(dev, wt, K, N):
    x = O.normal(K, 3, 1.0)
    Wf = O.normal(N * K, 4, 0.02)
    W = O.f16(Wf) if wt == mg.F16 else O.bf16(Wf) if wt == mg.BF16 else Wf
    ref = O.gemm_nk(x, W, wt, 1, N, K)
    dy = dev.empty(N, mg.F32)
    mg.dispatch_gemv(dev, None, dev.array(x, mg.F32), dev.array(W, wt, mg.LAYOUT_NK), dy, N, K).wait()
    assert_close(dy.read(np.float32), ref, TOL_F32)


def test_gemv_fp32_kn_config0(dev):
    # fp32 GEMV M=1, K=2048, N=8192, x and W row-major [K,N] ~U(-1,1)
    K, N = 2048, 8192
    x = O.uniform(K, 0x4D564C4D)
    W = O.uniform(K * N, 0x4D564C4E)
    ref = O.gemv_f32(x, W, N, K)
    dx, dW, dy = dev.array(x, mg.F32), dev.array(W, mg.F32, mg.LAYOUT_KN), dev.empty(N, mg.F32)
    outs = []
    for _ in range(3):  # repeated calls: the split-K tickets reset themselves; results identical
        mg.dispatch_gemv(dev, None, dx, dW, dy, N, K).wait()
        outs.append(dy.read(np.float32))
    assert_close(outs[0], ref, TOL_F32, "fp32 gemv KN")
    np.testing.assert_array_equal(outs[0], outs[1])
    np.testing.assert_array_equal(outs[0], outs[2])


@pytest.mark.parametrize("N,K", [(4, 16), (7, 300), (33, 513), (8, 2048), (8192, 2048)])
def test_gemv_fp16_image_vs_reference(dev, N, K):
    # fp16 x, fp16 weight image [K,N] (create_weight_image), fp16 y: the reference gemv's types
    x = O.f16(O.uniform(K, 0x3000 + N))
    W = O.f16(O.uniform(K * N, 0x4000 + K))
    ref16 = O.gemv_f16(x, W, N, K)  # bit-identical to the reference gemm.cl gemv (tests/test_oracle.py)
    ref32 = O.gemv_f32(O.f16_to_f32(x), O.f16_to_f32(W), N, K)
    img = dev.create_weight_image(K, N, W)
    dy = dev.empty(N, mg.F16)
    mg.dispatch_gemv(dev, None, dev.array(x, mg.F16), img, dy, N, K).wait()
    y = O.f16_to_f32(dy.read(np.uint16))
    assert_close(y, ref32, TOL_16, "vs fp32")
    assert_close(y, O.f16_to_f32(ref16), TOL_16, "vs reference fp16 output")


def test_gemv_rejects_bad_arguments(dev):
    x, y = dev.empty(64, mg.F32), dev.empty(16, mg.F32)
    W = dev.create_buffer(16 * 2 * 18, None, mg.Q4_0, mg.LAYOUT_NK)
    with pytest.raises(mg.MgpuError) as e:
        mg.gemv_q(dev, x, W, y, 16, 48, mg.Q4_0)  # K % 32 != 0
    assert e.value.code == mg.ERR_INVALID_ARG
    with pytest.raises(mg.MgpuError):
        mg.gemv_q(dev, x, W, y, 17, 64, mg.Q4_0)  # W too small for N
    with pytest.raises(mg.MgpuError):
        mg.dispatch_gemv(dev, None, x, W, y, 0, 64)
    dev.finish()  # nothing was enqueued; the device is still healthy
