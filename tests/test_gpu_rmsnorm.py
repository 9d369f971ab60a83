"""GPU parity of the RMSNorm path: mgpu_dispatch_rms_norm (replaces dispatch_rms_norm,
src/engine/compute.cpp:156-184, and its kernel src/kernels/layernorm.cl:41-146) against the
oracle's restatement, and mgpu_gemv_q_rmsnorm (the norm fused into the decode GEMV's prologue)
against the reference's unfused chain -- rms_norm storing x' in x's type, then dispatch_gemv
reading it (moondream2.cpp:359-367, :455-463) -- run both on the GPU (same bits) and in the
oracle (within the fp32 tolerance)."""
import numpy as np
import pytest

import mvlm_b200 as mg
import oracle as O
from tests.numerics import TOL_16, TOL_F32, assert_close

pytestmark = pytest.mark.gpu

CONV = {mg.F32: lambda a: np.ascontiguousarray(a, np.float32), mg.F16: O.f16, mg.BF16: O.bf16}
BACK = {mg.F32: lambda a: a, mg.F16: O.f16_to_f32, mg.BF16: O.bf16_to_f32}


@pytest.mark.parametrize("t", [mg.F16, mg.BF16, mg.F32])
@pytest.mark.parametrize("rows,H", [(1, 2048), (761, 2048), (2, 8192), (3, 1000), (5, 1152)])
def test_dispatch_rms_norm(dev, t, rows, H):
    eps = 1e-5
    x = CONV[t](O.normal(rows * H, rows + H, 2.0))
    w = O.f16(O.normal(H, H, 0.5))
    out = dev.empty(rows * H, t)
    mg.dispatch_rms_norm(dev, None, dev.array(x, t), out, dev.array(w, mg.F16), rows, H, eps).wait()
    ref = O.rms_norm(BACK[t](x), O.f16_to_f32(w), rows, H, eps, t)
    assert_close(BACK[t](out.read(mg.NP_DTYPE[t])), ref, TOL_F32 if t == mg.F32 else TOL_16, f"rms_norm t{t} {rows}x{H}")


@pytest.mark.parametrize("qt", [O.Q4_0, O.Q8_0])
@pytest.mark.parametrize("xt", [mg.F32, mg.F16])
@pytest.mark.parametrize("K,N", [(2048, 6144), (8192, 2048), (2048, 51200), (3072, 500)])
def test_gemv_q_rmsnorm_fused(dev, qt, xt, K, N):
    eps = 1e-5
    x = CONV[xt](O.normal(K, K + N, 1.5))
    gamma = O.f16(O.normal(K, K, 0.7))
    W = O.quantize(O.normal(N * K, N, 0.02), qt)
    dx, dg, dW = dev.array(x, xt), dev.array(gamma, mg.F16), dev.array(W, qt, mg.LAYOUT_NK)
    fused = dev.empty(N, mg.F32)
    mg.gemv_q_rmsnorm(dev, dx, dg, eps, dW, fused, N, K, qt).wait()
    # the reference's chain on the GPU: rms_norm storing x' in x's type, then the GEMV
    xn = dev.empty(K, xt)
    mg.dispatch_rms_norm(dev, None, dx, xn, dg, 1, K, eps)
    chain = dev.empty(N, mg.F32)
    mg.gemv_q(dev, xn, dW, chain, N, K, qt).wait()
    f, c = fused.read(np.float32), chain.read(np.float32)
    assert np.array_equal(f, c), f"fused and unfused differ: max {np.max(np.abs(f - c))}"
    # and the same chain in the oracle
    xr = O.rms_norm(BACK[xt](x), O.f16_to_f32(gamma), 1, K, eps, xt)
    ref = O.gemm_q(xr, W, 1, N, K, qt, threads=True)
    assert_close(f, ref, TOL_F32 if xt == mg.F32 else TOL_16, f"gemv_q_rmsnorm q{qt} x{xt} {K}x{N}")
