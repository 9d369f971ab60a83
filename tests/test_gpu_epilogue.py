"""GPU parity of mgpu_gemm_fused: C = act(A . op(B) + bias) + residual in the GEMM's epilogue,
against the reference's unfused chain restated in the oracle (the GEMM storing C, the
activation kernel of src/kernels/activations.cl:30-117 rewriting it, the residual add of
src/models/moondream2.cpp:297-300 on top, each rounding to C's type).

The shapes reach every epilogue of the library: the tcgen05 GEMM's own (one CTA or a CTA pair
per tile), its cluster split-K (DSMEM sum), its split-K over global partials (M <= 16, Q8_0)
and the skinny batched-decode kernel (M <= 32, Q4_0)."""
import numpy as np
import pytest

import mvlm_b200 as mg
import oracle as O
from tests.numerics import TOL_16, TOL_F32, assert_close

pytestmark = pytest.mark.gpu

ACTS = [mg.ACT_GELU, mg.ACT_SILU, mg.ACT_GELU_AS_SHIPPED]
BACK = {mg.F32: lambda a: a, mg.F16: O.f16_to_f32, mg.BF16: O.bf16_to_f32}
CONV = {mg.F32: lambda a: np.ascontiguousarray(a, np.float32), mg.F16: O.f16, mg.BF16: O.bf16}


def _quant_case(qt, M, N, K, seed):
    A = O.bf16(O.normal(M * K, seed, 1.0))
    W = O.quantize(O.normal(N * K, seed + 1, 0.02), qt)
    acc = O.gemm_q(O.bf16_to_f32(A), W, M, N, K, qt, threads=True)
    return (A, mg.BF16), (W, qt, mg.LAYOUT_NK), acc


def _run(dev, a, b, M, N, K, ct, bias, act, resid, in_place):
    dA = dev.array(a[0], a[1])
    dB = dev.array(*b)
    dbias = dev.array(bias, mg.F32) if bias is not None else None
    if in_place:
        dC = dev.array(CONV[ct](resid), ct)
        mg.gemm_fused(dev, dA, dB, dC, M, N, K, dbias, act, dC).wait()
    else:
        dR = dev.array(CONV[ct](resid), ct) if resid is not None else None
        dC = dev.empty(M * N, ct)
        mg.gemm_fused(dev, dA, dB, dC, M, N, K, dbias, act, dR).wait()
    return BACK[ct](dC.read(mg.NP_DTYPE[ct]))


@pytest.mark.parametrize("qt,M,N,K,path", [
    (O.Q8_0, 761, 2048, 2048, "cluster split-K"),
    (O.Q8_0, 2048, 4096, 1024, "one tile per CTA / CTA pairs"),
    (O.Q8_0, 8, 2048, 2048, "split-K over global partials"),
    (O.Q4_0, 8, 2048, 2048, "skinny"),
    (O.Q4_0, 32, 6144, 2048, "skinny, 32 sequences"),
    (O.Q8_0, 130, 300, 160, "ragged"),
])
@pytest.mark.parametrize("act", ACTS, ids=["gelu", "silu", "gelu_as_shipped"])
def test_fused_quantised(dev, qt, M, N, K, path, act):
    # The GEMM's operands are bf16 (the packed weights are dequantised to bf16 tiles), so the
    # product meets the 16-bit tensor-core tolerance against the oracle's exact fp32 dequant
    # whatever C's type; the epilogue's own element-wise accuracy is checked separately below.
    a, b, acc = _quant_case(qt, M, N, K, 1000 + M + N + act)
    bias = O.normal(N, 77 + N, 0.5)
    for ct in (mg.BF16, mg.F32):
        resid = BACK[ct](CONV[ct](O.normal(M * N, 5 + M, 1.0)))
        ref = O.unfused_epilogue(acc, bias, act, resid, M, N, ct)
        out = _run(dev, a, b, M, N, K, ct, bias, act, resid, in_place=False)
        assert_close(out, ref, TOL_16, f"{path} q{qt} {M}x{N}x{K} act{act} c{ct}")


def _act_truth(v, act):
    """act on fp32 pre-activations, in float64 through the sigmoid identities
    0.5 v (1 + tanh(u)) = v / (1 + exp(-2u)) and 0.5 v (1 - tanh(u)) = v / (1 + exp(2u)), which
    cancel nowhere (a 1 + tanh(u) evaluation loses all digits where tanh(u) is near -1)."""
    v = np.asarray(v, np.float64)
    inner = np.float64(np.float32(0.7978845608)) * (v + np.float64(np.float32(0.044715)) * v ** 3)
    z = {mg.ACT_SILU: v, mg.ACT_GELU: 2.0 * inner, mg.ACT_GELU_AS_SHIPPED: -2.0 * inner}[act]
    with np.errstate(over="ignore"):
        return v / (1.0 + np.exp(-z))


@pytest.mark.parametrize("qt,M,path", [(O.Q8_0, 761, "cluster split-K"), (O.Q8_0, 2048, "tiles / CTA pairs"),
                                       (O.Q8_0, 8, "split-K over global partials"), (O.Q4_0, 8, "skinny")])
@pytest.mark.parametrize("act", ACTS, ids=["gelu", "silu", "gelu_as_shipped"])
def test_fused_activation_elementwise(dev, qt, M, path, act):
    # A = 0 makes the accumulator exactly 0, so C = act(bias) with the bias spanning the
    # pre-activations [-12, 12]: each output is checked on its own against the float64 value,
    # tails included (silu(-10) = -4.5e-4 must come out with its sign and ~fp32 precision).
    N, K = 2048, 2048
    A = np.zeros(M * K, np.uint16)
    W = O.quantize(O.normal(N * K, 5, 0.02), qt)
    bias = np.linspace(-12.0, 12.0, N).astype(np.float32)
    truth = _act_truth(bias, act)
    dA, dW, db = dev.array(A, mg.BF16), dev.array(W, qt, mg.LAYOUT_NK), dev.array(bias, mg.F32)
    for ct, rtol in ((mg.F32, TOL_F32), (mg.BF16, 2.0 ** -8 + TOL_F32)):
        dC = dev.empty(M * N, ct)
        mg.gemm_fused(dev, dA, dW, dC, M, N, K, db, act, None).wait()
        out = BACK[ct](dC.read(mg.NP_DTYPE[ct])).reshape(M, N).astype(np.float64)
        err = np.abs(out - truth[None, :])
        bad = err > rtol * np.abs(truth)[None, :] + 1e-30
        assert not bad.any(), (f"{path} act{act} c{ct}: {int(bad.sum())} outputs off, worst at pre-activation "
                               f"{bias[np.argwhere(bad)[0][1]]}: {out[bad][0]} vs {truth[np.argwhere(bad)[0][1]]}")
        neg = truth < -1e-30
        assert np.all(np.signbit(out[:, neg])), f"{path} act{act} c{ct}: sign lost for negative outputs"


@pytest.mark.parametrize("qt,M,N,K", [(O.Q8_0, 761, 2048, 2048), (O.Q4_0, 8, 2048, 2048), (O.Q8_0, 8, 2048, 2048)])
def test_fused_residual_in_place(dev, qt, M, N, K):
    # hidden = hidden + (A . W^T): the residual buffer is C itself, as moondream2_forward's
    # dispatch_residual_add(hidden, residual_buf, hidden) writes in place
    a, b, acc = _quant_case(qt, M, N, K, 2000 + M)
    ct = mg.F16
    hidden = O.f16_to_f32(O.f16(O.normal(M * N, 3, 1.0)))
    ref = O.unfused_epilogue(acc, None, mg.ACT_NONE, hidden, M, N, ct)
    out = _run(dev, a, b, M, N, K, ct, None, mg.ACT_NONE, hidden, in_place=True)
    assert_close(out, ref, TOL_16, f"in-place residual q{qt} {M}x{N}x{K}")


@pytest.mark.parametrize("M,N,K", [(729, 4304, 1152), (729, 8192, 2304)])
def test_fused_fp16_reference_orientation(dev, M, N, K):
    # SigLIP fc1 and the projection MLP's first GEMM with GELU: fp16 activations and fp16
    # weights in the reference's B[K][N] orientation, fp16 C
    A = O.f16(O.normal(M * K, 40 + K, 1.0))
    B = O.f16(O.normal(K * N, 41 + N, 0.02))
    bias = O.normal(N, 42, 0.5)
    acc = O.gemm_naive_f32(O.f16_to_f32(A), O.f16_to_f32(B), M, N, K, threads=True)
    ref = O.unfused_epilogue(acc, bias, mg.ACT_GELU, None, M, N, mg.F16)
    out = _run(dev, (A, mg.F16), (B, mg.F16, mg.LAYOUT_KN), M, N, K, mg.F16, bias, mg.ACT_GELU, None, False)
    assert_close(out, ref, TOL_16, f"fp16 KN gelu {M}x{N}x{K}")


def test_fused_without_epilogue_matches_gemm(dev):
    # act NONE and no residual is mgpu_gemm bit for bit
    (A, at), (W, qt, lay), _ = _quant_case(O.Q8_0, 300, 1000, 512, 9)
    bias = O.normal(1000, 10, 0.5)
    dA, dW, db = dev.array(A, at), dev.array(W, qt, lay), dev.array(bias, mg.F32)
    c1, c2 = dev.empty(300 * 1000, mg.F32), dev.empty(300 * 1000, mg.F32)
    mg.gemm(dev, dA, dW, c1, 300, 1000, 512, db).wait()
    mg.gemm_fused(dev, dA, dW, c2, 300, 1000, 512, db, mg.ACT_NONE, None).wait()
    assert np.array_equal(c1.read(np.float32), c2.read(np.float32))


def test_fused_rejects_bad_arguments(dev):
    (A, at), (W, qt, lay), _ = _quant_case(O.Q8_0, 16, 64, 256, 11)
    dA, dW = dev.array(A, at), dev.array(W, qt, lay)
    C = dev.empty(16 * 64, mg.F32)
    with pytest.raises(mg.MgpuError, match="unknown activation"):
        mg.gemm_fused(dev, dA, dW, C, 16, 64, 256, None, 7, None)
    with pytest.raises(mg.MgpuError, match="residual buffer too small"):
        mg.gemm_fused(dev, dA, dW, C, 16, 64, 256, None, mg.ACT_NONE, dev.empty(16 * 63, mg.F32))
    C16 = dev.empty(16 * 64 + 8, mg.F16)
    with pytest.raises(mg.MgpuError, match="in-place residual"):
        mg.gemm_fused(dev, dA, dW, C16, 16, 64, 256, None, mg.ACT_NONE, C16.view(0, 16 * 64 * 2).set_format(mg.BF16))
    with pytest.raises(mg.MgpuError, match="overlaps C"):
        mg.gemm_fused(dev, dA, dW, C16, 16, 64, 256, None, mg.ACT_NONE, C16.view(16, 16 * 64 * 2))
    dev.finish()


@pytest.mark.parametrize("qt,M,N,K", [(O.Q8_0, 761, 8192, 2048), (O.Q4_0, 8, 8192, 2048), (O.Q8_0, 8, 2048, 2048),
                                      (O.Q8_0, 130, 300, 160)])
def test_silu_gate(dev, qt, M, N, K):
    # the SiLU-gated MLP of moondream2_forward (moondream2.cpp:465-495): up = A . W_up^T first,
    # then out = silu(A . W_gate^T) * up in the gate GEMM's epilogue, against the reference's
    # gate GEMM + silu_gate_multiply with fp16 stores in between
    a, b, acc = _quant_case(qt, M, N, K, 3000 + M + N)
    ct = mg.F16
    up = O.f16_to_f32(O.f16(O.normal(M * N, 31, 1.0)))
    ref = O.unfused_silu_gate(acc, up, ct)
    dA, dW = dev.array(a[0], a[1]), dev.array(*b)
    dU = dev.array(O.f16(up), ct)
    out = dev.empty(M * N, ct)
    mg.gemm_silu_gate(dev, dA, dW, dU, out, M, N, K).wait()
    assert_close(O.f16_to_f32(out.read(np.uint16)), ref, TOL_16, f"silu gate q{qt} {M}x{N}x{K}")
    # in place: the product overwrites up
    mg.gemm_silu_gate(dev, dA, dW, dU, dU, M, N, K).wait()
    assert_close(O.f16_to_f32(dU.read(np.uint16)), ref, TOL_16, f"silu gate in place q{qt} {M}x{N}x{K}")
