"""Dependent chains: each launch reads the previous launch's output.

The GEMV, the tcgen05 GEMM and the skinny GEMM are launched with programmatic dependent launch:
they stage weights before griddepcontrol.wait and read activations only after it.  These tests
run chains in which every input is the preceding kernel's output (eagerly and as a captured
graph) and compare the end of the chain with the CPU oracle applying the same steps, with the
same intermediate roundings."""
import numpy as np
import pytest

import mvlm_b200 as mg
import oracle as O
from tests.numerics import TOL_16, TOL_F32, assert_close

pytestmark = pytest.mark.gpu


def _weights(n, K, N, qt, seed):
    return [O.quantize(O.normal(N * K, seed + i, 0.02), qt) for i in range(n)]


@pytest.mark.parametrize("graph", [False, True], ids=["eager", "graph"])
@pytest.mark.parametrize("qt", [O.Q4_0, O.Q8_0])
def test_gemv_chain(dev, qt, graph):
    # x -> W0 -> W1 -> ... (square K = N = 2048, fp32 activations), six dependent GEMVs
    K = N = 2048
    Ws = _weights(6, K, N, qt, 40)
    x0 = O.normal(K, 41, 1.0)
    bufs = [dev.array(x0, mg.F32)] + [dev.empty(N, mg.F32) for _ in Ws]
    dWs = [dev.array(W, qt, mg.LAYOUT_NK) for W in Ws]

    def run():
        for i, dW in enumerate(dWs):
            mg.gemv_q(dev, bufs[i], dW, bufs[i + 1], N, K, qt)

    if graph:
        run()
        dev.finish()
        dev.capture_begin()
        run()
        g = dev.capture_end()
        for b in bufs[1:]:  # a replay that read a stale input would now read zeros
            b.write(np.zeros(N, np.float32))
        g.launch()
    else:
        run()
    dev.finish()
    ref = x0
    for W in Ws:
        ref = O.gemm_q(ref, W, 1, N, K, qt)
    # six fp32-output steps, each within TOL_F32 of its oracle step: the error can add up
    assert_close(bufs[-1].read(np.float32), ref, 6 * TOL_F32, "gemv chain")


@pytest.mark.parametrize("graph", [False, True], ids=["eager", "graph"])
def test_gemm_chain_prefill(dev, graph):
    # A (761 x 512 bf16) -> Q8_0 -> Q4_0 -> Q8_0: each output (bf16) is the next A
    M, K = 761, 512
    qts = [O.Q8_0, O.Q4_0, O.Q8_0]
    Ws = [O.quantize(O.normal(K * K, 50 + i, 0.05), qt) for i, qt in enumerate(qts)]
    A0 = O.bf16(O.normal(M * K, 51, 1.0))
    bufs = [dev.array(A0, mg.BF16)] + [dev.empty(M * K, mg.BF16) for _ in Ws]
    dWs = [dev.array(W, qt, mg.LAYOUT_NK) for W, qt in zip(Ws, qts)]

    def run():
        for i, (dW, qt) in enumerate(zip(dWs, qts)):
            mg.gemm_q(dev, bufs[i], dW, bufs[i + 1], M, K, K, qt)

    if graph:
        run()
        dev.finish()
        dev.capture_begin()
        run()
        g = dev.capture_end()
        for b in bufs[1:]:  # a replay that read a stale input would now read zeros
            b.write(np.zeros(M * K, np.uint16))
        g.launch()
    else:
        run()
    dev.finish()
    ref = O.bf16_to_f32(A0)
    for W, qt in zip(Ws, qts):
        ref = O.bf16_to_f32(O.bf16(O.gemm_q(ref, W, M, K, K, qt, threads=True)))
    out = O.bf16_to_f32(bufs[-1].read(np.uint16))
    # three tensor-core steps, each within TOL_16 of its oracle step (same bf16 roundings)
    assert_close(out, ref, 3 * TOL_16, "gemm chain")


@pytest.mark.parametrize("S", [8, 32])
def test_skinny_chain_batched_decode(dev, S):
    # S sequences through four Q4_0 layers (K = N = 2048), bf16 activations between them
    K = 2048
    Ws = _weights(4, K, K, O.Q4_0, 60)
    A0 = O.bf16(O.normal(S * K, 61, 1.0))
    bufs = [dev.array(A0, mg.BF16)] + [dev.empty(S * K, mg.BF16) for _ in Ws]
    dWs = [dev.array(W, O.Q4_0, mg.LAYOUT_NK) for W in Ws]
    for i, dW in enumerate(dWs):
        mg.gemm_q(dev, bufs[i], dW, bufs[i + 1], S, K, K, O.Q4_0)
    dev.finish()
    ref = O.bf16_to_f32(A0)
    for W in Ws:
        ref = O.bf16_to_f32(O.bf16(O.gemm_q(ref, W, S, K, K, O.Q4_0, threads=True)))
    out = O.bf16_to_f32(bufs[-1].read(np.uint16))
    assert_close(out, ref, 3 * TOL_16, f"skinny chain S={S}")


def test_mixed_chain(dev):
    # prefill GEMM (bf16 out) -> its last row as fp32 -> decode GEMV -> GEMV, as one stream
    M, K = 130, 1024
    Wg = O.quantize(O.normal(K * K, 70, 0.05), O.Q8_0)
    Wv = _weights(2, K, K, O.Q4_0, 71)
    A = O.bf16(O.normal(M * K, 72, 1.0))
    dA = dev.array(A, mg.BF16)
    dC = dev.empty(M * K, mg.F32)
    mg.gemm_q(dev, dA, dev.array(Wg, O.Q8_0, mg.LAYOUT_NK), dC, M, K, K, O.Q8_0)
    last = dC.view((M - 1) * K * 4, K * 4)
    y1, y2 = dev.empty(K, mg.F32), dev.empty(K, mg.F32)
    mg.gemv_q(dev, last, dev.array(Wv[0], O.Q4_0, mg.LAYOUT_NK), y1, K, K, O.Q4_0)
    mg.gemv_q(dev, y1, dev.array(Wv[1], O.Q4_0, mg.LAYOUT_NK), y2, K, K, O.Q4_0)
    dev.finish()
    C = O.gemm_q(O.bf16_to_f32(A), Wg, M, K, K, O.Q8_0, threads=True).reshape(M, K)
    ref = O.gemm_q(O.gemm_q(C[-1], Wv[0], 1, K, K, O.Q4_0), Wv[1], 1, K, K, O.Q4_0)
    assert_close(y2.read(np.float32), ref, TOL_16, "mixed chain")
