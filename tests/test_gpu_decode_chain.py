"""GPU parity of mgpu_gemv_chain, the decode step's GEMVs in one persistent launch.

The chain replaces moondream2_forward's run of dependent dispatch_gemv calls
(src/models/moondream2.cpp:357-542).  Each test builds links whose inputs are earlier links'
outputs (the Phi-1.5 layer order qkv -> out -> fc1 -> fc2 -> next layer, then the lm_head) and
checks every link's output against the CPU oracle applying the same GEMVs in the same order
with the same intermediate roundings.  A link that read its input before the producing link
had written all of it would read the other launch's values or the sentinel and fail here;
successive runs alternate between the mailboxes' two copies, so each test runs the chain more
than once (eagerly and from a captured graph)."""
import numpy as np
import pytest

import mvlm_b200 as mg
import oracle as O
from tests.numerics import TOL_16, TOL_F32, assert_close

pytestmark = pytest.mark.gpu

PHI = [("qkv", 2048, 6144), ("out", 2048, 2048), ("fc1", 2048, 8192), ("fc2", 8192, 2048)]  # (name, K, N)


def _phi_links(dev, qt, layers, head_n, seed, ytype=mg.F32):
    """links of `layers` Phi-1.5 layers + an lm_head of head_n rows; x of every link but the first
    is (a prefix of) the previous link's y.  Returns (links, host weights, x0)."""
    shapes = [s for _ in range(layers) for s in PHI] + [("head", 2048, head_n)]
    x0 = O.normal(2048, seed, 1.0)
    xb = dev.array(x0, mg.F32)
    links, Ws, prev = [], [], None
    for i, (_, K, N) in enumerate(shapes):
        W = O.quantize(O.normal(N * K, seed + 1 + i, 0.02), qt)
        Ws.append(W)
        y = dev.empty(N, ytype)
        if prev is None:
            x = xb
        else:
            esz = mg.TYPE_SIZE[ytype]
            x = prev.view(0, K * esz).set_format(ytype)
        links.append((x, dev.array(W, qt, mg.LAYOUT_NK), y, N, K))
        prev = y
    return links, Ws, x0, shapes


def _oracle_chain(x0, Ws, shapes, qt, ytype=mg.F32):
    outs, x = [], x0
    for W, (_, K, N) in zip(Ws, shapes):
        y = O.gemm_q(np.ascontiguousarray(x[:K], np.float32), W, 1, N, K, qt, threads=True)
        y = O.round_to(y, ytype)
        outs.append(y)
        x = y
    return outs


def _read(buf, ytype):
    v = buf.read(mg.NP_DTYPE[ytype])
    return O.f16_to_f32(v) if ytype == mg.F16 else O.bf16_to_f32(v) if ytype == mg.BF16 else v


@pytest.mark.parametrize("qt", [O.Q4_0, O.Q8_0])
def test_chain_phi_layers_eager_and_graph(dev, qt):
    links, Ws, x0, shapes = _phi_links(dev, qt, layers=2, head_n=51200, seed=0x4D564C4D + qt)
    refs = _oracle_chain(x0, Ws, shapes, qt)
    chain = mg.GemvChain(dev, links)
    n = len(links)
    for run in range(2):  # the second run uses the other mailbox copy
        for _, _, y, N, _ in links:
            y.write(np.full(N, np.nan, np.float32))
        chain.run().wait()
        dev.finish()
        for i, ((_, _, y, N, K), ref) in enumerate(zip(links, refs)):
            # i + 1 fp32-output steps, each within TOL_F32 of its oracle step
            assert_close(y.read(np.float32), ref, (i + 1) * TOL_F32, f"run {run} link {i} ({shapes[i][0]}) q{qt}")
    # the same chain from a captured graph, replayed three times
    dev.capture_begin()
    chain.run()
    g = dev.capture_end()
    outs = []
    for _ in range(3):
        for _, _, y, N, _ in links:
            y.write(np.full(N, np.nan, np.float32))
        g.launch()
        dev.finish()
        outs.append(links[-1][2].read(np.float32))
        assert_close(outs[-1], refs[-1], n * TOL_F32, f"graph replay q{qt}")
    # the sums are in a fixed order: every run gives the same bits
    assert np.array_equal(outs[0], outs[1]) and np.array_equal(outs[1], outs[2])
    chain.destroy()


@pytest.mark.parametrize("ytype", [mg.F16, mg.BF16])
def test_chain_16bit_outputs_feed_the_next_link(dev, ytype):
    # y stored as f16 / bf16: the next link must read exactly the rounded values (what a
    # separate launch reading y would read), not the fp32 sums
    qt = O.Q4_0
    links, Ws, x0, shapes = _phi_links(dev, qt, layers=1, head_n=4096, seed=77, ytype=ytype)
    refs = _oracle_chain(x0, Ws, shapes, qt, ytype)
    chain = mg.GemvChain(dev, links)
    for _ in range(2):
        chain.run().wait()
        dev.finish()
        for i, ((_, _, y, N, K), ref) in enumerate(zip(links, refs)):
            assert_close(_read(y, ytype), ref, TOL_16, f"link {i} y{ytype}")


def test_chain_matches_separate_launches(dev):
    # the same dataflow as six separate mgpu_gemv_q launches
    qt = O.Q4_0
    links, Ws, x0, shapes = _phi_links(dev, qt, layers=1, head_n=2048, seed=5)
    chain = mg.GemvChain(dev, links)
    chain.run().wait()
    dev.finish()
    got = [y.read(np.float32) for _, _, y, _, _ in links]
    sep = [dev.empty(N, mg.F32) for _, _, _, N, _ in links]
    x = links[0][0]
    for (_, W, _, N, K), y in zip(links, sep):
        mg.gemv_q(dev, x, W, y, N, K, qt)  # x holds at least K values; the first K are read
        x = y
    dev.finish()
    for i, (a, b) in enumerate(zip(got, sep)):
        assert_close(a, b.read(np.float32), (i + 1) * TOL_F32, f"chain vs separate launch, link {i}")


def test_chain_external_inputs_and_mixed_x_types(dev):
    # links whose x are independent buffers of every float type (no dataflow between them)
    qt = O.Q8_0
    cases = [(mg.F32, 1024, 3000), (mg.F16, 4096, 700), (mg.BF16, 8192, 2048), (mg.F32, 2048, 5)]
    links, refs = [], []
    for i, (xt, K, N) in enumerate(cases):
        xf = O.normal(K, 90 + i, 1.0)
        xs = O.f16(xf) if xt == mg.F16 else O.bf16(xf) if xt == mg.BF16 else xf
        xr = O.f16_to_f32(xs) if xt == mg.F16 else O.bf16_to_f32(xs) if xt == mg.BF16 else xf
        W = O.quantize(O.normal(N * K, 95 + i, 0.02), qt)
        refs.append(O.gemm_q(xr, W, 1, N, K, qt, threads=True))
        links.append((dev.array(xs, xt), dev.array(W, qt, mg.LAYOUT_NK), dev.empty(N, mg.F32), N, K))
    chain = mg.GemvChain(dev, links)
    for _ in range(2):
        chain.run().wait()
        dev.finish()
        for i, ((_, _, y, _, _), ref) in enumerate(zip(links, refs)):
            assert_close(y.read(np.float32), ref, TOL_F32, f"external link {i}")


def test_chain_reads_an_offset_view_and_an_older_link(dev):
    # link 2 reads link 0's output at an element offset (a later part of a qkv output), link 3
    # reads link 1's: dataflow need not be link i -> i + 1
    qt = O.Q4_0
    x0 = O.normal(2048, 3, 1.0)
    W = [O.quantize(O.normal(N * K, 10 + i, 0.02), qt) for i, (K, N) in
         enumerate([(2048, 6144), (2048, 2048), (2048, 1024), (2048, 3000)])]
    y = [dev.empty(6144, mg.F32), dev.empty(2048, mg.F32), dev.empty(1024, mg.F32), dev.empty(3000, mg.F32)]
    xb = dev.array(x0, mg.F32)
    links = [(xb, dev.array(W[0], qt, mg.LAYOUT_NK), y[0], 6144, 2048),
             (y[0].view(0, 2048 * 4).set_format(mg.F32), dev.array(W[1], qt, mg.LAYOUT_NK), y[1], 2048, 2048),
             (y[0].view(4096 * 4, 2048 * 4).set_format(mg.F32), dev.array(W[2], qt, mg.LAYOUT_NK), y[2], 1024, 2048),
             (y[1], dev.array(W[3], qt, mg.LAYOUT_NK), y[3], 3000, 2048)]
    r0 = O.gemm_q(x0, W[0], 1, 6144, 2048, qt)
    r1 = O.gemm_q(r0[:2048].copy(), W[1], 1, 2048, 2048, qt)
    r2 = O.gemm_q(r0[4096:].copy(), W[2], 1, 1024, 2048, qt)
    r3 = O.gemm_q(r1, W[3], 1, 3000, 2048, qt)
    chain = mg.GemvChain(dev, links)
    for _ in range(3):
        chain.run().wait()
        dev.finish()
        for i, r in enumerate((r0, r1, r2, r3)):
            assert_close(y[i].read(np.float32), r, 3 * TOL_F32, f"link {i}")


@pytest.mark.parametrize("n", [1, 3, 17, 64, 192])
def test_chain_lengths(dev, n):
    # the stage table lives in shared memory beside the weight ring, so its size changes the
    # ring's depth: every length up to the limit must launch and stay correct
    qt, K = O.Q8_0, 1024
    x0 = O.normal(K, n, 1.0)
    Ws = [O.quantize(O.normal(K * K, 1000 * n + i, 0.03), qt) for i in range(n)]
    ys = [dev.empty(K, mg.F32) for _ in range(n)]
    links, x = [], dev.array(x0, mg.F32)
    for W, y in zip(Ws, ys):
        links.append((x, dev.array(W, qt, mg.LAYOUT_NK), y, K, K))
        x = y
    chain = mg.GemvChain(dev, links)
    ref = x0
    for W in Ws:
        ref = O.gemm_q(ref, W, 1, K, K, qt)
    for _ in range(2):
        chain.run().wait()
        dev.finish()
        assert_close(ys[-1].read(np.float32), ref, n * TOL_F32, f"{n} links")
    with pytest.raises(mg.MgpuError) as e:
        mg.GemvChain(dev, links + links[:1] * (193 - n))
    assert e.value.code in (mg.ERR_UNSUPPORTED, mg.ERR_INVALID_ARG)


def test_chain_timed_run(dev):
    links, _, _, _ = _phi_links(dev, O.Q4_0, layers=1, head_n=51200, seed=8)
    chain = mg.GemvChain(dev, links)
    t = chain.run_timed()
    assert t.shape == (len(links),) and np.all(t > 0) and np.all(np.diff(t) >= 0), t


def test_chain_rejects_what_it_cannot_run(dev):
    qt = O.Q4_0
    W = dev.array(O.quantize(O.normal(64 * 2048, 1, 0.02), qt), qt, mg.LAYOUT_NK)
    x = dev.array(O.normal(2048, 2, 1.0), mg.F32)
    y = dev.empty(64, mg.F32)
    with pytest.raises(mg.MgpuError) as e:  # K outside the chain's shapes
        W3 = dev.array(O.quantize(O.normal(64 * 3072, 1, 0.02), qt), qt, mg.LAYOUT_NK)
        mg.GemvChain(dev, [(dev.array(O.normal(3072, 2, 1.0), mg.F32), W3, y, 64, 3072)])
    assert e.value.code == mg.ERR_UNSUPPORTED
    with pytest.raises(mg.MgpuError, match="overlapping y"):
        mg.GemvChain(dev, [(x, W, y, 64, 2048), (x, W, y, 64, 2048)])
    with pytest.raises(mg.MgpuError, match="without being a view"):
        big = dev.empty(4096, mg.F32)
        mg.GemvChain(dev, [(x, W, big.view(0, 64 * 4).set_format(mg.F32), 64, 2048),
                           (big.view(32 * 4, 2048 * 4).set_format(mg.F32), W, y, 64, 2048)])
    with pytest.raises(mg.MgpuError, match="W type"):
        W8 = dev.array(O.quantize(O.normal(64 * 2048, 1, 0.02), O.Q8_0), O.Q8_0, mg.LAYOUT_NK)
        mg.GemvChain(dev, [(x, W, y, 64, 2048), (x, W8, dev.empty(64, mg.F32), 64, 2048)])
    with pytest.raises(mg.MgpuError, match="input x"):
        x2 = dev.array(O.normal(2048, 4, 1.0), mg.F32)
        mg.GemvChain(dev, [(x, W, y, 64, 2048), (x2, W, x.view(0, 256).set_format(mg.F32), 64, 2048)])
    dev.finish()
