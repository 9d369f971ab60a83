"""GPU parity of the standalone block decoders, the device quantiser and the generators;
bounded-wait failure detection; CUDA-graph replay."""
import numpy as np
import pytest

import mvlm_b200 as mg
import oracle as O
from tests.numerics import TOL_F32, assert_close

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("qt", [O.Q4_0, O.Q8_0])
def test_dequant_bit_exact(dev, qt):
    g = np.load("tests/golden/gguf_quants.npz")
    name = "q4_0" if qt == O.Q4_0 else "q8_0"
    n = g["x"].size
    out = dev.empty(n, mg.F32)
    mg.dequant(dev, dev.array(g[name], qt, mg.LAYOUT_NK), out, n, qt).wait()
    np.testing.assert_array_equal(out.read(np.float32).view(np.uint32), g[name + "_deq"].view(np.uint32))
    for ot, conv in ((mg.F16, O.f16), (mg.BF16, O.bf16)):
        o16 = dev.empty(n, ot)
        mg.dequant(dev, dev.array(g[name], qt, mg.LAYOUT_NK), o16, n, qt).wait()
        np.testing.assert_array_equal(o16.read(np.uint16), conv(g[name + "_deq"]))


@pytest.mark.parametrize("qt", [O.Q4_0, O.Q8_0])
def test_device_quantiser_bit_exact(dev, qt):
    g = np.load("tests/golden/gguf_quants.npz")
    x = g["x"]
    name = "q4_0" if qt == O.Q4_0 else "q8_0"
    dst = dev.create_buffer(x.size // 32 * mg.BLOCK_BYTES[qt], None)
    dev.quantize(dev.array(x, mg.F32), dst, x.size, qt)
    np.testing.assert_array_equal(dst.read(np.uint8), g[name])


def test_generators_deterministic(dev):
    n = 1 << 16
    a, b = dev.empty(n, mg.F32), dev.empty(n, mg.F32)
    dev.fill_normal(a, n, 1234, 0.02)
    dev.fill_normal(b, n, 1234, 0.02)
    va, vb = a.read(np.float32), b.read(np.float32)
    np.testing.assert_array_equal(va, vb)
    assert abs(va.std() - 0.02) < 0.001 and abs(va.mean()) < 0.001
    dev.fill_uniform(a, n, 99, -1.0, 1.0)
    u = a.read(np.float32)
    assert u.min() >= -1.0 and u.max() < 1.0 and abs(u.mean()) < 0.02


def test_bounded_wait_reports_timeout_and_device_recovers(dev):
    dev.finish()
    dev.selftest_bounded_wait(2_000_000)  # 2 ms limit on a barrier nobody arrives on
    with pytest.raises(mg.MgpuError) as e:
        dev.finish()
    assert e.value.code == mg.ERR_DEVICE_TIMEOUT
    dev.finish()  # status was consumed; the context is still usable
    K, N = 256, 8
    x = O.uniform(K, 1)
    W = O.quantize(O.normal(N * K, 2, 0.02), O.Q4_0)
    y = dev.empty(N, mg.F32)
    mg.gemv_q(dev, dev.array(x, mg.F32), dev.array(W, mg.Q4_0, mg.LAYOUT_NK), y, N, K, mg.Q4_0).wait()
    assert_close(y.read(np.float32), O.gemm_q(x, W, 1, N, K, O.Q4_0), TOL_F32)


def test_graph_capture_replays_gemv(dev):
    K, N = 2048, 6144
    x = O.normal(K, 5, 1.0)
    W = O.quantize(O.normal(N * K, 6, 0.02), O.Q4_0)
    dx, dW, dy = dev.array(x, mg.F32), dev.array(W, mg.Q4_0, mg.LAYOUT_NK), dev.empty(N, mg.F32)
    mg.gemv_q(dev, dx, dW, dy, N, K, mg.Q4_0).wait()
    first = dy.read(np.float32)
    dev.capture_begin()
    mg.gemv_q(dev, dx, dW, dy, N, K, mg.Q4_0)
    g = dev.capture_end()
    x2 = O.normal(K, 7, 1.0)
    dx.write(x2)
    g.launch()
    dev.finish()
    assert_close(dy.read(np.float32), O.gemm_q(x2, W, 1, N, K, O.Q4_0, threads=True), TOL_F32)
    assert not np.array_equal(first, dy.read(np.float32))


@pytest.mark.parametrize("t", [mg.F16, mg.BF16, mg.F32])
def test_argmax_logits_matches_reference_scan(dev, t):
    # greedy decode over an lm_head's logits (vocab 51200): random values plus a repeated
    # maximum, subnormals, infinities and NaN, against the oracle of the reference's host scan
    n = 51200
    x = O.normal(n, 77, 4.0)
    x[[1000, 40000]] = 30.0  # the first of the tied maxima wins
    if t == mg.F16:
        raw = O.f16(x)
        raw[[7, 50000]] = [0x0003, 0x8002]      # subnormals read as 0
        raw[123] = 0xFC00                       # -Inf reads -1e30
    elif t == mg.BF16:
        raw = O.bf16(x)
        raw[123] = 0xFF80
    else:
        raw = x.view(np.uint32).copy()
        raw[123] = 0xFF800000
    buf = dev.array(raw, t)
    out = dev.empty(2, mg.F32)
    for _ in range(2):
        assert mg.argmax_logits(dev, buf, n) == O.argmax_logits(raw, t)[0] == 1000
        mg.argmax(dev, buf, n, out).wait()
        got = out.read(np.int32)
        assert got[0] == 1000 and np.float32(got[1:2].view(np.float32)[0]) == np.float32(O.argmax_logits(raw, t)[1])
    # a NaN with a clear sign bit reads +1e30 and wins
    raw2 = raw.copy()
    raw2[9] = {mg.F16: 0x7E00, mg.BF16: 0x7FC0, mg.F32: 0x7FC00000}[t]
    assert mg.argmax_logits(dev, dev.array(raw2, t), n) == O.argmax_logits(raw2, t)[0] == 9


@pytest.mark.parametrize("ranks", [2, 3, 8])
def test_argmax_combine_column_shards(dev, ranks):
    # the lm_head's logits column-sharded over `ranks` GPUs (emulated here on one): each shard's
    # mgpu_argmax, the pairs in rank order, then mgpu_argmax_combine, against the reference's
    # scan of the whole row; with a maximum tied across shards, and with nothing above -1e30
    from mvlm_b200.shard import column_shard
    n = 51203
    for case in range(3):
        x = O.normal(n, 300 + case, 3.0)
        if case == 1:
            x[[n - 5, 17]] = 40.0  # tied in the last and first shards: index 17 wins
        if case == 2:
            x[:] = -np.inf
        raw = x.view(np.uint32).copy()
        want_i, want_v = O.argmax_logits(raw, mg.F32)
        logits = dev.array(raw, mg.F32)
        pairs = dev.empty(2 * ranks, mg.F32)
        for r in range(ranks):
            a, b = column_shard(n, ranks, r)
            mg.argmax(dev, logits.view(4 * a, 4 * (b - a)).set_format(mg.F32), b - a, pairs.view(8 * r, 8))
        out = dev.empty(2, mg.F32)
        mg.argmax_combine(dev, pairs, ranks, n, out).wait()
        got = out.read(np.int32)
        assert got[0] == want_i, (case, got[0], want_i)
        assert np.float32(got[1:2].view(np.float32)[0]) == np.float32(want_v)


@pytest.mark.parametrize("rows,n,ld", [(1, 51200, 51200), (8, 6400, 6400), (5, 1000, 1029)])
def test_argmax_rows_matches_per_row_scan(dev, rows, n, ld):
    # a batch of sequences' logits against one lm_head shard: each row's pair equals the
    # reference scan of that row; rows at a pitch ld >= n (padding never read), a tie in row 0
    x = O.normal(rows * ld, 500 + rows, 3.0).reshape(rows, ld)
    x[:, n:] = 1e6  # beyond each row's n values: must not win
    x[0, [n // 3, n - 1]] = 50.0
    raw = x.reshape(-1).view(np.uint32).copy()
    out = dev.empty(2 * rows, mg.F32)
    mg.argmax_rows(dev, dev.array(raw, mg.F32), rows, n, ld, out).wait()
    got = out.read(np.int32).reshape(rows, 2)
    for r in range(rows):
        want_i, want_v = O.argmax_logits(raw[r * ld:r * ld + n].copy(), mg.F32)
        assert got[r, 0] == want_i, (r, got[r, 0], want_i)
        assert np.float32(got[r, 1:2].view(np.float32)[0]) == np.float32(want_v)
    assert got[0, 0] == n // 3
