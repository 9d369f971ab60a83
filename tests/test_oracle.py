"""Pins the CPU oracle (oracle/) before it is trusted as the checker of the CUDA path.

- against the reference's own gemm.cl (compiled unmodified under oracle/ref_shim) and its
  committed outputs (tests/golden/ref_gemmcl.npz): bit-exact;
- against gguf-py 0.19.0's Q4_0/Q8_0 quantiser and dequantiser (tests/golden/gguf_quants.npz):
  bit-exact;
- against the reference's ggml type table (src/models/gguf_loader.cpp:13-55, as pinned by
  tests/test_gguf.cpp:16-34 of the reference) and hand-made known-answer blocks.
"""
import os

import numpy as np
import pytest

import oracle as O

GOLD = os.path.join(os.path.dirname(__file__), "golden")


def test_type_table_matches_reference_tests():
    # reference tests/test_gguf.cpp:16-34
    assert O.type_size(O.F32) == 4 and O.type_size(O.F16) == 2
    assert O.type_size(O.Q4_0) == 18 and O.type_size(O.Q8_0) == 34
    assert O.lib().ora_block_size(O.Q4_0) == 32 and O.lib().ora_block_size(O.Q8_0) == 32
    R = O.ref_gguf()
    if R is None:
        pytest.skip("reference gguf_loader not built")
    for t in (O.F32, O.F16, O.Q4_0, O.Q8_0):
        assert R.ref_ggml_type_size(t) == O.type_size(t)
        assert R.ref_ggml_type_block_size(t) == O.lib().ora_block_size(t)


def test_gemm_cl_golden_bit_exact():
    g = np.load(os.path.join(GOLD, "ref_gemmcl.npz"))
    for i, (M, N, K) in enumerate(g["gemm_cases"]):
        C = O.gemm_naive_f16(g[f"gemm{i}_A"], g[f"gemm{i}_B"], int(M), int(N), int(K))
        for fn in ("ref_gemm_naive", "ref_gemm_tiled", "ref_gemm_image"):
            np.testing.assert_array_equal(C, g[f"gemm{i}_{fn}"], err_msg=f"case {i} {fn}")
    for i, (N, K) in enumerate(g["gemv_cases"]):
        y = O.gemv_f16(g[f"gemv{i}_x"], g[f"gemv{i}_W"], int(N), int(K))
        np.testing.assert_array_equal(y, g[f"gemv{i}_y"], err_msg=f"gemv case {i}")


@pytest.mark.parametrize("M,N,K", [(5, 9, 3), (20, 13, 77), (33, 31, 260)])
def test_gemm_cl_live_bit_exact(M, N, K):
    R = O.ref()
    if R is None:
        pytest.skip("reference gemm.cl shim not built")
    A = O.f16(O.uniform(M * K, 11 + M))
    B = O.f16(O.uniform(K * N, 12 + N))
    C0 = O.gemm_naive_f16(A, B, M, N, K)
    for fn in ("ref_gemm_naive", "ref_gemm_tiled", "ref_gemm_image"):
        C = np.zeros(M * N, np.uint16)
        getattr(R, fn)(O._p(A), O._p(B), O._p(C), M, N, K)
        np.testing.assert_array_equal(C, C0)
    x = O.f16(O.uniform(K, 13))
    y = np.zeros(N, np.uint16)
    R.ref_gemv(O._p(x), O._p(B), O._p(y), N, K)
    np.testing.assert_array_equal(y, O.gemv_f16(x, B, N, K))


def test_gemv_f32_is_gemv_f16_order():
    # the fp32 config path uses the same reduction order as gemv (gemm.cl:219-270)
    N, K = 9, 700
    x = O.uniform(K, 21)
    W = O.uniform(K * N, 22)
    y = O.gemv_f32(x, W, N, K)
    part = np.zeros((256, N), np.float32)
    for lid in range(256):
        acc = np.zeros(N, np.float32)
        for k in range(lid, K, 256):
            acc = (np.float64(x[k]) * W[k * N:(k + 1) * N] + acc).astype(np.float32)  # fma: exact product
        part[lid] = acc
    s = 128
    while s:
        part[:s] = part[:s] + part[s:2 * s]
        s >>= 1
    np.testing.assert_array_equal(y, part[0])


def test_quant_golden_bit_exact():
    g = np.load(os.path.join(GOLD, "gguf_quants.npz"))
    x = g["x"]
    for name, t in (("q4_0", O.Q4_0), ("q8_0", O.Q8_0)):
        q = O.quantize(x, t)
        np.testing.assert_array_equal(q, g[name], err_msg=name)
        d = O.dequant(g[name], x.size, t)
        np.testing.assert_array_equal(d.view(np.uint32), g[name + "_deq"].view(np.uint32), err_msg=name)


def test_quant_live_against_gguf():
    gguf = pytest.importorskip("gguf")
    x = O.normal(32 * 512, 99, 0.02)
    for t, qt in ((O.Q4_0, gguf.GGMLQuantizationType.Q4_0), (O.Q8_0, gguf.GGMLQuantizationType.Q8_0)):
        q = O.quantize(x, t)
        np.testing.assert_array_equal(q, gguf.quants.quantize(x.reshape(1, -1), qt).reshape(-1))


def _q4_block(d_bits: int, nibbles) -> np.ndarray:
    b = np.zeros(18, np.uint8)
    b[0], b[1] = d_bits & 0xFF, d_bits >> 8
    for j in range(16):
        b[2 + j] = (nibbles[j] & 0xF) | ((nibbles[j + 16] & 0xF) << 4)
    return b


def test_dequant_known_answers():
    one, mhalf, zero, sub, fmax = 0x3C00, 0xB800, 0x0000, 0x0001, 0x7BFF
    nib = list(range(16)) + list(range(15, -1, -1))
    exp = np.array([n - 8 for n in nib], np.float32)
    np.testing.assert_array_equal(O.dequant(_q4_block(one, nib), 32, O.Q4_0), exp)
    np.testing.assert_array_equal(O.dequant(_q4_block(mhalf, nib), 32, O.Q4_0), exp * np.float32(-0.5))
    np.testing.assert_array_equal(O.dequant(_q4_block(zero, nib), 32, O.Q4_0), np.zeros(32, np.float32) * exp)
    np.testing.assert_array_equal(O.dequant(_q4_block(sub, nib), 32, O.Q4_0), exp * np.float32(2.0 ** -24))
    assert O.dequant(_q4_block(fmax, [0] * 32), 32, O.Q4_0)[0] == np.float32(-524032.0)
    q8 = np.zeros(34 * 8, np.uint8)
    vals = np.arange(-128, 128, dtype=np.int32)
    for b in range(8):
        q8[34 * b], q8[34 * b + 1] = one & 0xFF, one >> 8
        q8[34 * b + 2: 34 * b + 34] = vals[32 * b: 32 * b + 32].astype(np.int8).view(np.uint8)
    np.testing.assert_array_equal(O.dequant(q8, 256, O.Q8_0), vals.astype(np.float32))


def test_f16_bf16_conversions_match_numpy():
    x = np.concatenate([O.normal(4096, 5, 3.0), np.array([65504, 65520, 1e-8, -0.0, 6.1e-5, 2.0 ** -25,
                                                          3 * 2.0 ** -26], np.float32)])
    np.testing.assert_array_equal(O.f16(x), x.astype(np.float16).view(np.uint16))
    h = np.arange(0, 65536, dtype=np.uint32).astype(np.uint16)
    finite = (h & 0x7C00) != 0x7C00
    np.testing.assert_array_equal(O.f16_to_f32(h)[finite], h.view(np.float16).astype(np.float32)[finite])
    # bf16 RNE: compare with the float64 nearest of the two candidates
    x = x[np.abs(x) > 1e-30]
    b = O.bf16(x)
    back = O.bf16_to_f32(b).astype(np.float64)
    up = O.bf16_to_f32(b + np.uint16(1)).astype(np.float64)
    dn = O.bf16_to_f32(b - np.uint16(1)).astype(np.float64)
    err = np.abs(back - x)
    assert np.all(err <= np.abs(up - x)) and np.all(err <= np.abs(dn - x))


def test_gemm_kats():
    M = N = K = 8
    eye = O.f16(np.eye(K, dtype=np.float32).reshape(-1))
    A = O.f16(O.uniform(M * K, 7))
    np.testing.assert_array_equal(O.gemm_naive_f16(A, eye, M, N, K), A)          # identity B
    onehot = np.zeros(M * K, np.float32)
    onehot[3 * K + 5] = 1.0
    B = O.f16(O.uniform(K * N, 8))
    C = O.gemm_naive_f16(O.f16(onehot), B, M, N, K).reshape(M, N)
    np.testing.assert_array_equal(C[3], B.reshape(K, N)[5])                       # one-hot row
    assert not C[np.arange(M) != 3].any()
    c1 = O.gemm_naive_f32(np.array([3.0], np.float32), np.array([0.5, -2.0], np.float32), 1, 2, 1)
    np.testing.assert_array_equal(c1, np.array([1.5, -6.0], np.float32))        # K = 1


def test_gemm_q_equals_dequant_then_naive():
    M, N, K = 3, 5, 96
    A = O.uniform(M * K, 31)
    Wf = O.normal(N * K, 32, 0.02)
    for t in (O.Q4_0, O.Q8_0):
        W = O.quantize(Wf, t)
        C = O.gemm_q(A, W, M, N, K, t)
        Wd = O.dequant(W, N * K, t).reshape(N, K)
        C2 = O.gemm_naive_f32(A, np.ascontiguousarray(Wd.T).reshape(-1), M, N, K)
        np.testing.assert_array_equal(C, C2)
        np.testing.assert_array_equal(O.gemm_q(A, W, M, N, K, t, threads=True), C)


def test_im2col_order():
    C, H, W, ph, pw = 3, 28, 42, 14, 14
    img = O.uniform(C * H * W, 41)
    p = O.im2col(img, C, H, W, ph, pw).reshape(-1, C * ph * pw)
    im = img.reshape(C, H, W)
    for idx in range(p.shape[0]):
        r, c = divmod(idx, W // pw)
        np.testing.assert_array_equal(p[idx], im[:, r * ph:(r + 1) * ph, c * pw:(c + 1) * pw].reshape(-1))


def test_argmax_logits_known_answers():
    # the reference's host scan (moondream2.cpp:551-591) on fp16 logits: subnormal -> 0,
    # Inf/NaN -> +-1e30 by sign, strictly greater replaces, so the first maximum wins
    h = lambda *v: np.array(v, np.uint16)
    assert O.argmax_logits(h(0xFC00, 0x3C00, 0x7E00, 0x4000), O.F16)[0] == 2      # NaN reads +1e30
    assert O.argmax_logits(h(0xBC00, 0x0001, 0xB800), O.F16)[0] == 1              # subnormal reads 0
    assert O.argmax_logits(h(0x3C00, 0x4000, 0x4000), O.F16)[0] == 1              # first of a tie
    assert O.argmax_logits(h(0xFC00, 0xFC00), O.F16) == (0, float(np.float32(-1e30)))  # nothing above -1e30
    assert O.argmax_logits(h(0xFBFF, 0x7C00, 0x7BFF), O.F16)[0] == 1              # +Inf reads 1e30
    f = np.array([-2.0, np.float32(1e-40), -1.0, 3.0, 3.0], np.float32)
    assert O.argmax_logits(f.view(np.uint32), O.F32)[0] == 3


def test_activation_restatement():
    # activations.cl:78-117 computes tanh as 1 - 2 / (1 + exp(-2a)) = -tanh(a), so the shipped
    # gelu is x - gelu(x) where gelu is the tanh form compute.h:48 states
    x = np.linspace(-12, 12, 4001).astype(np.float32)
    g, shipped, silu = O.activate(x, 1), O.activate(x, 3), O.activate(x, 2)
    assert np.max(np.abs(shipped - (x - g))) <= 2e-6 * np.max(np.abs(x))
    assert abs(float(O.activate(np.float32([1.0]), 1)[0]) - 0.8411920) < 1e-6
    assert abs(float(O.activate(np.float32([1.0]), 2)[0]) - 0.7310586) < 1e-6
    assert np.all(np.isfinite(O.activate(np.float32([-1e30, 1e30, -100, 100]), 1)))
    # silu = x * sigmoid(x): 0 at 0, -> x for large x, -> 0 for very negative x
    assert silu[2000] == 0.0 and abs(silu[-1] - 12) < 1e-4 and abs(silu[0]) < 1e-4


def test_unfused_epilogue_rounds_after_each_kernel():
    M, N = 3, 5
    acc = O.normal(M * N, 1, 3.0)
    bias = O.normal(N, 2, 1.0)
    resid = O.f16_to_f32(O.f16(O.normal(M * N, 3, 1.0)))
    c = O.f16_to_f32(O.f16(acc.reshape(M, N) + bias)).reshape(-1)
    c = O.f16_to_f32(O.f16(O.activate(c, 2)))
    want = O.f16_to_f32(O.f16(c + resid))
    assert np.array_equal(O.unfused_epilogue(acc, bias, 2, resid, M, N, 1), want)


def test_silu_gate_restatement():
    g = np.float32([-3.0, 0.0, 1.0, 2.5])
    u = np.float32([2.0, 5.0, -1.0, 0.5])
    want = O.round_to(O.activate(g, 2) * u, 1)
    assert np.allclose(O.unfused_silu_gate(g, u, 1), want, rtol=1e-3, atol=0)


def test_rms_norm_restatement_matches_float64():
    # layernorm.cl's rms_norm: x * rsqrt(mean(x^2) + eps) * w, fp32 arithmetic; checked against
    # the same formula in float64 (fp32 output, so only fp32 rounding separates them)
    rows, H, eps = 3, 1000, 1e-5
    x = O.normal(rows * H, 8, 2.0)
    w = O.normal(H, 9, 0.5)
    got = O.rms_norm(x, w, rows, H, eps, O.F32).reshape(rows, H)
    xd = x.astype(np.float64).reshape(rows, H)
    ref = xd / np.sqrt(np.mean(xd * xd, axis=1, keepdims=True) + eps) * w.astype(np.float64)
    assert np.max(np.abs(got - ref)) <= 1e-5 * np.max(np.abs(ref))
