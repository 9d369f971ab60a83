"""GPU parity of the GGUF weight upload chain (moondream2.cpp:62-84, gguf_loader.cpp:360-362):
a GGUF file written with Q4_0 / Q8_0 tensors (the structure of the reference's test fixture
builder, tests/test_utils.h:16-97) is read by the reference's own loader (oracle/_ref, built
from src/models/gguf_loader.cpp), its TensorInfo and bytes go through mgpu_upload_weight, and the
uploaded weight feeds the kernels through the reference's dispatch names.  Checked: the device
copy is the file's bytes, the device dequantisation is bit-exact with the oracle's, the decode
GEMV and the prefill GEMM match the oracle's dequantise + fp32 matmul."""
import ctypes

import numpy as np
import pytest

import mvlm_b200 as mg
import oracle as O
from tests.gguf_writer import write_gguf
from tests.numerics import TOL_16, TOL_F32, assert_close

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("qt", [O.Q4_0, O.Q8_0])
def test_gguf_file_to_kernels(dev, tmp_path, qt):
    R = O.ref_gguf()
    if R is None:
        pytest.skip("the reference loader (oracle/_ref/libref_gguf.so) was not built")
    K, N, N2 = 2048, 3000, 2048
    q_up = O.quantize(O.normal(N * K, 11 + qt, 0.02), qt)
    q_out = O.quantize(O.normal(N2 * K, 12 + qt, 0.02), qt)
    path = str(tmp_path / "model.gguf")
    write_gguf(path, [("blk.0.ffn_up.weight", [K, N], qt, q_up), ("blk.0.attn_output.weight", [K, N2], qt, q_out)],
               {"general.alignment": 32})
    for name, q, n in ((b"blk.0.ffn_up.weight", q_up, N), (b"blk.0.attn_output.weight", q_out, N2)):
        info = mg.TensorInfo()
        raw = np.zeros(q.size, np.uint8)
        got = R.ref_gguf_read_tensor(path.encode(), name, ctypes.byref(info), raw.ctypes.data, raw.size)
        assert got == q.size and info.dims[0] == K and info.dims[1] == n and info.type == qt
        W = dev.upload_weight(info, raw)
        # the packed blocks arrive unchanged
        assert np.array_equal(W.read(np.uint8)[: q.size], q)
        # the device dequantisation is the oracle's, bit for bit
        deq = dev.empty(n * K, mg.F32)
        mg.dequant(dev, W, deq, n * K, qt).wait()
        assert np.array_equal(deq.read(np.float32), O.dequant(q, n * K, qt))
        # decode: the reference's dispatch_gemv on the uploaded weight
        x = O.normal(K, 13, 1.0)
        y = dev.empty(n, mg.F32)
        mg.dispatch_gemv(dev, None, dev.array(x, mg.F32), W, y, n, K).wait()
        assert_close(y.read(np.float32), O.gemm_q(x, q, 1, n, K, qt, threads=True), TOL_F32, f"gemv {name}")
        # prefill: the reference's dispatch_gemm_image on the same weight, bf16 activations
        M = 761
        A = O.bf16(O.normal(M * K, 14, 1.0))
        C = dev.empty(M * n, mg.F32)
        mg.dispatch_gemm_image(dev, None, dev.array(A, mg.BF16), W, C, M, n, K).wait()
        ref = O.gemm_q(O.bf16_to_f32(A), q, M, n, K, qt, threads=True)
        assert_close(C.read(np.float32), ref, TOL_16, f"gemm {name}")
