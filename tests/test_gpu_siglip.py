"""GPU parity of the SigLIP encoder GEMMs at the batch sizes the benchmark times (BASELINE
config 3: B = 8 and 64 images, M = 729 B tokens), with fp16 activations and fp16 weights in
GGUF [N][K] order, fp16 output: the planner's large-M choices (CTA pairs, several waves, ragged
N = 4304) are compared with the CPU oracle on rows sampled across the output, tile boundaries
included.  New call sites of the same GEMM entry point: the reference's vision layers are
pass-through copies (src/kernels/vision.cl:293-390)."""
import numpy as np
import pytest

import mvlm_b200 as mg
import oracle as O
from tests.numerics import TOL_16, assert_close

pytestmark = pytest.mark.gpu

SHAPES = [(1152, 3456), (1152, 1152), (1152, 4304), (4304, 1152), (2304, 8192), (8192, 2048)]  # (K, N)


@pytest.mark.parametrize("B", [8, 64])
@pytest.mark.parametrize("K,N", SHAPES)
def test_siglip_batched_gguf_nk(dev, B, K, N):
    M = 729 * B
    A = dev.create_buffer(M * K * 2, None, mg.F16)
    dev.fill_normal(A, M * K, 0x5EED + K + B, 1.0)
    W = dev.create_buffer(N * K * 2, None, mg.F16, mg.LAYOUT_NK, N, K)
    dev.fill_normal(W, N * K, 0x5EED + N, 0.02)
    C = dev.empty(M * N, mg.F16)
    mg.gemm(dev, A, W, C, M, N, K).wait()
    rows = sorted({0, 1, 127, 128, 255, 256, 511, 729, M // 3, M // 2, M - 257, M - 129, M - 2, M - 1}
                  | set(range(5, M, max(1, M // 24))))
    Ah = np.concatenate([O.f16_to_f32(A.read(np.uint16, K, 2 * r * K)) for r in rows])
    got = np.concatenate([O.f16_to_f32(C.read(np.uint16, N, 2 * r * N)) for r in rows])
    ref = O.gemm_nk(Ah, W.read(np.uint16), mg.F16, len(rows), N, K, threads=True)
    assert_close(got, ref, TOL_16, f"SigLIP B={B} {K}x{N}")
