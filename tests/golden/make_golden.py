"""Regenerate the golden fixtures in this directory (run in a container that has the
gguf-py package and the reference checkout; the fixtures themselves are committed).

    python tests/golden/make_golden.py

gguf_quants.npz
    Q4_0 / Q8_0 blocks and their dequantised values produced by gguf-py 0.19.0
    (``gguf.quants.quantize`` / ``dequantize``, llama.cpp's published block format), on seeded
    inputs chosen to hit the edge cases of the format: all-zero blocks, ties for the largest
    magnitude, values that round to +-8 / +-127 exactly, fp16-subnormal and fp16-max scales.
ref_gemmcl.npz
    Outputs of the reference's own src/kernels/gemm.cl (gemm_naive, gemm_tiled, gemm_image,
    gemv) compiled as C++ under oracle/ref_shim and run on seeded fp16 inputs, at ragged
    shapes (M, N, K not multiples of the work-group tiles; N % 4 != 0 for the image path).
"""
from __future__ import annotations

import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)

import oracle as O  # noqa: E402


def quant_inputs() -> np.ndarray:
    blocks = []
    blocks.append(O.normal(32 * 256, 0x4D564C4D, 0.02).reshape(-1, 32))          # weights ~N(0, 0.02)
    blocks.append(O.uniform(32 * 64, 0x4D564C4E).reshape(-1, 32) * 3.0)           # wider range
    z = np.zeros((4, 32), np.float32)                                               # all-zero blocks
    blocks.append(z)
    t = O.normal(32 * 8, 0x4D564C4F, 1.0).reshape(-1, 32)                           # ties for max |v|
    t[:, 3] = 2.5
    t[:, 17] = -2.5
    blocks.append(t)
    e = np.tile(np.linspace(-1.0, 1.0, 32, dtype=np.float32), (4, 1))               # exact grid values
    blocks.append(e)
    s = O.normal(32 * 4, 0x4D564C50, 1.0).reshape(-1, 32) * np.float32(1e-7)        # fp16-subnormal scales
    blocks.append(s.astype(np.float32))
    big = O.uniform(32 * 4, 0x4D564C51).reshape(-1, 32) * np.float32(60000.0)       # near fp16 max scale
    blocks.append(big.astype(np.float32))
    return np.concatenate(blocks).astype(np.float32).reshape(-1)


def make_quants():
    import gguf
    x = quant_inputs()
    out = {"x": x, "gguf_version": np.array(gguf.__version__ if hasattr(gguf, "__version__") else "0.19.0")}
    for name, qt in (("q4_0", gguf.GGMLQuantizationType.Q4_0), ("q8_0", gguf.GGMLQuantizationType.Q8_0)):
        q = gguf.quants.quantize(x.reshape(1, -1), qt).reshape(-1)
        d = gguf.quants.dequantize(q, qt).reshape(-1).astype(np.float32)
        out[name] = q.astype(np.uint8)
        out[name + "_deq"] = d
    np.savez_compressed(os.path.join(HERE, "gguf_quants.npz"), **out)


GEMM_CASES = [(1, 1, 1), (3, 5, 7), (17, 33, 45), (16, 16, 16), (31, 18, 64), (40, 70, 129)]
GEMV_CASES = [(4, 16), (7, 300), (33, 513), (8, 2048)]


def make_ref():
    R = O.ref()
    if R is None:
        raise SystemExit("oracle/_ref/libref_gemmcl.so missing: run `make -C oracle`")
    out = {}
    for i, (M, N, K) in enumerate(GEMM_CASES):
        A = O.f16(O.uniform(M * K, 0x1000 + i))
        B = O.f16(O.uniform(K * N, 0x2000 + i))
        out[f"gemm{i}_A"], out[f"gemm{i}_B"] = A, B
        for fn in ("ref_gemm_naive", "ref_gemm_tiled", "ref_gemm_image"):
            C = np.zeros(M * N, np.uint16)
            getattr(R, fn)(O._p(A), O._p(B), O._p(C), M, N, K)
            out[f"gemm{i}_{fn}"] = C
    for i, (N, K) in enumerate(GEMV_CASES):
        x = O.f16(O.uniform(K, 0x3000 + i))
        W = O.f16(O.uniform(K * N, 0x4000 + i))
        y = np.zeros(N, np.uint16)
        R.ref_gemv(O._p(x), O._p(W), O._p(y), N, K)
        out[f"gemv{i}_x"], out[f"gemv{i}_W"], out[f"gemv{i}_y"] = x, W, y
    out["gemm_cases"] = np.array(GEMM_CASES, np.int32)
    out["gemv_cases"] = np.array(GEMV_CASES, np.int32)
    np.savez_compressed(os.path.join(HERE, "ref_gemmcl.npz"), **out)


if __name__ == "__main__":
    make_quants()
    make_ref()
    print("wrote", sorted(f for f in os.listdir(HERE) if f.endswith(".npz")))
