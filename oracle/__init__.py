"""ctypes bindings for the CPU oracle.  TEST INFRASTRUCTURE ONLY.

Loaded by tests/, ``__graft_entry__.smoke()`` and the CPU-baseline leg of ``bench.py`` as
the checker of the CUDA path.  The product package (``mvlm_b200``) never imports it.

``liboracle.so`` is the C restatement (oracle.c).  ``_ref/libref_gemmcl.so`` is the
reference's own ``src/kernels/gemm.cl`` compiled as C++ under ``ref_shim/clshim.hpp`` and
``_ref/libref_gguf.so`` is the reference's ``src/models/gguf_loader.cpp``; both are built
from the reference tree by ``oracle/Makefile`` and are optional at run time.
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
F32, F16, Q4_0, Q8_0, BF16 = 0, 1, 2, 8, 30

_lib = None
_ref = None
_ref_gguf = None


def build(quiet: bool = True) -> None:
    out = subprocess.run(["make", "-C", HERE], capture_output=True, text=True)
    if out.returncode != 0:
        raise RuntimeError("oracle build failed:\n" + out.stdout + out.stderr)
    if not quiet:
        print(out.stdout)


def _p(a: np.ndarray):
    return a.ctypes.data_as(ctypes.c_void_p)


def lib():
    global _lib
    if _lib is None:
        path = os.path.join(HERE, "liboracle.so")
        if not os.path.exists(path):
            build()
        _lib = ctypes.CDLL(path)
        L = _lib
        vp, i32, i64, u64, sz = (ctypes.c_void_p, ctypes.c_int, ctypes.c_int64, ctypes.c_uint64,
                                 ctypes.c_size_t)
        L.ora_fill_uniform.argtypes = [vp, sz, u64]
        L.ora_fill_normal.argtypes = [vp, sz, u64, ctypes.c_float]
        L.ora_quantize_q4_0.argtypes = [vp, vp, i64]
        L.ora_quantize_q8_0.argtypes = [vp, vp, i64]
        L.ora_dequant.argtypes = [vp, vp, i64, i32]
        for n in ("ora_gemm_naive_f16", "ora_gemm_naive_f32", "ora_gemm_naive_f32_mt"):
            getattr(L, n).argtypes = [vp, vp, vp, i32, i32, i32]
        for n in ("ora_gemv_f16", "ora_gemv_f32", "ora_gemv_f32_kn_mt"):
            getattr(L, n).argtypes = [vp, vp, vp, i32, i32]
        for n in ("ora_gemm_q", "ora_gemm_q_mt"):
            getattr(L, n).argtypes = [vp, vp, vp, i32, i32, i32, i32]
        L.ora_gemv_q_mt.argtypes = [vp, vp, vp, i32, i32, i32]
        for n in ("ora_gemm_nk", "ora_gemm_nk_mt"):
            getattr(L, n).argtypes = [vp, vp, i32, vp, i32, i32, i32]
        L.ora_add_bias.argtypes = [vp, vp, i32, i32]
        L.ora_im2col.argtypes = [vp, vp, i32, i32, i32, i32, i32]
        L.ora_activate.argtypes = [ctypes.c_float, i32]
        L.ora_activate.restype = ctypes.c_float
        L.ora_activate_n.argtypes = [vp, sz, i32]
        L.ora_silu_gate_n.argtypes = [vp, vp, vp, sz]
        L.ora_rms_norm.argtypes = [vp, vp, vp, ctypes.c_int, ctypes.c_int, ctypes.c_float]
        for n in ("ora_f32_to_f16_n", "ora_f16_to_f32_n", "ora_f32_to_bf16_n", "ora_bf16_to_f32_n"):
            getattr(L, n).argtypes = [vp, vp, sz]
        L.ora_type_size.argtypes = [i32]
        L.ora_type_size.restype = sz
        L.ora_block_size.argtypes = [i32]
        L.ora_row_bytes.argtypes = [i32, i64]
        L.ora_row_bytes.restype = sz
        L.ora_max_threads.restype = i32
        L.ora_set_threads.argtypes = [i32]
    return _lib


def ref():
    """The reference's gemm.cl under the host shim, or None when it was not built."""
    global _ref
    if _ref is None:
        path = os.path.join(HERE, "_ref", "libref_gemmcl.so")
        if not os.path.exists(path):
            return None
        _ref = ctypes.CDLL(path)
        vp, i32 = ctypes.c_void_p, ctypes.c_int
        for n in ("ref_gemm_naive", "ref_gemm_tiled", "ref_gemm_image"):
            getattr(_ref, n).argtypes = [vp, vp, vp, i32, i32, i32]
        _ref.ref_gemv.argtypes = [vp, vp, vp, i32, i32]
    return _ref


def ref_gguf():
    """The reference's gguf_loader.cpp, or None when it was not built."""
    global _ref_gguf
    if _ref_gguf is None:
        path = os.path.join(HERE, "_ref", "libref_gguf.so")
        if not os.path.exists(path):
            return None
        _ref_gguf = ctypes.CDLL(path)
        R = _ref_gguf
        R.ref_ggml_type_size.argtypes = [ctypes.c_uint32]
        R.ref_ggml_type_size.restype = ctypes.c_size_t
        R.ref_ggml_type_block_size.argtypes = [ctypes.c_uint32]
        R.ref_tensor_info_size.restype = ctypes.c_size_t
        R.ref_gguf_read_tensor.argtypes = [ctypes.c_char_p, ctypes.c_char_p, ctypes.c_void_p,
                                           ctypes.c_void_p, ctypes.c_size_t]
        R.ref_gguf_read_tensor.restype = ctypes.c_longlong
    return _ref_gguf


# ---------------------------------------------------------------------------------------
# numpy-facing helpers
# ---------------------------------------------------------------------------------------
def uniform(n: int, seed: int) -> np.ndarray:
    out = np.empty(n, np.float32)
    lib().ora_fill_uniform(_p(out), n, seed)
    return out


def normal(n: int, seed: int, sigma: float = 1.0) -> np.ndarray:
    out = np.empty(n, np.float32)
    lib().ora_fill_normal(_p(out), n, seed, sigma)
    return out


def type_size(t: int) -> int:
    return lib().ora_type_size(t)


def row_bytes(t: int, k: int) -> int:
    return lib().ora_row_bytes(t, k)


def quantize(x: np.ndarray, t: int) -> np.ndarray:
    x = np.ascontiguousarray(x, np.float32)
    assert x.size % 32 == 0
    out = np.empty(x.size // 32 * type_size(t), np.uint8)
    fn = lib().ora_quantize_q4_0 if t == Q4_0 else lib().ora_quantize_q8_0
    fn(_p(x), _p(out), x.size)
    return out


def dequant(blocks: np.ndarray, n: int, t: int) -> np.ndarray:
    blocks = np.ascontiguousarray(blocks, np.uint8)
    out = np.empty(n, np.float32)
    lib().ora_dequant(_p(blocks), _p(out), n, t)
    return out


def f16(x: np.ndarray) -> np.ndarray:
    x = np.ascontiguousarray(x, np.float32)
    out = np.empty(x.shape, np.uint16)
    lib().ora_f32_to_f16_n(_p(x), _p(out), x.size)
    return out


def f16_to_f32(h: np.ndarray) -> np.ndarray:
    h = np.ascontiguousarray(h, np.uint16)
    out = np.empty(h.shape, np.float32)
    lib().ora_f16_to_f32_n(_p(h), _p(out), h.size)
    return out


def bf16(x: np.ndarray) -> np.ndarray:
    x = np.ascontiguousarray(x, np.float32)
    out = np.empty(x.shape, np.uint16)
    lib().ora_f32_to_bf16_n(_p(x), _p(out), x.size)
    return out


def bf16_to_f32(h: np.ndarray) -> np.ndarray:
    h = np.ascontiguousarray(h, np.uint16)
    out = np.empty(h.shape, np.float32)
    lib().ora_bf16_to_f32_n(_p(h), _p(out), h.size)
    return out


def gemm_naive_f16(A: np.ndarray, B: np.ndarray, M: int, N: int, K: int) -> np.ndarray:
    C = np.empty(M * N, np.uint16)
    lib().ora_gemm_naive_f16(_p(np.ascontiguousarray(A)), _p(np.ascontiguousarray(B)), _p(C), M, N, K)
    return C


def gemm_naive_f32(A, B, M, N, K, threads: bool = False):
    C = np.empty(M * N, np.float32)
    fn = lib().ora_gemm_naive_f32_mt if threads else lib().ora_gemm_naive_f32
    fn(_p(np.ascontiguousarray(A, np.float32)),
                             _p(np.ascontiguousarray(B, np.float32)), _p(C), M, N, K)
    return C


def gemv_f16(x, W, N, K):
    y = np.empty(N, np.uint16)
    lib().ora_gemv_f16(_p(np.ascontiguousarray(x)), _p(np.ascontiguousarray(W)), _p(y), N, K)
    return y


def gemv_f32(x, W, N, K):
    y = np.empty(N, np.float32)
    lib().ora_gemv_f32(_p(np.ascontiguousarray(x, np.float32)), _p(np.ascontiguousarray(W, np.float32)),
                       _p(y), N, K)
    return y


def gemm_q(A, W, M, N, K, t, threads: bool = False):
    C = np.empty(M * N, np.float32)
    fn = lib().ora_gemm_q_mt if threads else lib().ora_gemm_q
    fn(_p(np.ascontiguousarray(A, np.float32)), _p(np.ascontiguousarray(W, np.uint8)), _p(C), M, N, K, t)
    return C


def gemm_nk(A, W, wtype, M, N, K, threads: bool = False):
    C = np.empty(M * N, np.float32)
    fn = lib().ora_gemm_nk_mt if threads else lib().ora_gemm_nk
    fn(_p(np.ascontiguousarray(A, np.float32)), _p(np.ascontiguousarray(W)), wtype, _p(C), M, N, K)
    return C


def add_bias(C, bias, M, N):
    C = np.ascontiguousarray(C, np.float32).copy()
    lib().ora_add_bias(_p(C), _p(np.ascontiguousarray(bias, np.float32)), M, N)
    return C


def activate(x, act: int):
    """activations.cl's silu / gelu on fp32 values (act 1 gelu with tanh, 2 silu, 3 gelu as
    activations.cl:78-117 computes it)."""
    y = np.ascontiguousarray(x, np.float32).copy()
    lib().ora_activate_n(_p(y), y.size, int(act))
    return y


def round_to(x, t: int):
    """x rounded to the storage type t (F32 0, F16 1, BF16 30) and read back as fp32."""
    if t == 1:
        return f16_to_f32(f16(x))
    if t == 30:
        return bf16_to_f32(bf16(x))
    return np.ascontiguousarray(x, np.float32)


def unfused_epilogue(acc, bias, act: int, resid, M: int, N: int, ctype: int):
    """The reference's chain after a GEMM, each kernel storing its output in ctype: the GEMM
    (+ bias, vision.cl:430-434) stores C, the activation kernel (activations.cl:30-117) reads
    and rewrites it, the residual add (vector_add, activations.cl:271-299, through
    dispatch_residual_add, moondream2.cpp:297-300) adds resid.  resid is fp32 values already
    in their storage type."""
    c = np.ascontiguousarray(acc, np.float32).reshape(M * N)
    if bias is not None:
        c = add_bias(c, bias, M, N)
    c = round_to(c, ctype)
    if act:
        c = round_to(activate(c, act), ctype)
    if resid is not None:
        c = round_to(c + np.ascontiguousarray(resid, np.float32).reshape(M * N), ctype)
    return c


def rms_norm(x, w, rows: int, hidden: int, eps: float, otype: int):
    """layernorm.cl's rms_norm on fp32 values (x already in its storage type), rounded to otype."""
    out = np.empty(rows * hidden, np.float32)
    lib().ora_rms_norm(_p(np.ascontiguousarray(x, np.float32)), _p(np.ascontiguousarray(w, np.float32)), _p(out),
                       rows, hidden, float(eps))
    return round_to(out, otype)


def unfused_silu_gate(gate_acc, up, ctype: int):
    """The reference's gate chain: the gate GEMM stores its output in ctype, then
    silu_gate_multiply (activations.cl:219-265) reads gate and up and stores
    silu(gate) * up in ctype.  up is fp32 values already in their storage type."""
    g = round_to(gate_acc, ctype)
    u = np.ascontiguousarray(up, np.float32).reshape(-1)
    out = np.empty_like(g)
    lib().ora_silu_gate_n(_p(g), _p(u), _p(out), g.size)
    return round_to(out, ctype)


def im2col(img, C, H, W, ph, pw):
    out = np.empty((H // ph) * (W // pw) * C * ph * pw, np.float32)
    lib().ora_im2col(_p(np.ascontiguousarray(img, np.float32)), _p(out), C, H, W, ph, pw)
    return out


def max_threads() -> int:
    return lib().ora_max_threads()


def set_threads(n: int) -> None:
    """Use n host threads in the multithreaded variants."""
    lib().ora_set_threads(int(n))


def argmax_logits(raw: np.ndarray, t: int) -> tuple[int, float]:
    """Greedy decode as src/models/moondream2.cpp:551-591 (argmax_logits) scans fp16 logits on
    the host: each value decoded with exponent field 0 -> 0.0, exponent all ones (Inf/NaN) ->
    +-1e30 by the sign bit, else the number; best = (-1e30, index 0) and an index replaces it
    only when its value is strictly greater (so the first maximum wins).  `raw` holds the
    logits' bits: uint16 for F16 / BF16, uint32 for F32 (bf16 / fp32 use the same rule on
    their own exponent fields).  Returns (index, value)."""
    best_id, best_val = 0, np.float32(-1e30)
    for i, h in enumerate(raw.tolist()):
        if t == F16:
            e, sign = (h >> 10) & 0x1F, h & 0x8000
            if e == 0:
                val = np.float32(0.0)
            elif e == 31:
                val = np.float32(-1e30 if sign else 1e30)
            else:
                val = np.array([h], np.uint16).view(np.float16)[0].astype(np.float32)
        else:
            b = h if t == F32 else h << 16
            e, sign = (b >> 23) & 0xFF, b & 0x80000000
            if e == 0:
                val = np.float32(0.0)
            elif e == 255:
                val = np.float32(-1e30 if sign else 1e30)
            else:
                val = np.array([b], np.uint32).view(np.float32)[0]
        if val > best_val:
            best_val, best_id = val, i
    return best_id, float(best_val)
