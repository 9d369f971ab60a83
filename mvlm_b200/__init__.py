"""mvlm_b200 - B200 (sm_100a) matmul path of MVLM behind a C ABI.

The product is ``libmgpu.so`` (built from ``csrc/`` by ``mvlm_b200.build``), whose entry
points are declared in ``include/mgpu_cuda.h``.  This module is the Python view of that ABI
(ctypes), mirroring the reference's dispatch interface (``src/engine/compute.h``) with the
same names and argument order: ``dispatch_gemm_naive / _tiled / _image``, ``dispatch_gemv``,
``dispatch_patch_embed``, ``dispatch_vision_proj``; dispatch calls return an event or
``None`` on error like the reference's ``cl_event`` / ``nullptr``.

There is no CPU fallback: importing works without a GPU, but every call that needs the
device raises ``MgpuError`` when the library or the device is missing.
"""
from __future__ import annotations

import ctypes
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libmgpu.so")

F32, F16, Q4_0, Q8_0, BF16 = 0, 1, 2, 8, 30
LAYOUT_KN, LAYOUT_NK = 0, 1
ACT_NONE, ACT_GELU, ACT_SILU, ACT_GELU_AS_SHIPPED = 0, 1, 2, 3
OK, ERR_INVALID_ARG, ERR_UNSUPPORTED, ERR_CUDA, ERR_OUT_OF_MEMORY, ERR_DEVICE_TIMEOUT = range(6)

TYPE_SIZE = {F32: 4, F16: 2, BF16: 2}
BLOCK_BYTES = {Q4_0: 18, Q8_0: 34}
NP_DTYPE = {F32: np.float32, F16: np.uint16, BF16: np.uint16}

# Every symbol include/mgpu_cuda.h declares, with (restype, argtypes).
_vp, _i, _i64, _u64, _sz, _f, _d, _cp = (ctypes.c_void_p, ctypes.c_int, ctypes.c_int64, ctypes.c_uint64,
                                         ctypes.c_size_t, ctypes.c_float, ctypes.c_double, ctypes.c_char_p)
SIGNATURES = {
    "mgpu_last_error": (_i, []),
    "mgpu_last_error_string": (_cp, []),
    "mgpu_clear_error": (None, []),
    "mgpu_init_device": (_vp, [_i]),
    "mgpu_release_device": (None, [_vp]),
    "mgpu_device_ordinal": (_i, [_vp]),
    "mgpu_device_sm_count": (_i, [_vp]),
    "mgpu_device_l2_bytes": (_sz, [_vp]),
    "mgpu_device_stream": (_vp, [_vp]),
    "mgpu_set_stream": (_i, [_vp, _vp]),
    "mgpu_set_event_mode": (_i, [_vp, _i]),
    "mgpu_finish": (_i, [_vp]),
    "mgpu_create_buffer": (_vp, [_vp, _sz, _vp]),
    "mgpu_create_weight_image": (_vp, [_vp, _i, _i, _vp]),
    "mgpu_wrap_buffer": (_vp, [_vp, _vp, _sz]),
    "mgpu_buf_view": (_vp, [_vp, _sz, _sz]),
    "mgpu_buf_set_format": (_i, [_vp, _i, _i, _i64, _i64, _i64]),
    "mgpu_buf_device_ptr": (_vp, [_vp]),
    "mgpu_buf_bytes": (_sz, [_vp]),
    "mgpu_buf_write": (_i, [_vp, _sz, _vp, _sz]),
    "mgpu_buf_read": (_i, [_vp, _sz, _vp, _sz]),
    "mgpu_buf_write_async": (_i, [_vp, _sz, _vp, _sz]),
    "mgpu_buf_read_async": (_i, [_vp, _sz, _vp, _sz]),
    "mgpu_buf_copy_async": (_i, [_vp, _sz, _vp, _sz, _sz]),
    "mgpu_host_alloc": (_vp, [_sz]),
    "mgpu_host_free": (None, [_vp]),
    "mgpu_release_buffer": (None, [_vp]),
    "mgpu_upload_weight": (_vp, [_vp, _vp, _vp]),
    "mgpu_dispatch_gemm_naive": (_vp, [_vp, _vp, _vp, _vp, _vp, _i, _i, _i]),
    "mgpu_dispatch_gemm_tiled": (_vp, [_vp, _vp, _vp, _vp, _vp, _i, _i, _i]),
    "mgpu_dispatch_gemm_image": (_vp, [_vp, _vp, _vp, _vp, _vp, _i, _i, _i]),
    "mgpu_dispatch_gemv": (_vp, [_vp, _vp, _vp, _vp, _vp, _i, _i]),
    "mgpu_dispatch_patch_embed": (_vp, [_vp, _vp, _vp, _vp, _vp, _vp, _i, _i, _i, _i, _i, _i]),
    "mgpu_dispatch_vision_proj": (_vp, [_vp, _vp, _vp, _vp, _vp, _vp, _i, _i, _i]),
    "mgpu_dispatch_gemv_noalloc": (_i, [_vp, _vp, _vp, _vp, _i, _i]),
    "mgpu_gemv_q": (_vp, [_vp, _vp, _vp, _vp, _i, _i, _i]),
    "mgpu_dispatch_rms_norm": (_vp, [_vp, _vp, _vp, _vp, _vp, _i, _i, _f]),
    "mgpu_gemv_q_rmsnorm": (_vp, [_vp, _vp, _vp, _f, _vp, _vp, _i, _i, _i]),
    "mgpu_gemv_chain_create": (_vp, [_vp, _vp, _i]),
    "mgpu_gemv_chain_run": (_vp, [_vp]),
    "mgpu_gemv_chain_run_timed": (_i, [_vp, _vp]),
    "mgpu_gemv_chain_links": (_i, [_vp]),
    "mgpu_gemv_chain_destroy": (None, [_vp]),
    "mgpu_gemm_q": (_vp, [_vp, _vp, _vp, _vp, _i, _i, _i, _i, _vp]),
    "mgpu_gemm": (_vp, [_vp, _vp, _vp, _vp, _i, _i, _i, _vp]),
    "mgpu_gemm_fused": (_vp, [_vp, _vp, _vp, _vp, _i, _i, _i, _vp, _i, _vp]),
    "mgpu_gemm_silu_gate": (_vp, [_vp, _vp, _vp, _vp, _vp, _i, _i, _i]),
    "mgpu_dequant": (_vp, [_vp, _vp, _vp, _i64, _i]),
    "mgpu_argmax": (_vp, [_vp, _vp, _i, _vp]),
    "mgpu_argmax_logits": (_i, [_vp, _vp, _i]),
    "mgpu_argmax_rows": (_vp, [_vp, _vp, _i, _i, _i64, _vp]),
    "mgpu_argmax_combine": (_vp, [_vp, _vp, _i, _i, _vp]),
    "mgpu_peer_group_create": (_vp, [_vp, _i, _i, _sz]),
    "mgpu_peer_group_handle": (_i, [_vp, _vp]),
    "mgpu_peer_group_connect": (_i, [_vp, _vp]),
    "mgpu_peer_group_connect_ptrs": (_i, [_vp, _vp]),
    "mgpu_peer_group_local_ptr": (_vp, [_vp]),
    "mgpu_peer_group_slots": (_vp, [_vp]),
    "mgpu_peer_group_set_wait_limit": (_i, [_vp, _u64]),
    "mgpu_peer_allgather": (_vp, [_vp, _vp, _sz]),
    "mgpu_peer_alltoall": (_vp, [_vp, _vp, _sz]),
    "mgpu_peer_group_destroy": (None, [_vp]),
    "mgpu_wait_event": (_i, [_vp]),
    "mgpu_release_event": (None, [_vp]),
    "mgpu_profile_end": (_d, [_vp]),
    "mgpu_event_elapsed_ms": (_f, [_vp, _vp]),
    "mgpu_record_event": (_vp, [_vp]),
    "mgpu_capture_begin": (_i, [_vp]),
    "mgpu_capture_end": (_vp, [_vp]),
    "mgpu_graph_launch": (_i, [_vp]),
    "mgpu_graph_release": (None, [_vp]),
    "mgpu_selftest_bounded_wait": (_i, [_vp, _u64]),
    "mgpu_ggml_type_size": (_sz, [_i]),
    "mgpu_ggml_type_block_size": (_i, [_i]),
    "mgpu_fill_uniform": (_i, [_vp, _vp, _i64, _u64, _f, _f]),
    "mgpu_fill_normal": (_i, [_vp, _vp, _i64, _u64, _f]),
    "mgpu_quantize": (_i, [_vp, _vp, _vp, _i64, _i]),
    "mgpu_convert": (_i, [_vp, _vp, _vp, _i64]),
}


class MgpuError(RuntimeError):
    def __init__(self, code: int, msg: str):
        super().__init__(f"mgpu error {code}: {msg}")
        self.code = code


class TensorInfo(ctypes.Structure):
    """Binary-compatible with the reference's TensorInfo (src/models/gguf_loader.h:51-58)."""
    _fields_ = [("name", ctypes.c_char * 256), ("n_dims", ctypes.c_uint32), ("dims", ctypes.c_uint64 * 4),
                ("type", ctypes.c_uint32), ("offset", ctypes.c_uint64), ("data_size", ctypes.c_size_t)]


class GemvLink(ctypes.Structure):
    """mgpu_gemv_link: one GEMV of a chain (x may be a view of an earlier link's y)."""
    _fields_ = [("x", ctypes.c_void_p), ("W", ctypes.c_void_p), ("y", ctypes.c_void_p), ("N", ctypes.c_int),
                ("K", ctypes.c_int)]


_lib = None


def lib() -> ctypes.CDLL:
    """Load libmgpu.so (fails loudly if it was not built)."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise MgpuError(ERR_UNSUPPORTED, f"{LIB_PATH} is missing: run `python -m mvlm_b200.build`")
        L = ctypes.CDLL(LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


def last_error() -> tuple[int, str]:
    L = lib()
    return L.mgpu_last_error(), (L.mgpu_last_error_string() or b"").decode()


def _raise_last(what: str):
    code, msg = last_error()
    raise MgpuError(code or ERR_CUDA, f"{what}: {msg}")


def _check(rc: int, what: str):
    if rc != OK:
        _raise_last(what)


class Event:
    """cl_event stand-in: wait(), profile_ms() (profile_end), release on drop."""

    def __init__(self, handle):
        self.h = handle

    def wait(self):
        if self.h:
            _check(lib().mgpu_wait_event(self.h), "wait_event")

    def profile_ms(self) -> float:
        return lib().mgpu_profile_end(self.h) if self.h else 0.0

    def elapsed_ms(self, later: "Event") -> float:
        """Device time from this marker to a later one (mgpu_event_elapsed_ms)."""
        return lib().mgpu_event_elapsed_ms(self.h, later.h)

    def __del__(self):
        if getattr(self, "h", None) and _lib is not None:
            _lib.mgpu_release_event(self.h)
            self.h = None


class Buffer:
    """cl_mem stand-in: owns (or wraps) device memory and carries its type / layout tag."""

    def __init__(self, dev: "Device", handle, nbytes: int):
        self.dev, self.h, self.nbytes = dev, handle, nbytes

    @property
    def ptr(self) -> int:
        return lib().mgpu_buf_device_ptr(self.h)

    def set_format(self, type_: int, layout: int = LAYOUT_KN, rows: int = 0, cols: int = 0, ld: int = 0):
        _check(lib().mgpu_buf_set_format(self.h, type_, layout, rows, cols, ld), "buf_set_format")
        return self

    def write(self, arr: np.ndarray, offset: int = 0):
        arr = np.ascontiguousarray(arr)
        _check(lib().mgpu_buf_write(self.h, offset, arr.ctypes.data, arr.nbytes), "buf_write")
        return self

    def read(self, dtype, count: int | None = None, offset: int = 0) -> np.ndarray:
        dtype = np.dtype(dtype)
        if count is None:
            count = (self.nbytes - offset) // dtype.itemsize
        out = np.empty(count, dtype)
        _check(lib().mgpu_buf_read(self.h, offset, out.ctypes.data, out.nbytes), "buf_read")
        return out

    def view(self, offset: int, nbytes: int) -> "Buffer":
        h = lib().mgpu_buf_view(self.h, offset, nbytes)
        if not h:
            _raise_last("buf_view")
        return Buffer(self.dev, h, nbytes)

    def release(self):
        if self.h and _lib is not None:
            _lib.mgpu_release_buffer(self.h)
        self.h = None

    def __del__(self):
        self.release()


class Device:
    """DeviceInfo stand-in (src/engine/device.h:13-55): one CUDA device, one in-order stream."""

    def __init__(self, ordinal: int = 0):
        h = lib().mgpu_init_device(ordinal)
        if not h:
            _raise_last("init_device")
        self.h = h
        self.ordinal = ordinal

    @property
    def sm_count(self) -> int:
        return lib().mgpu_device_sm_count(self.h)

    @property
    def l2_bytes(self) -> int:
        return lib().mgpu_device_l2_bytes(self.h)

    @property
    def stream(self) -> int:
        return lib().mgpu_device_stream(self.h)

    def set_stream(self, stream_ptr: int | None):
        _check(lib().mgpu_set_stream(self.h, stream_ptr), "set_stream")

    def set_event_mode(self, mode: int):
        _check(lib().mgpu_set_event_mode(self.h, mode), "set_event_mode")

    def finish(self):
        _check(lib().mgpu_finish(self.h), "finish")

    # ---- memory.h ----
    def create_buffer(self, nbytes: int, host: np.ndarray | None = None, type_: int | None = None,
                      layout: int = LAYOUT_KN, rows: int = 0, cols: int = 0, ld: int = 0) -> Buffer:
        src = None
        if host is not None:
            host = np.ascontiguousarray(host)
            assert host.nbytes <= nbytes
            if host.nbytes < nbytes:
                pad = np.zeros(nbytes, np.uint8)
                pad[: host.nbytes] = host.view(np.uint8).reshape(-1)
                host = pad
            src = host.ctypes.data
        h = lib().mgpu_create_buffer(self.h, nbytes, src)
        if not h:
            _raise_last("create_buffer")
        b = Buffer(self, h, nbytes)
        if type_ is not None:
            b.set_format(type_, layout, rows, cols, ld)
        return b

    def array(self, arr: np.ndarray, type_: int, layout: int = LAYOUT_KN, rows: int = 0, cols: int = 0,
              ld: int = 0) -> Buffer:
        arr = np.ascontiguousarray(arr)
        return self.create_buffer(arr.nbytes, arr, type_, layout, rows, cols, ld)

    def empty(self, count: int, type_: int) -> Buffer:
        return self.create_buffer(count * TYPE_SIZE[type_], None, type_)

    def create_weight_image(self, rows: int, cols: int, fp16: np.ndarray) -> Buffer:
        fp16 = np.ascontiguousarray(fp16, np.uint16)
        h = lib().mgpu_create_weight_image(self.h, rows, cols, fp16.ctypes.data)
        if not h:
            _raise_last("create_weight_image")
        return Buffer(self, h, lib().mgpu_buf_bytes(h))

    def wrap(self, ptr: int, nbytes: int, type_: int, layout: int = LAYOUT_KN, rows: int = 0, cols: int = 0,
             ld: int = 0) -> Buffer:
        h = lib().mgpu_wrap_buffer(self.h, ptr, nbytes)
        if not h:
            _raise_last("wrap_buffer")
        return Buffer(self, h, nbytes).set_format(type_, layout, rows, cols, ld)

    def upload_weight(self, info: TensorInfo, data: np.ndarray) -> Buffer:
        data = np.ascontiguousarray(data)
        h = lib().mgpu_upload_weight(self.h, ctypes.byref(info), data.ctypes.data)
        if not h:
            _raise_last("upload_weight")
        return Buffer(self, h, lib().mgpu_buf_bytes(h))

    # ---- synthetic data ----
    def fill_uniform(self, buf: Buffer, n: int, seed: int, lo: float = -1.0, hi: float = 1.0):
        _check(lib().mgpu_fill_uniform(self.h, buf.h, n, seed, lo, hi), "fill_uniform")

    def fill_normal(self, buf: Buffer, n: int, seed: int, sigma: float = 1.0):
        _check(lib().mgpu_fill_normal(self.h, buf.h, n, seed, sigma), "fill_normal")

    def quantize(self, src: Buffer, dst: Buffer, n: int, qtype: int):
        _check(lib().mgpu_quantize(self.h, src.h, dst.h, n, qtype), "quantize")

    def convert(self, src: Buffer, dst: Buffer, n: int):
        _check(lib().mgpu_convert(self.h, src.h, dst.h, n), "convert")

    # ---- graphs ----
    def capture_begin(self):
        _check(lib().mgpu_capture_begin(self.h), "capture_begin")

    def capture_end(self) -> "Graph":
        h = lib().mgpu_capture_end(self.h)
        if not h:
            _raise_last("capture_end")
        return Graph(h)

    def record_event(self) -> Event:
        h = lib().mgpu_record_event(self.h)
        if not h:
            _raise_last("record_event")
        return Event(h)

    def selftest_bounded_wait(self, limit_ns: int):
        _check(lib().mgpu_selftest_bounded_wait(self.h, limit_ns), "selftest_bounded_wait")

    def release(self):
        if getattr(self, "h", None) and _lib is not None:
            _lib.mgpu_release_device(self.h)
        self.h = None


class Graph:
    """A captured dispatch sequence (mgpu_capture_begin / mgpu_capture_end)."""

    def __init__(self, handle):
        self.h = handle

    def launch(self):
        _check(lib().mgpu_graph_launch(self.h), "graph_launch")

    def __del__(self):
        if getattr(self, "h", None) and _lib is not None:
            _lib.mgpu_graph_release(self.h)
            self.h = None


def _ev(handle, what: str) -> Event:
    if not handle:
        code, _ = last_error()
        if code != OK:
            _raise_last(what)
    return Event(handle)


def _h(b):
    return b.h if b is not None else None


# ---- compute.h mirror (same names and argument order; program is accepted and ignored) ----
def dispatch_gemm_naive(dev: Device, program, A: Buffer, B: Buffer, C: Buffer, M: int, N: int, K: int) -> Event:
    return _ev(lib().mgpu_dispatch_gemm_naive(dev.h, None, A.h, B.h, C.h, M, N, K), "dispatch_gemm_naive")


def dispatch_gemm_tiled(dev: Device, program, A: Buffer, B: Buffer, C: Buffer, M: int, N: int, K: int) -> Event:
    return _ev(lib().mgpu_dispatch_gemm_tiled(dev.h, None, A.h, B.h, C.h, M, N, K), "dispatch_gemm_tiled")


def dispatch_gemm_image(dev: Device, program, A: Buffer, B_img: Buffer, C: Buffer, M: int, N: int, K: int) -> Event:
    return _ev(lib().mgpu_dispatch_gemm_image(dev.h, None, A.h, B_img.h, C.h, M, N, K), "dispatch_gemm_image")


def dispatch_gemv(dev: Device, program, x: Buffer, W_img: Buffer, y: Buffer, N: int, K: int) -> Event:
    return _ev(lib().mgpu_dispatch_gemv(dev.h, None, x.h, W_img.h, y.h, N, K), "dispatch_gemv")


def dispatch_patch_embed(dev: Device, program, image: Buffer, proj_weight: Buffer, proj_bias: Buffer | None,
                         patches: Buffer, C: int, H: int, W: int, patch_h: int, patch_w: int,
                         embed_dim: int) -> Event:
    return _ev(lib().mgpu_dispatch_patch_embed(dev.h, None, image.h, proj_weight.h, _h(proj_bias), patches.h, C, H,
                                               W, patch_h, patch_w, embed_dim), "dispatch_patch_embed")


def dispatch_vision_proj(dev: Device, program, visual_tokens: Buffer, proj_weight: Buffer,
                         proj_bias: Buffer | None, output: Buffer, num_patches: int, vision_dim: int,
                         llm_dim: int) -> Event:
    return _ev(lib().mgpu_dispatch_vision_proj(dev.h, None, visual_tokens.h, proj_weight.h, _h(proj_bias), output.h,
                                               num_patches, vision_dim, llm_dim), "dispatch_vision_proj")


def dispatch_gemv_noalloc(dev: Device, x: Buffer, W_img: Buffer, y: Buffer, N: int, K: int) -> None:
    """mgpu_dispatch_gemv_noalloc: the [K][N] GEMV with its scratch in a fixed device array of
    the library (no allocation; N <= 262144; calls that overlap on the GPU race)."""
    _check(lib().mgpu_dispatch_gemv_noalloc(dev.h, x.h, W_img.h, y.h, N, K), "dispatch_gemv_noalloc")


def dispatch_rms_norm(dev: Device, program, input: Buffer, output: Buffer, weight: Buffer, num_rows: int,
                      hidden_size: int, eps: float) -> Event:
    return _ev(lib().mgpu_dispatch_rms_norm(dev.h, None, input.h, output.h, weight.h, num_rows, hidden_size, eps),
               "dispatch_rms_norm")


def gemv_q_rmsnorm(dev: Device, x: Buffer, norm_weight: Buffer, eps: float, W: Buffer, y: Buffer, N: int, K: int,
                   qtype: int) -> Event:
    """y = RMSNorm(x) . dequant(W)^T with the norm in the GEMV's prologue (mgpu_gemv_q_rmsnorm)."""
    return _ev(lib().mgpu_gemv_q_rmsnorm(dev.h, x.h, norm_weight.h, eps, W.h, y.h, N, K, qtype), "gemv_q_rmsnorm")


def gemv_q(dev: Device, x: Buffer, W: Buffer, y: Buffer, N: int, K: int, qtype: int) -> Event:
    return _ev(lib().mgpu_gemv_q(dev.h, x.h, W.h, y.h, N, K, qtype), "gemv_q")


class GemvChain:
    """mgpu_gemv_chain: a decode step's dependent GEMVs in one persistent launch.

    links: (x, W, y, N, K) per GEMV in order; an x that is a view of an earlier link's y reads
    that link's output (the chain's dataflow), any other x is read as it is when the chain runs.
    The buffers must outlive the chain (this object keeps references to them)."""

    def __init__(self, dev: Device, links):
        self.dev = dev
        self._keep = [(x, W, y) for x, W, y, _, _ in links]
        arr = (GemvLink * len(links))(*[GemvLink(x.h, W.h, y.h, N, K) for x, W, y, N, K in links])
        h = lib().mgpu_gemv_chain_create(dev.h, arr, len(links))
        if not h:
            _raise_last("gemv_chain_create")
        self.h = h
        self.n = len(links)

    def run(self) -> Event:
        return _ev(lib().mgpu_gemv_chain_run(self.h), "gemv_chain_run")

    def run_timed(self) -> np.ndarray:
        """One synchronous run; microseconds from the run's start to the end of each link."""
        out = np.zeros(self.n, np.float64)
        _check(lib().mgpu_gemv_chain_run_timed(self.h, out.ctypes.data), "gemv_chain_run_timed")
        return out

    def destroy(self):
        if getattr(self, "h", None) and _lib is not None:
            _lib.mgpu_gemv_chain_destroy(self.h)
        self.h = None

    def __del__(self):
        self.destroy()


def gemm_q(dev: Device, A: Buffer, W: Buffer, C: Buffer, M: int, N: int, K: int, qtype: int,
           bias: Buffer | None = None) -> Event:
    return _ev(lib().mgpu_gemm_q(dev.h, A.h, W.h, C.h, M, N, K, qtype, _h(bias)), "gemm_q")


def gemm(dev: Device, A: Buffer, B: Buffer, C: Buffer, M: int, N: int, K: int, bias: Buffer | None = None) -> Event:
    return _ev(lib().mgpu_gemm(dev.h, A.h, B.h, C.h, M, N, K, _h(bias)), "gemm")


def gemm_fused(dev: Device, A: Buffer, B: Buffer, C: Buffer, M: int, N: int, K: int, bias: Buffer | None = None,
               act: int = ACT_NONE, residual: Buffer | None = None) -> Event:
    """C = act(A . op(B) + bias) + residual in one GEMM (the reference's GEMM, activation and
    residual-add kernels in sequence); residual may be C itself."""
    return _ev(lib().mgpu_gemm_fused(dev.h, A.h, B.h, C.h, M, N, K, _h(bias), act, _h(residual)), "gemm_fused")


def gemm_silu_gate(dev: Device, A: Buffer, W_gate: Buffer, up: Buffer, out: Buffer, M: int, N: int, K: int) -> Event:
    """out = silu(A . op(W_gate)) * up (the gate GEMM and silu_gate_multiply in one kernel)."""
    return _ev(lib().mgpu_gemm_silu_gate(dev.h, A.h, W_gate.h, up.h, out.h, M, N, K), "gemm_silu_gate")


def dequant(dev: Device, W: Buffer, out: Buffer, n: int, qtype: int) -> Event:
    return _ev(lib().mgpu_dequant(dev.h, W.h, out.h, n, qtype), "dequant")


def argmax(dev: Device, logits: Buffer, n: int, out: Buffer) -> Event:
    """out (8 bytes) <- {int32 index, fp32 value}: the reference's argmax_logits on the device."""
    return _ev(lib().mgpu_argmax(dev.h, logits.h, n, out.h), "argmax")


def argmax_rows(dev: Device, logits: Buffer, rows: int, n: int, ld: int, out: Buffer) -> Event:
    """out (8 bytes per row) <- mgpu_argmax of each of `rows` rows of n logits, row r at element
    r * ld: one launch for a batch of sequences."""
    return _ev(lib().mgpu_argmax_rows(dev.h, logits.h, rows, n, ld, out.h), "argmax_rows")


def argmax_combine(dev: Device, pairs: Buffer, n_ranks: int, n_total: int, out: Buffer) -> Event:
    """out (8 bytes) <- the global {index, value} from the ranks' gathered mgpu_argmax pairs of a
    row column-sharded over n_ranks GPUs (the reference's first maximum over the whole row)."""
    return _ev(lib().mgpu_argmax_combine(dev.h, pairs.h, n_ranks, n_total, out.h), "argmax_combine")


class PeerGroup:
    """Exchanges between the GPUs of one node through peer memory (mgpu_peer_group_*): world
    receive slots of slot_bytes on every GPU, mapped by the others through CUDA IPC.  Connect
    with the handles of all ranks in rank order (`handle()` on each, exchanged by the caller), or
    with `connect_ptrs` when the groups live in one process."""

    def __init__(self, dev: Device, rank: int, world: int, slot_bytes: int):
        h = lib().mgpu_peer_group_create(dev.h, rank, world, slot_bytes)
        if not h:
            _raise_last("peer_group_create")
        self.dev, self.h, self.rank, self.world = dev, h, rank, world
        self.slot_bytes = (slot_bytes + 7) // 8 * 8

    def handle(self) -> bytes:
        buf = ctypes.create_string_buffer(64)
        _check(lib().mgpu_peer_group_handle(self.h, buf), "peer_group_handle")
        return buf.raw

    def connect(self, handles):
        blob = b"".join(handles)
        if len(blob) != 64 * self.world:
            raise MgpuError(ERR_INVALID_ARG, "peer_group_connect: one 64-byte handle per rank")
        _check(lib().mgpu_peer_group_connect(self.h, blob), "peer_group_connect")
        return self

    def connect_ptrs(self, ptrs):
        arr = (ctypes.c_void_p * self.world)(*ptrs)
        _check(lib().mgpu_peer_group_connect_ptrs(self.h, arr), "peer_group_connect_ptrs")
        return self

    def local_ptr(self) -> int:
        return lib().mgpu_peer_group_local_ptr(self.h)

    def slots(self, type_: int) -> Buffer:
        """A view of this GPU's slots (slot r = rank r's bytes), tagged with type_."""
        v = lib().mgpu_buf_view(lib().mgpu_peer_group_slots(self.h), 0, self.world * self.slot_bytes)
        if not v:
            _raise_last("peer_group_slots")
        return Buffer(self.dev, v, self.world * self.slot_bytes).set_format(type_)

    def set_wait_limit(self, ns: int):
        _check(lib().mgpu_peer_group_set_wait_limit(self.h, ns), "peer_group_set_wait_limit")

    def allgather(self, src: Buffer, nbytes: int) -> Event:
        return _ev(lib().mgpu_peer_allgather(self.h, src.h, nbytes), "peer_allgather")

    def alltoall(self, src: Buffer, bytes_per_peer: int) -> Event:
        return _ev(lib().mgpu_peer_alltoall(self.h, src.h, bytes_per_peer), "peer_alltoall")

    def destroy(self):
        if self.h and _lib is not None:
            _lib.mgpu_peer_group_destroy(self.h)
        self.h = None

    def __del__(self):
        self.destroy()


def argmax_logits(dev: Device, logits: Buffer, vocab_size: int) -> int:
    """argmax_logits(device, logits, vocab_size) (src/models/moondream2.cpp:551): the token id."""
    idx = lib().mgpu_argmax_logits(dev.h, logits.h, vocab_size)
    if idx < 0:
        _raise_last("argmax_logits")
    return idx


def ggml_type_size(t: int) -> int:
    return lib().mgpu_ggml_type_size(t)


def ggml_type_block_size(t: int) -> int:
    return lib().mgpu_ggml_type_block_size(t)


def row_bytes(t: int, k: int) -> int:
    if t in BLOCK_BYTES:
        return (k + 31) // 32 * BLOCK_BYTES[t]
    return k * TYPE_SIZE[t]
