"""The C ABI library loads and exports every symbol include/mgpu_cuda.h declares; the C++
mirror header compiles a reference-style call site; host-only entry points agree with the
reference's ggml table and TensorInfo layout.  No GPU needed."""
import ctypes
import os
import re
import subprocess

import pytest

import mvlm_b200 as mg

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "mgpu_cuda.h")


def header_symbols() -> set[str]:
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return set(re.findall(r"^[A-Za-z_][\w\s\*]*?\b(mgpu_[a-z0-9_]+)\s*\(", text, flags=re.M))


def test_header_declares_expected_boundary():
    syms = header_symbols()
    for s in ("mgpu_dispatch_gemm_naive", "mgpu_dispatch_gemm_tiled", "mgpu_dispatch_gemm_image",
              "mgpu_dispatch_gemv", "mgpu_dispatch_patch_embed", "mgpu_dispatch_vision_proj", "mgpu_gemv_q",
              "mgpu_gemm_q", "mgpu_dequant", "mgpu_upload_weight", "mgpu_init_device", "mgpu_profile_end"):
        assert s in syms, s


def test_library_exports_every_declared_symbol():
    L = mg.lib()
    syms = header_symbols()
    missing = [s for s in sorted(syms) if not hasattr(L, s)]
    assert not missing, missing
    assert set(mg.SIGNATURES) == syms, set(mg.SIGNATURES) ^ syms


def test_cpp_mirror_compiles_reference_call_site(tmp_path):
    src = tmp_path / "callsite.cpp"
    src.write_text(r'''
#include "mgpu_compute.hpp"
using namespace mgpu;
// The shape of moondream2_forward's GEMV / GEMM call sites (src/models/moondream2.cpp:370-403).
int forward_like(const DeviceInfo* device, cl_program gemm_program, cl_mem residual_buf, cl_mem q_proj_weight,
                 cl_mem scratch_q, int seq_len, int llm_dim, bool is_decode) {
    cl_event ev = nullptr;
    if (is_decode) ev = dispatch_gemv(device, gemm_program, residual_buf, q_proj_weight, scratch_q, llm_dim, llm_dim);
    else ev = dispatch_gemm_image(device, gemm_program, residual_buf, q_proj_weight, scratch_q, seq_len, llm_dim, llm_dim);
    if (ev) { clWaitForEvents(1, &ev); clReleaseEvent(ev); }
    return ev ? 0 : 1;
}
''')
    r = subprocess.run(["g++", "-std=c++17", "-fsyntax-only", "-Wall", "-Werror", "-I", os.path.join(ROOT, "include"),
                        str(src)], capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
    r = subprocess.run(["gcc", "-std=c11", "-fsyntax-only", "-Wall", "-Werror", "-x", "c", HEADER],
                       capture_output=True, text=True)
    assert r.returncode == 0, r.stderr


def test_ggml_table_matches_reference():
    for t, size, block in ((mg.F32, 4, 1), (mg.F16, 2, 1), (mg.Q4_0, 18, 32), (mg.Q8_0, 34, 32), (mg.BF16, 2, 1)):
        assert mg.ggml_type_size(t) == size and mg.ggml_type_block_size(t) == block
    import oracle as O
    R = O.ref_gguf()
    if R is None:
        pytest.skip("reference gguf_loader not built")
    for t in (mg.F32, mg.F16, mg.Q4_0, mg.Q8_0):
        assert mg.ggml_type_size(t) == R.ref_ggml_type_size(t)
        assert mg.ggml_type_block_size(t) == R.ref_ggml_type_block_size(t)


def test_tensor_info_is_binary_compatible(tmp_path):
    import numpy as np
    import oracle as O
    from tests.gguf_writer import write_gguf
    R = O.ref_gguf()
    if R is None:
        pytest.skip("reference gguf_loader not built")
    assert ctypes.sizeof(mg.TensorInfo) == R.ref_tensor_info_size()
    K, N = 256, 12
    q = O.quantize(O.normal(K * N, 3, 0.02), O.Q4_0)
    path = str(tmp_path / "w.gguf")
    write_gguf(path, [("blk.0.ffn_up.weight", [K, N], O.Q4_0, q)], {"general.alignment": 32})
    info = mg.TensorInfo()
    buf = np.zeros(q.size, np.uint8)
    n = R.ref_gguf_read_tensor(path.encode(), b"blk.0.ffn_up.weight", ctypes.byref(info), buf.ctypes.data, buf.size)
    assert n == q.size
    assert info.n_dims == 2 and info.dims[0] == K and info.dims[1] == N and info.type == O.Q4_0
    assert info.data_size == N * K // 32 * 18
    np.testing.assert_array_equal(buf, q)


def test_no_device_is_an_error_not_a_crash():
    import torch
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    L = mg.lib()
    assert not L.mgpu_init_device(0)
    code, msg = mg.last_error()
    assert code != mg.OK and msg
    with pytest.raises(mg.MgpuError):
        mg.Device(0)


def test_engine_dropin_harness_links():
    # oracle/_ref/libref_dropin.so: the reference's moondream2_forward (extracted unmodified from
    # src/models/moondream2.cpp) compiled with the reference's headers over include/cl_compat and
    # linked to libmgpu through mvlm_b200/engine/engine_cuda.cpp; the GPU run is
    # tests/test_gpu_dropin.py
    ref = os.path.join(ROOT, "oracle", "_ref")
    lib_path = os.path.join(ref, "libref_dropin.so")
    if not os.path.exists(lib_path):
        pytest.skip("built only where the reference checkout is present")
    with open(os.path.join(ref, "moondream2_forward.inc")) as f:
        text = f.read()
    assert "cl_mem moondream2_forward(Moondream2Model* model" in text and "kv_cache_append" in text
    mg.lib()  # libmgpu first, as the harness links it
    L = ctypes.CDLL(lib_path)
    assert hasattr(L, "dropin_forward_decode")
