"""GPU test of mgpu_dispatch_gemv_noalloc, the GEMV entry point that allocates nothing.

Callers that cannot let the library allocate (engines that give all GPU memory to their own
pool at start-up; decode loops that must not stall on cudaMalloc / cudaFree) call this
variant instead of mgpu_dispatch_gemv.  Its split-K scratch is a fixed device array inside the
library, so this test checks that, through the C ABI, two calls in a row give the same result
as the allocating entry point (same tolerance as the other GPU tests), and that sizes beyond
the array are refused before anything runs.  This file is collected last on purpose.
"""
import numpy as np
import pytest

import mvlm_b200 as mg
import oracle as O
from tests.numerics import TOL_16, TOL_F32, assert_close

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("K,N", [(2048, 8192), (512, 300), (1024, 51200)])
def test_noalloc_matches_allocating_entry_fp32(dev, K, N):
    x = O.uniform(K, 0x4D564C4D + N)
    W = O.uniform(K * N, 0x4D564C4E + K)
    dx, dW = dev.array(x, mg.F32), dev.array(W, mg.F32, mg.LAYOUT_KN)
    y_ref, y_new = dev.empty(N, mg.F32), dev.empty(N, mg.F32)
    mg.dispatch_gemv(dev, None, dx, dW, y_ref, N, K).wait()
    ref = y_ref.read(np.float32)
    # the allocating entry itself against the oracle's restatement of the reference gemv
    assert_close(ref, O.gemv_f32(x, W, N, K), TOL_F32, f"dispatch_gemv fp32 {K}x{N}")
    for _ in range(2):  # two calls in a row: the shared array must come back clean
        y_new.write(np.full(N, np.nan, np.float32))
        mg.dispatch_gemv_noalloc(dev, dx, dW, y_new, N, K)
        dev.finish()
        assert_close(y_new.read(np.float32), ref, TOL_F32, f"noalloc fp32 {K}x{N}")


def test_noalloc_matches_allocating_entry_fp16_image(dev):
    # the reference gemv's own types: fp16 x, fp16 weight image [K][N], fp16 y
    K, N = 2048, 2048
    x = O.f16(O.uniform(K, 7))
    W = O.f16(O.uniform(K * N, 8))
    dx, img = dev.array(x, mg.F16), dev.create_weight_image(K, N, W)
    y_ref, y_new = dev.empty(N, mg.F16), dev.empty(N, mg.F16)
    mg.dispatch_gemv(dev, None, dx, img, y_ref, N, K).wait()
    ref = O.f16_to_f32(y_ref.read(np.uint16))
    # the oracle's restatement of the reference gemv on the same fp16 data
    assert_close(ref, O.f16_to_f32(O.gemv_f16(x, W, N, K)), TOL_16, "dispatch_gemv fp16 image")
    for _ in range(2):
        mg.dispatch_gemv_noalloc(dev, dx, img, y_new, N, K)
        dev.finish()
        got = O.f16_to_f32(y_new.read(np.uint16))
        assert_close(got, ref, TOL_16, "noalloc fp16 image")
        assert_close(got, O.f16_to_f32(O.gemv_f16(x, W, N, K)), TOL_16, "noalloc fp16 image vs oracle")


def test_noalloc_largest_size_and_mixed_types(dev):
    # N = 262144 is the largest size the array holds: the K split drops to one and the fp32
    # partials fill the whole array.  Then bf16 x against f16 weights with an f16 y, which
    # take other instantiations of the launcher's type switch.
    K, N = 64, 262144
    x = O.uniform(K, 11)
    W = O.uniform(K * N, 12)
    dx, dW = dev.array(x, mg.F32), dev.array(W, mg.F32, mg.LAYOUT_KN)
    y_ref, y_new = dev.empty(N, mg.F32), dev.empty(N, mg.F32)
    mg.dispatch_gemv(dev, None, dx, dW, y_ref, N, K).wait()
    ref = y_ref.read(np.float32)
    oracle = O.gemv_f32(x, W, N, K)
    assert_close(ref, oracle, TOL_F32, "dispatch_gemv fp32 at the size limit")
    for _ in range(2):
        y_new.write(np.full(N, np.nan, np.float32))
        mg.dispatch_gemv_noalloc(dev, dx, dW, y_new, N, K)
        dev.finish()
        assert_close(y_new.read(np.float32), oracle, TOL_F32, "noalloc fp32 at the size limit")
    K, N = 1024, 3000
    xb = O.bf16(O.uniform(K, 13))
    Wh = O.f16(O.uniform(K * N, 14))
    dx, dW = dev.array(xb, mg.BF16), dev.array(Wh, mg.F16, mg.LAYOUT_KN)
    y_ref, y_new = dev.empty(N, mg.F16), dev.empty(N, mg.F16)
    mg.dispatch_gemv(dev, None, dx, dW, y_ref, N, K).wait()
    ref = O.f16_to_f32(y_ref.read(np.uint16))
    oracle = O.gemv_f32(O.bf16_to_f32(xb), O.f16_to_f32(Wh), N, K)
    assert_close(ref, oracle, TOL_16, "dispatch_gemv bf16 x, f16 W and y")
    for _ in range(2):
        mg.dispatch_gemv_noalloc(dev, dx, dW, y_new, N, K)
        dev.finish()
        assert_close(O.f16_to_f32(y_new.read(np.uint16)), oracle, TOL_16, "noalloc bf16 x, f16 W and y")


def test_noalloc_allocates_nothing(dev):
    # the device's free memory is the same before and after a run of calls (cudaMalloc
    # reserves in 2 MiB pages, so any allocation would show); the allocating entry, for
    # contrast, may grow the library's scratch arena on its first split-K call
    import torch
    K, N = 4096, 16384
    dx = dev.array(O.uniform(K, 21), mg.F32)
    dW = dev.array(O.uniform(K * N, 22), mg.F32, mg.LAYOUT_KN)
    y = dev.empty(N, mg.F32)
    mg.dispatch_gemv_noalloc(dev, dx, dW, y, N, K)  # first use: the array's address lookup
    dev.finish()
    free0, _ = torch.cuda.mem_get_info(dev.ordinal)
    for _ in range(20):
        mg.dispatch_gemv_noalloc(dev, dx, dW, y, N, K)
    dev.finish()
    free1, _ = torch.cuda.mem_get_info(dev.ordinal)
    assert free1 == free0, (free0, free1)
    assert_close(y.read(np.float32), O.gemv_f32(O.uniform(K, 21), O.uniform(K * N, 22), N, K), TOL_F32,
                 "noalloc after 20 calls")


def test_noalloc_rejects_sizes_beyond_its_array(dev):
    N, K = 262145, 1  # one more column than the fixed scratch holds
    x, W, y = dev.empty(K, mg.F32), dev.empty(K * N, mg.F32), dev.empty(N, mg.F32)
    with pytest.raises(mg.MgpuError) as e:
        mg.dispatch_gemv_noalloc(dev, x, W, y, N, K)
    assert e.value.code == mg.ERR_INVALID_ARG and "262144" in str(e.value)
    dev.finish()
