"""Tolerance rule shared by the GPU parity tests.

Error norm: max_i |out_i - ref_i| divided by the max-norm of the fp32 reference output,
||ref||_inf = max_i |ref_i| (max-abs error relative to the output's norm).  Bounds (the
path's stated tolerances):
  fp32 path (fp32 activations, fp32 output)            <= 1e-4
  fp16 / bf16 tensor-core paths and 16-bit outputs     <= 1e-2
Integer / byte work (dequantisation, quantisation) is compared bit for bit.
"""
import numpy as np

TOL_F32 = 1e-4
TOL_16 = 1e-2


def rel_err(out, ref) -> float:
    out = np.asarray(out, np.float64).reshape(-1)
    ref = np.asarray(ref, np.float64).reshape(-1)
    return float(np.max(np.abs(out - ref)) / max(float(np.max(np.abs(ref))), 1e-30))


def assert_close(out, ref, tol, what=""):
    e = rel_err(out, ref)
    assert np.all(np.isfinite(out)), f"{what}: non-finite output"
    assert e <= tol, f"{what}: max|err|/max|ref| = {e:.3e} > {tol:.1e}"
    return e
