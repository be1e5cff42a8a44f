"""Shared helpers for the parity tests."""
import glob
import os

import numpy as np

GOLDEN_DIR = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")

# Tolerances (normwise relative error, see rel_err): fp32 results must match the
# float64 oracle within 1e-4, fp16/bf16 results within 1e-2.
TOL = {"float32": 1e-4, "float16": 1e-2, "bfloat16": 1e-2}


# Elementwise bound checked beside the normwise one (assert_close):
#   |a - b| <= ATOL * max|b| + RTOL * |b|      (b is the reference)
# RTOL is the normwise tolerance itself.  ATOL bounds the error of elements that
# are small against the tensor's largest: half the normwise tolerance for
# bf16 (its 16-bit column operand alone costs ~3e-3 normwise), a fifth for
# fp16 (eight times finer rounding), a tenth for fp32.
RTOL = dict(TOL)
ATOL = {"float32": 1e-5, "float16": 2e-3, "bfloat16": 5e-3}


def assert_close(actual, ref, dtype: str, what: str = "") -> None:
    """Normwise (rel_err <= TOL) and elementwise (ATOL/RTOL above) parity of
    `actual` against the reference `ref`; NaN or Inf anywhere fails."""
    a = to_np(actual)
    b = to_np(ref)
    assert a.shape == b.shape, f"{what}: shape {a.shape} != {b.shape}"
    if b.size == 0:
        return
    scale = max(float(np.abs(b).max()), 1e-30)
    err = np.abs(a - b)
    nw = float(err.max()) / scale
    assert nw <= TOL[dtype], f"{what}: normwise error {nw:.3e} > {TOL[dtype]:.0e}"
    excess = err - RTOL[dtype] * np.abs(b)
    need = float(excess.max()) / scale
    at = np.unravel_index(int(np.argmax(excess)), b.shape)
    assert need <= ATOL[dtype], (f"{what}: elementwise check needs atol {need:.3e} > {ATOL[dtype]:.0e} "
                                 f"at {at}: got {a[at]:.6e}, reference {b[at]:.6e}")


def rel_err(a, b) -> float:
    """Normwise relative error max|a - b| / max(max|b|, 1e-30) (b is the reference)."""
    a = np.asarray(a, dtype=np.float64)
    b = np.asarray(b, dtype=np.float64)
    if b.size == 0:
        return 0.0
    return float(np.abs(a - b).max() / max(np.abs(b).max(), 1e-30))


def to_np(t):
    if t is None:
        return None
    if hasattr(t, "detach"):
        return t.detach().float().cpu().double().numpy()
    return np.asarray(t, dtype=np.float64)


def golden_cases():
    return sorted(os.path.basename(p)[:-4] for p in glob.glob(os.path.join(GOLDEN_DIR, "*.npz")))


def load_golden(name):
    d = np.load(os.path.join(GOLDEN_DIR, name + ".npz"))
    return {k: d[k] for k in d.files}
