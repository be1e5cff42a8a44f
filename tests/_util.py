"""Shared helpers for the parity tests."""
import glob
import os

import numpy as np

GOLDEN_DIR = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")

# Tolerances (normwise relative error, see rel_err): fp32 results must match the
# float64 oracle within 1e-4, fp16/bf16 results within 1e-2.
TOL = {"float32": 1e-4, "float16": 1e-2, "bfloat16": 1e-2}


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
