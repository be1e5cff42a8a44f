"""The bounds-checked build (libdcn_b200_bounds.so, -DDCN_DEBUG_BOUNDS): every
golden case in every dtype, and tensor-core shapes that take each producer
and dgrad epilogue variant (8, 16, 32 and 64 channels per offset group,
output-channel tails, far and out-of-image offsets), run forward and backward
through its C ABI.  No index of the gather and scatter math may leave its
tensor (dcn_debug_bounds_read counts zero), and the results still match the
float64 oracle within the parity tolerances (tests/_util.assert_close)."""
import ctypes
import os

import numpy as np
import pytest
import torch

from _util import assert_close, golden_cases, load_golden
from oracle import oracle

pytestmark = pytest.mark.gpu

DTYPES = {"float32": torch.float32, "float16": torch.float16, "bfloat16": torch.bfloat16}
CASES = [c for c in golden_cases() if c != "empty_batch"]

# (B, C, H, W, Co, groups, og, k, stride, pad, dil, mask, bias, offset_scale)
TC_SHAPES = {
    "c64_og1_wide": (2, 64, 12, 10, 64, 1, 1, 3, 1, 1, 1, True, True, 2.0),
    "c64_og2_sw32": (2, 64, 9, 11, 64, 1, 2, 3, 1, 1, 1, True, False, 3.0),
    "c64_og4_sw16": (2, 64, 9, 11, 96, 1, 4, 3, 1, 1, 1, True, True, 3.0),
    "c64_og8_quad_far": (2, 64, 9, 11, 64, 1, 8, 3, 1, 1, 1, True, False, 10.0),
    "c128_g2_og4_dil2": (2, 128, 10, 10, 128, 2, 4, 3, 1, 2, 2, True, True, 3.0),
    "c192_co96_tail": (3, 192, 7, 9, 96, 1, 2, 3, 1, 1, 1, True, True, 2.0),
    "c64_og8_outside": (1, 64, 6, 7, 64, 1, 8, 3, 1, 1, 1, True, True, 3e3),
    "c64_og1_outside": (1, 64, 6, 7, 64, 1, 1, 3, 2, 1, 1, False, True, 3e3),
}


@pytest.fixture(scope="module")
def blib():
    from mps_deform_conv import _abi
    assert os.path.exists(_abi.BOUNDS_LIB_PATH), "libdcn_b200_bounds.so not built (build.py)"
    lib = _abi.load_bounds()
    assert lib.dcn_debug_bounds_enabled() == 1
    _abi.bounds_record(lib)  # clear
    return lib


def _run_and_check(T, st, pd, dl, dtype, lib):
    from mps_deform_conv import _abi
    out = _abi.call_forward(T["input"], T["offset"], T["weight"], T["bias"], st, pd, dl, T["mask"], lib=lib)
    gi, goff, gw, gb, gm = _abi.call_backward(T["grad_output"], T["input"], T["offset"], T["weight"], st, pd, dl,
                                              T["mask"], with_bias=T["bias"] is not None, lib=lib)
    rec = _abi.bounds_record(lib)
    assert rec.count == 0, (f"{rec.count} out-of-bounds indices; first: site {rec.site}, index {rec.index}, "
                            f"width {rec.width}, extent {rec.extent}")
    ref = oracle.forward(T["input"], T["offset"], T["weight"], T["bias"], st, pd, dl, T["mask"])
    rgi, rgoff, rgw, rgb, rgm = oracle.backward(T["grad_output"], T["input"], T["offset"], T["weight"], st, pd, dl,
                                                T["mask"], T["bias"] is not None)
    assert_close(out, ref, dtype, "out")
    assert_close(gi, rgi, dtype, "gi")
    assert_close(goff, rgoff, dtype, "goff")
    assert_close(gw, rgw, dtype, "gw")
    if T["bias"] is not None:
        assert_close(gb, rgb, dtype, "gb")
    if T["mask"] is not None:
        assert_close(gm, rgm, dtype, "gm")


@pytest.mark.parametrize("dtype", list(DTYPES))
@pytest.mark.parametrize("name", CASES)
def test_bounds_golden(name, dtype, cuda, blib):
    d = load_golden(name)
    t = lambda a: None if a is None else torch.from_numpy(np.ascontiguousarray(a)).to(cuda, DTYPES[dtype])
    T = dict(input=t(d["input"]), offset=t(d["offset"]), weight=t(d["weight"]), bias=t(d.get("bias")),
             mask=t(d.get("mask")), grad_output=t(d["grad_output"]))
    geo = [tuple(int(v) for v in d[k]) for k in ("stride", "padding", "dilation")]
    _run_and_check(T, *geo, dtype, blib)


@pytest.mark.parametrize("dtype", ["float16", "bfloat16"])
@pytest.mark.parametrize("name", list(TC_SHAPES))
def test_bounds_tensor_core_shapes(name, dtype, cuda, blib):
    B, C, H, W, Co, G, og, k, s, p, dil, use_mask, use_bias, osc = TC_SHAPES[name]
    g = torch.Generator().manual_seed(3)
    Ho = (H + 2 * p - (dil * (k - 1) + 1)) // s + 1
    Wo = (W + 2 * p - (dil * (k - 1) + 1)) // s + 1
    dt = DTYPES[dtype]
    cv = lambda a: None if a is None else a.to(cuda, dt)
    off = torch.randn(B, 2 * og * k * k, Ho, Wo, generator=g) * osc
    if osc > 100:  # every sample far outside the image, and a few inside
        off[:, :, 0, 0] = torch.randn(B, 2 * og * k * k, generator=g)
    T = dict(input=cv(torch.randn(B, C, H, W, generator=g)),
             weight=cv(torch.randn(Co, C // G, k, k, generator=g) / np.sqrt(C // G * k * k)),
             offset=cv(off),
             mask=cv(torch.sigmoid(torch.randn(B, og * k * k, Ho, Wo, generator=g))) if use_mask else None,
             bias=cv(torch.randn(Co, generator=g) * 0.1) if use_bias else None,
             grad_output=cv(torch.randn(B, Co, Ho, Wo, generator=g)))
    from mps_deform_conv import _abi
    d = _abi.desc_for(T["input"], T["weight"], T["offset"], (s, s), (p, p), (dil, dil), T["mask"])
    assert blib.dcn_uses_tensor_cores(ctypes.byref(d)) == 1
    _run_and_check(T, (s, s), (p, p), (dil, dil), dtype, blib)
