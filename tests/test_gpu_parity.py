"""GPU parity: the CUDA kernels against the float64 oracle and the torchvision
golden fixtures, for every dtype, through the C ABI (ctypes, libdcn_b200.so)
and through the Python API (mps_deform_conv, autograd).

Tolerance: normwise relative error (tests/_util.rel_err) <= 1e-4 for fp32 and
<= 1e-2 for fp16/bf16, per output and per gradient.  For fp16/bf16 the oracle
runs on the same rounded inputs the GPU sees.
"""
import ctypes

import numpy as np
import pytest
import torch

from _util import TOL, golden_cases, load_golden, assert_close, rel_err, to_np
from oracle import oracle

pytestmark = pytest.mark.gpu

DTYPES = {"float32": torch.float32, "float16": torch.float16, "bfloat16": torch.bfloat16}
CASES = [c for c in golden_cases() if c != "empty_batch"]


def _tensors(d, dtype, dev):
    t = lambda a: None if a is None else torch.from_numpy(np.ascontiguousarray(a)).to(dev, dtype)
    return dict(input=t(d["input"]), offset=t(d["offset"]), weight=t(d["weight"]),
                bias=t(d.get("bias")), mask=t(d.get("mask")), grad_output=t(d["grad_output"]))


def _geo(d):
    return tuple(int(v) for v in d["stride"]), tuple(int(v) for v in d["padding"]), \
        tuple(int(v) for v in d["dilation"])


@pytest.mark.parametrize("dtype", list(DTYPES))
@pytest.mark.parametrize("name", CASES)
def test_abi_forward_backward_vs_oracle(name, dtype, cuda):
    from mps_deform_conv import _abi
    d = load_golden(name)
    st, pd, dl = _geo(d)
    T = _tensors(d, DTYPES[dtype], cuda)
    out = _abi.call_forward(T["input"], T["offset"], T["weight"], T["bias"], st, pd, dl, T["mask"])
    gi, goff, gw, gb, gm = _abi.call_backward(T["grad_output"], T["input"], T["offset"], T["weight"],
                                              st, pd, dl, T["mask"], with_bias=T["bias"] is not None)
    torch.cuda.synchronize()
    # oracle on exactly the values the GPU saw
    ref_out = oracle.forward(T["input"], T["offset"], T["weight"], T["bias"], st, pd, dl, T["mask"])
    rgi, rgoff, rgw, rgb, rgm = oracle.backward(T["grad_output"], T["input"], T["offset"], T["weight"],
                                                st, pd, dl, T["mask"], T["bias"] is not None)
    tol = TOL[dtype]
    assert_close(out, ref_out, dtype, 'out')
    assert_close(gi, rgi, dtype, 'gi')
    assert_close(goff, rgoff, dtype, 'goff')
    assert_close(gw, rgw, dtype, 'gw')
    if T["bias"] is not None:
        assert_close(gb, rgb, dtype, 'gb')
    if T["mask"] is not None:
        assert_close(gm, rgm, dtype, 'gm')
    if dtype == "float32":  # and directly against the torchvision fixtures
        assert_close(out, d["output"], dtype, 'out')
        assert_close(gi, d["grad_input"], dtype, 'gi')
        assert_close(goff, d["grad_offset"], dtype, 'goff')
        assert_close(gw, d["grad_weight"], dtype, 'gw')


@pytest.mark.parametrize("dtype", list(DTYPES))
@pytest.mark.parametrize("name", ["mask_bias_g2_og2", "stride2_dil2", "basic_v1", "far_offsets_og4"])
def test_python_api_autograd_vs_oracle(name, dtype, cuda):
    import mps_deform_conv as mdc
    d = load_golden(name)
    st, pd, dl = _geo(d)
    T = _tensors(d, DTYPES[dtype], cuda)
    leaves = {k: T[k].clone().requires_grad_(True) for k in ("input", "offset", "weight", "bias", "mask")
              if T[k] is not None}
    out = mdc.deform_conv2d(leaves["input"], leaves["offset"], leaves["weight"], leaves.get("bias"),
                            st, pd, dl, leaves.get("mask"))
    out.backward(T["grad_output"])
    ref_out = oracle.forward(T["input"], T["offset"], T["weight"], T["bias"], st, pd, dl, T["mask"])
    rgi, rgoff, rgw, rgb, rgm = oracle.backward(T["grad_output"], T["input"], T["offset"], T["weight"],
                                                st, pd, dl, T["mask"], T["bias"] is not None)
    tol = TOL[dtype]
    assert out.dtype == DTYPES[dtype] and out.is_cuda
    assert_close(out, ref_out, dtype, 'out')
    assert_close(leaves["input"].grad, rgi, dtype, 'leaves["input"].grad')
    assert_close(leaves["offset"].grad, rgoff, dtype, 'leaves["offset"].grad')
    assert_close(leaves["weight"].grad, rgw, dtype, 'leaves["weight"].grad')
    if "bias" in leaves:
        assert_close(leaves["bias"].grad, rgb, dtype, 'leaves["bias"].grad')
    if "mask" in leaves:
        assert_close(leaves["mask"].grad, rgm, dtype, 'leaves["mask"].grad')


@pytest.mark.parametrize("dtype", list(DTYPES))
def test_reference_column_interface(dtype, cuda):
    """The reference FFI's column-buffer functions: deformable_im2col,
    deform_conv2d_backward_input, deform_conv2d_backward_offset_mask."""
    import mps_deform_conv as mdc
    lib = mdc._get_lib()
    d = load_golden("mask_bias_g2_og2")
    st, pd, dl = _geo(d)
    T = _tensors(d, DTYPES[dtype], cuda)
    kh, kw = T["weight"].shape[2:]
    og = T["offset"].shape[1] // (2 * kh * kw)
    x, off, m = T["input"], T["offset"], T["mask"]
    cols = lib.deformable_im2col(x, off, m, kh, kw, st[0], st[1], pd[0], pd[1], dl[0], dl[1], og, True)
    rcols = oracle.im2col(x, off, m, kh, kw, st, pd, dl, og)
    assert tuple(cols.shape) == rcols.shape
    assert_close(cols, rcols, dtype, 'cols')
    gcol = torch.randn(cols.shape, device=cuda, dtype=torch.float32).to(DTYPES[dtype])
    gi = lib.deform_conv2d_backward_input(gcol, x, off, m, x.shape[2], x.shape[3], st[0], st[1], pd[0],
                                          pd[1], dl[0], dl[1], kh, kw, og, True)
    rgi = oracle.col2im(gcol, tuple(x.shape), off, m, kh, kw, st, pd, dl, og)
    assert_close(gi, rgi, dtype, 'gi')
    goff, gm = lib.deform_conv2d_backward_offset_mask(gcol, x, off, m, kh, kw, st[0], st[1], pd[0],
                                                      pd[1], dl[0], dl[1], og, True)
    rgoff, rgm = oracle.col2im_coord(gcol, x, off, m, kh, kw, st, pd, dl, og)
    assert_close(goff, rgoff, dtype, 'goff')
    assert_close(gm, rgm, dtype, 'gm')


def test_empty_batch(cuda):
    import mps_deform_conv as mdc
    d = load_golden("empty_batch")
    st, pd, dl = _geo(d)
    T = _tensors(d, torch.float32, cuda)
    w = T["weight"].clone().requires_grad_(True)
    b = T["bias"].clone().requires_grad_(True)
    out = mdc.deform_conv2d(T["input"], T["offset"], w, b, st, pd, dl, T["mask"])
    assert tuple(out.shape) == d["output"].shape
    out.sum().backward()
    assert torch.count_nonzero(w.grad) == 0 and torch.count_nonzero(b.grad) == 0


@pytest.mark.parametrize("shape", [(1, 64, 16, 16, 64, 1), (2, 32, 12, 10, 48, 2), (3, 40, 9, 11, 200, 1)])
def test_fp32_tensor_core_gemms_vs_oracle(shape, cuda):
    """fp32 problems materialize their columns and run the three GEMMs on the
    tensor cores (tf32 MMAs with the hi/lo split): forward bitwise repeatable,
    forward and all five gradients at fp32 tolerance against the oracle.
    The shapes cover row/column tile tails (200 output channels = a 128 and a
    72-wide tile; K = 40*9 = 360, not a multiple of the 32-deep K chunk) and
    groups."""
    from mps_deform_conv import _abi
    import mps_deform_conv as mdc
    B, C, H, W, Co, G = shape
    g = torch.Generator().manual_seed(53)
    x = torch.randn(B, C, H, W, generator=g)
    w = torch.randn(Co, C // G, 3, 3, generator=g) / np.sqrt(C // G * 9)
    off = torch.randn(B, 18, H, W, generator=g) * 1.5
    m = torch.sigmoid(torch.randn(B, 9, H, W, generator=g))
    b = torch.randn(Co, generator=g) * 0.1
    go = torch.randn(B, Co, H, W, generator=g)
    d = _abi.desc_for(x, w, off, (1, 1), (1, 1), (1, 1), m)
    lib = _abi.load()
    assert lib.dcn_forward_workspace_size(ctypes.byref(d)) == (4 * C * 9 * B * H * W + 255) // 256 * 256  # fp32 columns
    dev = [t.to(cuda) for t in (x, off, w, b, m)]
    a = _abi.call_forward(dev[0], dev[1], dev[2], dev[3], (1, 1), (1, 1), (1, 1), dev[4])
    a2 = _abi.call_forward(dev[0], dev[1], dev[2], dev[3], (1, 1), (1, 1), (1, 1), dev[4])
    torch.cuda.synchronize()
    assert torch.equal(a, a2)
    ref = oracle.forward(x, off, w, b, (1, 1), (1, 1), (1, 1), m)
    assert_close(a, ref, "float32", "output")
    leaves = [t.clone().requires_grad_(True) for t in dev]
    out = mdc.deform_conv2d(leaves[0], leaves[1], leaves[2], leaves[3], 1, 1, 1, leaves[4])
    grads = torch.autograd.grad(out, leaves, go.to(cuda))
    refs = oracle.backward(go.double(), x.double(), off.double(), w.double(), (1, 1), (1, 1), (1, 1),
                           m.double(), True)
    for nm, gv, rv in zip(("grad_input", "grad_offset", "grad_weight", "grad_bias", "grad_mask"),
                          (grads[0], grads[1], grads[2], grads[3], grads[4]), refs):
        assert_close(gv, rv, "float32", nm)


def test_fp32_training_state_keeps_the_columns(cuda):
    """fp32 problems keep the forward's fp32 columns as the training state
    (dcn_saved_state_bytes = the column bytes); the backward's weight gradient
    reads them instead of gathering again, bitwise the same as with the cache
    off, and matches the oracle."""
    from mps_deform_conv import _abi
    import mps_deform_conv as mdc
    B, C, H, W, Co = 2, 48, 10, 12, 40
    g = torch.Generator().manual_seed(61)
    x = torch.randn(B, C, H, W, generator=g)
    w = torch.randn(Co, C, 3, 3, generator=g) / np.sqrt(C * 9)
    off = torch.randn(B, 18, H, W, generator=g) * 1.5
    m = torch.sigmoid(torch.randn(B, 9, H, W, generator=g))
    b = torch.randn(Co, generator=g) * 0.1
    go = torch.randn(B, Co, H, W, generator=g)
    d = _abi.desc_for(x, w, off, (1, 1), (1, 1), (1, 1), m)
    assert _abi.load().dcn_saved_state_bytes(ctypes.byref(d)) == (4 * C * 9 * B * H * W + 255) // 256 * 256
    runs = []
    try:
        for cache in (True, False):
            mdc.set_training_cache(cache)
            leaves = [t.to(cuda).requires_grad_(True) for t in (x, off, w, b, m)]
            out = mdc.deform_conv2d(leaves[0], leaves[1], leaves[2], leaves[3], 1, 1, 1, leaves[4])
            runs.append([out] + list(torch.autograd.grad(out, leaves, go.to(cuda))))
    finally:
        mdc.set_training_cache(True)
    # output, grad_offset and grad_mask are computed in a fixed order: bitwise
    # equal; grad_input and grad_weight are accumulated with atomics
    for i in (0, 2, 5):
        assert torch.equal(runs[0][i], runs[1][i])
    for i in (1, 3, 4):
        assert rel_err(runs[0][i].double().cpu().numpy(), runs[1][i].double().cpu().numpy()) < 1e-6
    refs = oracle.backward(go.double(), x.double(), off.double(), w.double(), (1, 1), (1, 1), (1, 1),
                           m.double(), True)
    for nm, gv, rv in zip(("grad_input", "grad_offset", "grad_weight", "grad_bias", "grad_mask"), runs[0][1:], refs):
        assert_close(gv, rv, "float32", nm)


def test_device_status_clean_after_runs(cuda):
    import mps_deform_conv as mdc
    mdc._get_lib().device_status()
