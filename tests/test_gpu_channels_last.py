"""Channels-last (NHWC) input, output and gradients.

The tensor-core kernels read a channels_last input in place (no repack), write
a channels_last output, take a channels_last grad_output as the pixel-major
GEMM operand and return grad_input channels_last.  Results must equal the
NCHW path: the forward bitwise (same gather and epilogue arithmetic), and
grad_weight bitwise (deterministic reduction over the same operands).  The
atomically accumulated gradients match within half the dtype tolerance, and
everything matches the float64 oracle within the dtype tolerance.  Problems outside the
tensor-core path run on NCHW copies and still return channels_last outputs.
"""
import pytest
import torch

from _util import TOL, assert_close, rel_err, to_np
from oracle import oracle
from test_gpu_tc import SHAPES, _make

pytestmark = pytest.mark.gpu

DTYPES = {"float16": torch.float16, "bfloat16": torch.bfloat16}
CL = torch.channels_last


def _run(T, in_cl, go_cl):
    import mps_deform_conv as mdc
    st, pd, dl = T["stride"], T["padding"], T["dilation"]
    x = T["input"].contiguous(memory_format=CL) if in_cl else T["input"].contiguous()
    leaves = {"input": x.detach().clone(memory_format=torch.preserve_format).requires_grad_(True)}
    for k in ("offset", "weight", "bias", "mask"):
        if T[k] is not None:
            leaves[k] = T[k].detach().clone().requires_grad_(True)
    out = mdc.deform_conv2d(leaves["input"], leaves["offset"], leaves["weight"], leaves.get("bias"), st, pd, dl,
                            leaves.get("mask"))
    go = T["grad_output"].contiguous(memory_format=CL) if go_cl else T["grad_output"].contiguous()
    keys = list(leaves)
    grads = torch.autograd.grad(out, [leaves[k] for k in keys], go)
    torch.cuda.synchronize()
    mdc._get_lib().device_status()
    return out, dict(zip(keys, grads))


@pytest.mark.parametrize("dtype", list(DTYPES))
@pytest.mark.parametrize("name", ["c64_og1", "c128_g2_og4_dil2", "c64_og8_far", "c192_co96_tail"])
def test_channels_last_matches_nchw_and_oracle(name, dtype, cuda):
    T = _make(SHAPES[name], DTYPES[dtype], cuda, seed=41)
    out0, g0 = _run(T, False, False)
    for in_cl, go_cl in ((True, True), (True, False), (False, True)):
        out, g = _run(T, in_cl, go_cl)
        if in_cl:
            assert out.is_contiguous(memory_format=CL) and not out.is_contiguous()
            assert g["input"].is_contiguous(memory_format=CL)
        assert torch.equal(out, out0), (in_cl, go_cl)
        assert torch.equal(g["weight"], g0["weight"]), (in_cl, go_cl)
        # accumulated with fp32 atomics in run-dependent order: last-bit flips
        # after rounding to 16 bits (a layout error would be of order 1)
        for k in ("input", "offset", "mask", "bias"):
            if k in g:
                assert rel_err(to_np(g[k]), to_np(g0[k])) <= TOL[dtype] / 2, (k, in_cl, go_cl)
    st, pd, dl = T["stride"], T["padding"], T["dilation"]
    ref = oracle.forward(T["input"], T["offset"], T["weight"], T["bias"], st, pd, dl, T["mask"])
    rgi, rgoff, rgw, rgb, rgm = oracle.backward(T["grad_output"], T["input"], T["offset"], T["weight"], st, pd, dl,
                                                T["mask"], T["bias"] is not None)
    tol = TOL[dtype]
    assert_close(out, ref, dtype, 'out')
    assert_close(g["input"], rgi, dtype, 'g["input"]')
    assert_close(g["offset"], rgoff, dtype, 'g["offset"]')
    assert_close(g["weight"], rgw, dtype, 'g["weight"]')


def test_channels_last_fp32_falls_back_and_keeps_format(cuda):
    """fp32 runs on the SIMT kernels (NCHW copies); the output still comes
    back channels_last and matches the NCHW result."""
    T = _make(SHAPES["c64_og1"], torch.float32, cuda, seed=43)
    out0, g0 = _run(T, False, False)
    out, g = _run(T, True, True)
    assert out.is_contiguous(memory_format=CL)
    assert rel_err(to_np(out), to_np(out0)) <= 1e-6
    for k in g0:
        assert rel_err(to_np(g[k]), to_np(g0[k])) <= 1e-5, k


def test_channels_last_unaligned_storage(cuda):
    """A channels_last input whose data starts 2 bytes past a 16-byte boundary
    is copied to an aligned one (the gather reads 16-byte vectors)."""
    import mps_deform_conv as mdc
    T = _make(SHAPES["c64_og1"], torch.bfloat16, cuda, seed=47)
    x = T["input"].contiguous(memory_format=CL)
    buf = torch.empty(x.numel() + 1, dtype=x.dtype, device=cuda)
    B, C, H, W = x.shape
    xu = buf[1:].view(B, H, W, C).permute(0, 3, 1, 2)  # channels_last strides, 2-byte offset
    xu.copy_(x)
    assert xu.is_contiguous(memory_format=CL) and xu.data_ptr() % 16 == 2
    st, pd, dl = T["stride"], T["padding"], T["dilation"]
    a = mdc.deform_conv2d(x, T["offset"], T["weight"], T["bias"], st, pd, dl, T["mask"])
    b = mdc.deform_conv2d(xu, T["offset"], T["weight"], T["bias"], st, pd, dl, T["mask"])
    torch.cuda.synchronize()
    assert torch.equal(a, b)


def test_channels_last_fused_head_module(cuda):
    """ModulatedDeformConv2d on a channels_last input: fused head route and
    the reference's composition agree, and the output is channels_last."""
    import mps_deform_conv as mdc
    torch.manual_seed(7)
    mod = mdc.ModulatedDeformConv2d(64, 64, 3, padding=1)
    with torch.no_grad():
        mod.offset_conv.weight.normal_(0, 0.05)
        mod.offset_conv.bias.normal_(0, 0.5)
    mod = mod.to(cuda, torch.bfloat16).to(memory_format=CL)
    x0 = torch.randn(2, 64, 12, 10, device=cuda, dtype=torch.bfloat16).contiguous(memory_format=CL)
    res = {}
    for fused in (True, False):
        mdc.set_head_fusion(fused)
        try:
            mod.zero_grad(set_to_none=True)
            x = x0.clone(memory_format=torch.preserve_format).requires_grad_(True)
            out = mod(x)
            out.float().square().mean().backward()
        finally:
            mdc.set_head_fusion(True)
        res[fused] = [out.detach(), x.grad, mod.weight.grad, mod.offset_conv.weight.grad]
    torch.cuda.synchronize()
    assert res[True][0].is_contiguous(memory_format=CL)
    for i, (a, b) in enumerate(zip(res[True], res[False])):
        assert rel_err(to_np(a), to_np(b)) <= 2e-2, i
