"""Registered operators (mps_deform_conv.ops) on the CPU: schemas, fake
implementations through autograd on meta tensors, and torch.compile tracing
without graph breaks.  The kernels themselves need a CUDA device: a CPU tensor
reaching the operator fails loudly."""
import pytest
import torch
import torch._dynamo.testing

import mps_deform_conv as mdc

ops = torch.ops.mps_deform_conv


def test_schemas():
    fwd = str(ops.deform_conv2d_forward.default._schema)
    bwd = str(ops.deform_conv2d_backward.default._schema)
    args = ("Tensor input, Tensor weight, Tensor offset, Tensor mask, Tensor bias, SymInt stride_h, SymInt stride_w, "
            "SymInt pad_h, SymInt pad_w, SymInt dilation_h, SymInt dilation_w, SymInt groups, SymInt offset_groups, "
            "bool use_mask")
    assert fwd == f"mps_deform_conv::deform_conv2d_forward({args}) -> Tensor"
    assert bwd == (f"mps_deform_conv::deform_conv2d_backward(Tensor grad, {args}) "
                   "-> (Tensor, Tensor, Tensor, Tensor, Tensor)")


def _meta(*shape, grad=True):
    return torch.empty(*shape, device="meta", requires_grad=grad)


@pytest.mark.parametrize("B,C,H,W,Co,G,og,k,s,p,d,mask,bias", [
    (2, 8, 10, 12, 6, 1, 2, 3, 1, 1, 1, True, True),
    (1, 16, 9, 7, 8, 2, 4, 3, 2, 1, 2, False, True),
    (3, 4, 5, 6, 4, 1, 1, 1, 1, 0, 1, True, False),
    (0, 8, 6, 6, 8, 2, 1, 3, 1, 1, 1, True, True),
])
def test_meta_forward_and_gradient_shapes(B, C, H, W, Co, G, og, k, s, p, d, mask, bias):
    Ho = (H + 2 * p - (d * (k - 1) + 1)) // s + 1
    Wo = (W + 2 * p - (d * (k - 1) + 1)) // s + 1
    x, w = _meta(B, C, H, W), _meta(Co, C // G, k, k)
    off = _meta(B, 2 * og * k * k, Ho, Wo)
    m = _meta(B, og * k * k, Ho, Wo) if mask else None
    b = _meta(Co) if bias else None
    out = mdc.deform_conv2d(x, off, w, b, (s, s), (p, p), (d, d), m)
    assert out.shape == (B, Co, Ho, Wo) and out.device.type == "meta"
    leaves = [t for t in (x, off, w, b, m) if t is not None]
    grads = torch.autograd.grad(out, leaves, torch.empty_like(out))
    for t, g in zip(leaves, grads):
        assert g.shape == t.shape


def test_meta_validation_still_applies():
    x, w = _meta(1, 6, 5, 5), _meta(4, 4, 3, 3)  # 6 input channels, weight expects a divisor of 6 times 4
    with pytest.raises(ValueError):
        mdc.deform_conv2d(x, _meta(1, 18, 3, 3), w)


def test_compile_traces_module_without_graph_break():
    mod = mdc.ModulatedDeformConv2d(8, 6, 3, padding=1, offset_groups=2).to("meta")
    x = _meta(2, 8, 10, 12)
    counter = torch._dynamo.testing.CompileCounter()
    compiled = torch.compile(mod, fullgraph=True, backend=counter)
    out = compiled(x)
    assert out.shape == (2, 6, 10, 12)
    assert counter.frame_count == 1
    torch._dynamo.reset()
    compiled = torch.compile(mod, fullgraph=True, backend="aot_eager")
    out = compiled(x)
    out.sum().backward()
    assert x.grad.shape == x.shape and mod.weight.grad.shape == mod.weight.shape
    assert mod.offset_conv.weight.grad.shape == mod.offset_conv.weight.shape
    torch._dynamo.reset()


def test_cpu_tensors_fail_loudly():
    x, w = torch.randn(1, 4, 5, 5), torch.randn(4, 4, 3, 3)
    off, e = torch.zeros(1, 18, 5, 5), torch.empty(0)
    with pytest.raises(RuntimeError, match="CUDA"):
        ops.deform_conv2d_forward(x, w, off, e, e, 1, 1, 1, 1, 1, 1, 1, 1, False)
