"""The registered operators (mps_deform_conv.ops) on the GPU.

* torch.library.opcheck on both operators: schema, fake (meta) implementation
  against the real kernels' outputs, autograd registration, and the operator
  run through AOT dispatch with dynamic shapes.
* ModulatedDeformConv2d compiled with torch.compile(fullgraph=True) -- the
  route that keeps the operator pair in one graph -- against the eager module:
  output and the gradients of the input and of both weights.
"""
import pytest
import torch

from _util import assert_close

pytestmark = pytest.mark.gpu

ops = torch.ops.mps_deform_conv
DTYPES = {"bfloat16": torch.bfloat16, "float32": torch.float32}


def _args(dtype, dev, mask=True, bias=True):
    g = torch.Generator().manual_seed(5)
    B, C, H, W, Co, G, og = 2, 64, 8, 9, 64, 1, 2
    x = torch.randn(B, C, H, W, generator=g)
    w = torch.randn(Co, C // G, 3, 3, generator=g) / 24.0
    off = torch.randn(B, 2 * og * 9, H, W, generator=g) * 1.5
    m = torch.sigmoid(torch.randn(B, og * 9, H, W, generator=g)) if mask else torch.empty(0)
    b = torch.randn(Co, generator=g) * 0.1 if bias else torch.empty(0)
    cv = lambda t: t.to(dev, dtype)
    return [cv(x), cv(w), cv(off), cv(m), cv(b), 1, 1, 1, 1, 1, 1, G, og, mask]


@pytest.mark.parametrize("dtype", list(DTYPES))
@pytest.mark.parametrize("mask", [True, False])
def test_opcheck_forward(dtype, mask, cuda):
    args = _args(DTYPES[dtype], cuda, mask=mask)
    for i in range(5):
        if args[i].numel():
            args[i].requires_grad_(True)
    torch.library.opcheck(ops.deform_conv2d_forward.default, args)


@pytest.mark.parametrize("dtype", list(DTYPES))
def test_opcheck_backward(dtype, cuda):
    args = _args(DTYPES[dtype], cuda)
    g = torch.Generator().manual_seed(9)
    grad = torch.randn(2, 64, 8, 9, generator=g).to(cuda, DTYPES[dtype])
    torch.library.opcheck(ops.deform_conv2d_backward.default, [grad] + args,
                          test_utils=("test_schema", "test_faketensor", "test_autograd_registration"))


@pytest.mark.parametrize("backend", ["aot_eager", "inductor"])
def test_compiled_module_matches_eager(backend, cuda):
    import mps_deform_conv as mdc
    torch.manual_seed(3)
    mod = mdc.ModulatedDeformConv2d(64, 64, 3, padding=1, offset_groups=2).to(cuda, torch.bfloat16)
    with torch.no_grad():  # a non-zero offset head, so the sampling points move
        mod.offset_conv.weight.normal_(0.0, 0.05)
    x = torch.randn(2, 64, 12, 10, device=cuda, dtype=torch.bfloat16)
    go = torch.randn(2, 64, 12, 10, device=cuda, dtype=torch.bfloat16)

    def run(fn):
        xi = x.clone().requires_grad_(True)
        mod.zero_grad(set_to_none=True)
        out = fn(xi)
        out.backward(go)
        return out.detach(), xi.grad, mod.weight.grad.clone(), mod.offset_conv.weight.grad.clone()

    eager = run(mod)
    torch._dynamo.reset()
    compiled = torch.compile(mod, fullgraph=True, backend=backend)
    got = run(compiled)
    torch.cuda.synchronize()
    for name, a, b in zip(("output", "grad_input", "grad_weight", "grad_offset_conv_weight"), got, eager):
        assert torch.isfinite(a).all(), name
        assert_close(a, b, "bfloat16", f"{backend} {name}")
    torch._dynamo.reset()
