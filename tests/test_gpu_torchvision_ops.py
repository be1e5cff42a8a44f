"""torchvision.ops.deform_conv2d served by this package's kernels after
mps_deform_conv.torchvision_ops.register_torchvision_ops(): forward and all
gradients through torchvision's own Python API and autograd, against the
float64 oracle, and proof that the library's kernels ran (launch count)."""
import pytest
import torch

from _util import TOL, assert_close, rel_err, to_np
from oracle import oracle

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("dtype,C,mask", [(torch.bfloat16, 64, True), (torch.float32, 8, True),
                                          (torch.float16, 128, False)])
def test_torchvision_deform_conv2d_runs_on_b200_kernels(dtype, C, mask, cuda):
    from torchvision.ops import deform_conv2d as tv_deform_conv2d
    from mps_deform_conv import _abi
    from mps_deform_conv.torchvision_ops import register_torchvision_ops
    register_torchvision_ops()
    g = torch.Generator().manual_seed(21)
    B, H, W, Co, og = 2, 9, 10, 64, 2
    x = torch.randn(B, C, H, W, generator=g)
    w = torch.randn(Co, C, 3, 3, generator=g) / (3 * C ** 0.5)
    b = torch.randn(Co, generator=g) * 0.1
    off = torch.randn(B, 2 * og * 9, H, W, generator=g) * 2
    m = torch.sigmoid(torch.randn(B, og * 9, H, W, generator=g)) if mask else None
    go = torch.randn(B, Co, H, W, generator=g)
    cv = lambda t: None if t is None else t.to(cuda, dtype)
    X, Wt, Bt, OFF, M, GO = (cv(t) for t in (x, w, b, off, m, go))
    leaves = [t.clone().requires_grad_(True) if t is not None else None for t in (X, OFF, Wt, Bt, M)]
    n0 = _abi.launch_count()
    out = tv_deform_conv2d(leaves[0], leaves[1], leaves[2], leaves[3], padding=(1, 1), mask=leaves[4])
    out.backward(GO)
    torch.cuda.synchronize()
    assert _abi.launch_count() > n0  # this library's kernels served the call
    DTN = {torch.float32: "float32", torch.float16: "float16", torch.bfloat16: "bfloat16"}[dtype]
    ref = oracle.forward(X, OFF, Wt, Bt, 1, 1, 1, M)
    rgi, rgoff, rgw, rgb, rgm = oracle.backward(GO, X, OFF, Wt, 1, 1, 1, M, True)
    assert_close(out, ref, DTN, 'out')
    assert_close(leaves[0].grad, rgi, DTN, 'leaves[0].grad')
    assert_close(leaves[1].grad, rgoff, DTN, 'leaves[1].grad')
    assert_close(leaves[2].grad, rgw, DTN, 'leaves[2].grad')
    assert_close(leaves[3].grad, rgb, DTN, 'leaves[3].grad')
    if mask:
        assert_close(leaves[4].grad, rgm, DTN, 'leaves[4].grad')
