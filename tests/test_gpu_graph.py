"""A training step (deform_conv2d forward + autograd backward) captured in a
CUDA graph and replayed with new data copied into its static inputs -- the
form in which bench.py times the step.

Each replay must give bitwise the forward output and grad_weight of an eager
step on the same data (both are deterministic on every path), and all five
gradients must match the float64 oracle within the parity tolerance (grad_input,
grad_offset and grad_mask are accumulated with atomics, so they are compared
with the oracle rather than bitwise with the eager step).
"""
import pytest
import torch

from _util import assert_close
from oracle import oracle

pytestmark = pytest.mark.gpu

DTYPES = {"bfloat16": torch.bfloat16, "float16": torch.float16, "float32": torch.float32}
# (B, C, H, W, Co, groups, offset groups, stride, pad, dilation): a small
# grouped tensor-core problem shaped like the large training step, and a
# plain one (fp32 runs it on the SIMT kernels)
SHAPES = {
    "g2_og4_dil2": (2, 128, 12, 12, 128, 2, 4, 1, 2, 2),
    "g1_og1": (2, 64, 10, 9, 64, 1, 1, 1, 1, 1),
}


def _data(shape, dtype, dev, seed):
    B, C, H, W, Co, G, og, s, p, d = shape
    g = torch.Generator().manual_seed(seed)
    Ho = (H + 2 * p - (d * 2 + 1)) // s + 1
    Wo = (W + 2 * p - (d * 2 + 1)) // s + 1
    t = {
        "input": torch.randn(B, C, H, W, generator=g),
        "offset": torch.randn(B, 2 * og * 9, Ho, Wo, generator=g) * 2.0,
        "mask": torch.sigmoid(torch.randn(B, og * 9, Ho, Wo, generator=g)),
        "weight": torch.randn(Co, C // G, 3, 3, generator=g) / (C // G * 9) ** 0.5,
        "bias": torch.randn(Co, generator=g) * 0.01,
        "grad_output": torch.randn(B, Co, Ho, Wo, generator=g),
    }
    return {k: v.to(dev, dtype) for k, v in t.items()}


@pytest.mark.parametrize("dtype", list(DTYPES))
@pytest.mark.parametrize("shape", list(SHAPES))
def test_graph_replayed_training_step(shape, dtype, cuda):
    import mps_deform_conv as mdc
    dt = DTYPES[dtype]
    geo = SHAPES[shape]
    st, pd, dl = (geo[7],) * 2, (geo[8],) * 2, (geo[9],) * 2
    static = _data(geo, dt, cuda, seed=0)
    names = ("input", "offset", "weight", "bias", "mask")
    leaves = [static[k].requires_grad_(True) for k in names]

    def step(ts):
        out = mdc.deform_conv2d(ts[0], ts[1], ts[2], ts[3], st, pd, dl, ts[4])
        return (out,) + torch.autograd.grad(out, ts, static["grad_output"])

    side = torch.cuda.Stream(cuda)
    side.wait_stream(torch.cuda.current_stream(cuda))
    with torch.cuda.stream(side):
        for _ in range(3):
            step(leaves)
    torch.cuda.current_stream(cuda).wait_stream(side)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        captured = step(leaves)

    for seed in (1, 2):  # new data in the same static buffers, weights included
        new = _data(geo, dt, cuda, seed=seed)
        with torch.no_grad():
            for k in names + ("grad_output",):
                static[k].copy_(new[k])
        graph.replay()
        torch.cuda.synchronize()
        got = [t.clone() for t in captured]
        eager = step([new[k].clone().requires_grad_(True) for k in names])
        torch.cuda.synchronize()
        mdc._get_lib().device_status()
        assert torch.equal(got[0], eager[0]), "forward differs from the eager step"
        assert torch.equal(got[3], eager[3]), "grad_weight differs from the eager step"
        ref_out = oracle.forward(new["input"], new["offset"], new["weight"], new["bias"], st, pd, dl, new["mask"])
        rgi, rgoff, rgw, rgb, rgm = oracle.backward(new["grad_output"], new["input"], new["offset"], new["weight"],
                                                    st, pd, dl, new["mask"], True)
        assert_close(got[0], ref_out, dtype, f"replay {seed} output")
        assert_close(got[1], rgi, dtype, f"replay {seed} grad_input")
        assert_close(got[2], rgoff, dtype, f"replay {seed} grad_offset")
        assert_close(got[3], rgw, dtype, f"replay {seed} grad_weight")
        assert_close(got[4], rgb, dtype, f"replay {seed} grad_bias")
        assert_close(got[5], rgm, dtype, f"replay {seed} grad_mask")
    del graph
