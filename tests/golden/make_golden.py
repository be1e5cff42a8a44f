"""Generate the golden fixtures in tests/golden/ from torchvision on CPU (float64).

torchvision.ops.deform_conv2d is the ground truth that mps-deform-conv declares
parity with (its README's torchvision comparison; its kernels restate
torchvision's deformable_im2col / col2im / col2im_coord).  Each fixture holds
seeded float64 inputs, the forward output and all five gradients for a seeded
grad_output.  Run from the repo root:

    python tests/golden/make_golden.py

The fixtures are committed; the GPU machine never runs this script.
"""
from __future__ import annotations

import os

import numpy as np
import torch
from torchvision.ops import deform_conv2d

HERE = os.path.dirname(os.path.abspath(__file__))

# name: (B, C, H, W, Co, groups, og, (kh, kw), stride, pad, dil, mask, bias, offset_kind)
CASES = {
    "basic_v1":          (2, 4, 5, 6, 3, 1, 1, (3, 3), (1, 1), (1, 1), (1, 1), False, False, "n2"),
    "mask_bias_g2_og2":  (2, 4, 6, 5, 4, 2, 2, (3, 3), (1, 1), (1, 1), (1, 1), True, True, "n2"),
    "stride2_dil2":      (1, 3, 9, 8, 2, 1, 1, (3, 3), (2, 2), (2, 2), (2, 2), True, True, "n1"),
    "rect_kernel":       (2, 2, 6, 7, 3, 1, 1, (2, 3), (2, 1), (1, 0), (1, 2), True, False, "n1"),
    "integer_offsets":   (1, 2, 5, 5, 2, 1, 1, (3, 3), (1, 1), (1, 1), (1, 1), True, True, "int"),
    "far_offsets_og4":   (2, 8, 6, 6, 4, 1, 4, (3, 3), (1, 1), (1, 1), (1, 1), True, True, "u10"),
    "kernel1x1":         (2, 4, 4, 5, 6, 2, 2, (1, 1), (1, 1), (0, 0), (1, 1), True, True, "n1"),
    "groups4_og2":       (1, 8, 5, 5, 8, 4, 2, (3, 3), (1, 1), (1, 1), (1, 1), True, True, "n1"),
    "ref_grad_case":     (1, 4, 6, 6, 4, 1, 1, (3, 3), (1, 1), (0, 0), (1, 1), False, False, "small"),
    "ref_bench_like":    (1, 8, 9, 9, 8, 1, 1, (3, 3), (1, 1), (0, 0), (1, 1), False, False, "small"),
    "empty_batch":       (0, 4, 5, 5, 4, 1, 1, (3, 3), (1, 1), (1, 1), (1, 1), True, True, "n1"),
    "near_integer_offsets": (2, 4, 7, 8, 3, 1, 2, (3, 3), (1, 1), (1, 1), (1, 1), True, True, "near_int"),
}


def case_arrays(spec, seed):
    """The fixture arrays of one case (inputs, output, gradients, geometry)."""
    (B, C, H, W, Co, groups, og, (kh, kw), stride, pad, dil, use_mask, use_bias, okind) = spec
    g = torch.Generator().manual_seed(seed)
    Ho = (H + 2 * pad[0] - (dil[0] * (kh - 1) + 1)) // stride[0] + 1
    Wo = (W + 2 * pad[1] - (dil[1] * (kw - 1) + 1)) // stride[1] + 1
    dt = torch.float64
    x = torch.randn(B, C, H, W, generator=g, dtype=dt)
    w = torch.randn(Co, C // groups, kh, kw, generator=g, dtype=dt) / np.sqrt(C // groups * kh * kw)
    oshape = (B, 2 * og * kh * kw, Ho, Wo)
    if okind == "n2":
        off = torch.randn(*oshape, generator=g, dtype=dt) * 2.0
    elif okind == "n1":
        off = torch.randn(*oshape, generator=g, dtype=dt)
    elif okind == "small":
        off = torch.randn(*oshape, generator=g, dtype=dt) * 0.1
    elif okind == "u10":
        off = (torch.rand(*oshape, generator=g, dtype=dt) * 2 - 1) * 10.0
    elif okind == "int":
        # integer and half-integer displacements: samples land exactly on grid
        # points and on the -1 / H borders, which exercises every validity branch
        off = torch.randint(-3, 4, oshape, generator=g).to(dt)
        off += (torch.randint(0, 2, oshape, generator=g).to(dt)) * 0.5
    elif okind == "near_int":
        # within +-2e-6 of an integer (+-n * 2^-22, exactly representable in
        # fp32): base + offset sits within an fp32 rounding step of a grid
        # line, where the bilinear derivative jumps
        off = torch.randint(-3, 4, oshape, generator=g).to(dt)
        n = torch.randint(1, 9, oshape, generator=g).to(dt)
        sgn = torch.randint(0, 2, oshape, generator=g).to(dt) * 2 - 1
        off += sgn * n * 2.0 ** -22
    else:
        raise ValueError(okind)
    mask = torch.sigmoid(torch.randn(B, og * kh * kw, Ho, Wo, generator=g, dtype=dt)) if use_mask else None
    bias = torch.randn(Co, generator=g, dtype=dt) * 0.1 if use_bias else None
    gout = torch.randn(B, Co, Ho, Wo, generator=g, dtype=dt)

    xs = x.clone().requires_grad_(True)
    ws = w.clone().requires_grad_(True)
    offs = off.clone().requires_grad_(True)
    ms = mask.clone().requires_grad_(True) if mask is not None else None
    bs = bias.clone().requires_grad_(True) if bias is not None else None
    out = deform_conv2d(xs, offs, ws, bs, stride=stride, padding=pad, dilation=dil, mask=ms)
    if B > 0:
        out.backward(gout)
    arrays = dict(
        input=x.numpy(), weight=w.numpy(), offset=off.numpy(), grad_output=gout.numpy(),
        output=out.detach().numpy(),
        stride=np.array(stride), padding=np.array(pad), dilation=np.array(dil),
    )
    if B > 0:
        arrays.update(grad_input=xs.grad.numpy(), grad_weight=ws.grad.numpy(),
                      grad_offset=offs.grad.numpy())
    if mask is not None:
        arrays["mask"] = mask.numpy()
        if B > 0:
            arrays["grad_mask"] = ms.grad.numpy()
    if bias is not None:
        arrays["bias"] = bias.numpy()
        if B > 0:
            arrays["grad_bias"] = bs.grad.numpy()
    return arrays


def seeds():
    """name -> seed: cases in sorted order from 1000."""
    return {name: 1000 + i for i, name in enumerate(sorted(CASES))}


def main():
    for name, seed in seeds().items():
        np.savez_compressed(os.path.join(HERE, f"{name}.npz"), **case_arrays(CASES[name], seed))
        print("wrote", name)


if __name__ == "__main__":
    main()
