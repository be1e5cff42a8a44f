"""The benchmark problems of this package as seeded synthetic inputs.

Five deformable-convolution layers, from a CPU-sized DCNv1 layer to a large
grouped DCNv2 training step.  Distributions: input ~N(0,1); weight
~N(0, 1/sqrt(fan_in)); offsets in pixels as listed; mask = sigmoid(N(0,1));
grad_output ~N(0,1).  Everything is generated in fp32 from one seed on the
target device, then cast to the problem's dtype.
"""
from __future__ import annotations

import dataclasses
import math
from typing import Dict, Optional

import torch


@dataclasses.dataclass(frozen=True)
class Problem:
    name: str
    description: str
    batch: int
    in_channels: int
    out_channels: int
    height: int
    width: int
    kernel: int = 3
    stride: int = 1
    padding: int = 1
    dilation: int = 1
    groups: int = 1
    offset_groups: int = 1
    use_mask: bool = True
    use_bias: bool = False
    dtype: torch.dtype = torch.float32
    training: bool = False          # forward + backward
    offset_kind: str = "normal"     # "normal" (std = offset_scale) or "uniform" (+-offset_scale)
    offset_scale: float = 1.0

    @property
    def out_hw(self):
        k = self.dilation * (self.kernel - 1) + 1
        return ((self.height + 2 * self.padding - k) // self.stride + 1,
                (self.width + 2 * self.padding - k) // self.stride + 1)

    @property
    def k_red(self) -> int:
        return self.in_channels // self.groups * self.kernel * self.kernel

    def flops_forward(self, batch: Optional[int] = None) -> float:
        ho, wo = self.out_hw
        b = self.batch if batch is None else batch
        return 2.0 * self.out_channels * self.k_red * b * ho * wo

    def flops(self, batch: Optional[int] = None) -> float:
        """Algorithmic FLOPs of one step: forward, plus dgrad and wgrad when training."""
        return self.flops_forward(batch) * (3.0 if self.training else 1.0)

    def min_hbm_bytes(self, batch: Optional[int] = None) -> float:
        """Unique tensor bytes a step must move: read inputs once, write outputs once."""
        b = self.batch if batch is None else batch
        es = torch.tensor([], dtype=self.dtype).element_size()
        ho, wo = self.out_hw
        t = self.kernel * self.kernel
        x = b * self.in_channels * self.height * self.width
        off = b * 2 * self.offset_groups * t * ho * wo
        msk = b * self.offset_groups * t * ho * wo if self.use_mask else 0
        w = self.out_channels * self.k_red
        out = b * self.out_channels * ho * wo
        bias = self.out_channels if self.use_bias else 0
        fwd = x + off + msk + w + out + bias
        if not self.training:
            return float(fwd * es)
        # backward reads grad_out, x, offset, mask, w; writes gI, gOff, gMask, gW, gB
        bwd = out + x + off + msk + w + x + off + msk + w + bias
        return float((fwd + bwd) * es)


PROBLEMS: Dict[str, Problem] = {
    "c1_dcnv1_fp32": Problem(
        "c1_dcnv1_fp32", "DCNv1 forward fp32, 1x64x32x32, 64->64, 3x3 pad 1, no mask/bias",
        batch=1, in_channels=64, out_channels=64, height=32, width=32, use_mask=False,
        dtype=torch.float32, offset_scale=1.0),
    "c2_dcnv2_fp32": Problem(
        "c2_dcnv2_fp32", "DCNv2 forward+backward fp32, 2x128x64x64, 128->128, bias",
        batch=2, in_channels=128, out_channels=128, height=64, width=64, use_bias=True,
        dtype=torch.float32, training=True, offset_scale=2.0),
    "c3a_backbone_bf16": Problem(
        "c3a_backbone_bf16", "ResNet-50 C4-stage DCN forward bf16, 8x256x50x68, 256->256",
        batch=8, in_channels=256, out_channels=256, height=50, width=68,
        dtype=torch.bfloat16, offset_scale=1.5),
    "c3b_backbone_s2_bf16": Problem(
        "c3b_backbone_s2_bf16", "stride-2 DCN forward bf16, 8x256x100x100, 256->512",
        batch=8, in_channels=256, out_channels=512, height=100, width=100, stride=2,
        dtype=torch.bfloat16, offset_scale=1.5),
    "c4_video_fp16": Problem(
        "c4_video_fp16", "video-alignment DCNv2 fwd+bwd fp16, 16x64x180x320, og=8, U(-10,10) px",
        batch=16, in_channels=64, out_channels=64, height=180, width=320, offset_groups=8,
        dtype=torch.float16, training=True, offset_kind="uniform", offset_scale=10.0),
    "c5_train_bf16": Problem(
        "c5_train_bf16", "training step bf16, 64x512x38x38, g=2, og=4, pad 2 dil 2, bias",
        batch=64, in_channels=512, out_channels=512, height=38, width=38, padding=2, dilation=2,
        groups=2, offset_groups=4, use_bias=True, dtype=torch.bfloat16, training=True,
        offset_scale=3.0),
}


def make_inputs(p: Problem, device="cpu", batch: Optional[int] = None, seed: int = 0,
                dtype: Optional[torch.dtype] = None, batch_offset: int = 0):
    """Seeded inputs for problem `p`: dict(input, offset, weight, bias, mask, grad_output).

    `batch` overrides the batch size.  `batch_offset` selects a slice of a larger
    batch: sample i of the result is sample batch_offset + i of the full problem
    (per-sample generators), so shards of one global batch are consistent.
    """
    b = p.batch if batch is None else batch
    dt = p.dtype if dtype is None else dtype
    ho, wo = p.out_hw
    t = p.kernel * p.kernel
    dev = torch.device(device)

    def gen(s):
        g = torch.Generator(device=dev)
        g.manual_seed(s)
        return g

    gw = gen(seed)
    fan_in = p.k_red
    weight = torch.randn(p.out_channels, p.in_channels // p.groups, p.kernel, p.kernel,
                         generator=gw, device=dev) / math.sqrt(fan_in)
    bias = (torch.randn(p.out_channels, generator=gw, device=dev) * 0.01) if p.use_bias else None
    xs, offs, masks, gos = [], [], [], []
    for i in range(b):
        gs = gen(seed * 1000003 + 7919 * (batch_offset + i) + 1)
        xs.append(torch.randn(p.in_channels, p.height, p.width, generator=gs, device=dev))
        oshape = (2 * p.offset_groups * t, ho, wo)
        if p.offset_kind == "uniform":
            offs.append((torch.rand(oshape, generator=gs, device=dev) * 2 - 1) * p.offset_scale)
        else:
            offs.append(torch.randn(oshape, generator=gs, device=dev) * p.offset_scale)
        if p.use_mask:
            masks.append(torch.sigmoid(torch.randn(p.offset_groups * t, ho, wo, generator=gs, device=dev)))
        gos.append(torch.randn(p.out_channels, ho, wo, generator=gs, device=dev))

    def stack(lst, shape):
        return torch.stack(lst).to(dt) if lst else torch.empty(shape, device=dev, dtype=dt)

    return dict(
        input=stack(xs, (0, p.in_channels, p.height, p.width)),
        offset=stack(offs, (0, 2 * p.offset_groups * t, ho, wo)),
        mask=stack(masks, (0, p.offset_groups * t, ho, wo)) if p.use_mask else None,
        weight=weight.to(dt),
        bias=bias.to(dt) if bias is not None else None,
        grad_output=stack(gos, (0, p.out_channels, ho, wo)),
    )
