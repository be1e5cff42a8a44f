"""The operator pair as registered PyTorch operators, for tracing.

``torch.ops.mps_deform_conv.deform_conv2d_forward`` and
``torch.ops.mps_deform_conv.deform_conv2d_backward`` take the argument lists of
the reference's native forward (mps_deform_conv/csrc/deform_conv2d_mps.mm:603-615,
which is the ``torchvision::deform_conv2d`` schema) and of
``torchvision::_deform_conv2d_backward``.  Each has a fake (meta)
implementation that only computes output shapes, and the forward has autograd
wired to the backward, so ``torch.compile`` and FX tracing see two opaque
operators instead of breaking the graph at the extension call.

``deform_conv2d`` takes this route while a compiler traces it
(``torch.compiler.is_compiling()``) or when its input is a meta tensor; eager
calls go through ``_DeformConv2dFunction`` (training cache, parameter-gradient
hook, channels_last in place), which these operators do not offer: they make
their tensors contiguous, so the layouts their fake implementations report
are always the ones the kernels return.  An absent mask or bias is an empty
tensor, as in the reference (mps_deform_conv/__init__.py:224-225).
"""
from __future__ import annotations

from typing import Tuple

import torch
from torch import Tensor

_NS = "mps_deform_conv"


def _out_hw(input: Tensor, weight: Tensor, stride_h, stride_w, pad_h, pad_w, dilation_h, dilation_w):
    kh, kw = weight.shape[2], weight.shape[3]
    out_h = (input.shape[2] + 2 * pad_h - (dilation_h * (kh - 1) + 1)) // stride_h + 1
    out_w = (input.shape[3] + 2 * pad_w - (dilation_w * (kw - 1) + 1)) // stride_w + 1
    return out_h, out_w


@torch.library.custom_op(f"{_NS}::deform_conv2d_forward", mutates_args=())
def deform_conv2d_forward(input: Tensor, weight: Tensor, offset: Tensor, mask: Tensor, bias: Tensor,
                          stride_h: int, stride_w: int, pad_h: int, pad_w: int, dilation_h: int,
                          dilation_w: int, groups: int, offset_groups: int, use_mask: bool) -> Tensor:
    from mps_deform_conv import _get_lib
    return _get_lib().deform_conv2d_forward(
        input.contiguous(), weight, offset, mask, bias, stride_h, stride_w, pad_h, pad_w, dilation_h,
        dilation_w, groups, offset_groups, use_mask)


@deform_conv2d_forward.register_fake
def _forward_fake(input, weight, offset, mask, bias, stride_h, stride_w, pad_h, pad_w, dilation_h, dilation_w,
                  groups, offset_groups, use_mask):
    out_h, out_w = _out_hw(input, weight, stride_h, stride_w, pad_h, pad_w, dilation_h, dilation_w)
    return input.new_empty((input.shape[0], weight.shape[0], out_h, out_w))


@torch.library.custom_op(f"{_NS}::deform_conv2d_backward", mutates_args=())
def deform_conv2d_backward(grad: Tensor, input: Tensor, weight: Tensor, offset: Tensor, mask: Tensor,
                           bias: Tensor, stride_h: int, stride_w: int, pad_h: int, pad_w: int, dilation_h: int,
                           dilation_w: int, groups: int, offset_groups: int,
                           use_mask: bool) -> Tuple[Tensor, Tensor, Tensor, Tensor, Tensor]:
    """(grad_input, grad_weight, grad_offset, grad_mask, grad_bias); the last two
    are zeros shaped like an absent mask / bias."""
    from mps_deform_conv import _get_lib
    gi, gw, goff, gm, gb = _get_lib().deform_conv2d_backward(
        grad.contiguous(), input.contiguous(), weight, offset, mask, bias, stride_h, stride_w, pad_h, pad_w,
        dilation_h, dilation_w, groups, offset_groups, use_mask, [True] * 5, None)
    if gm is None:
        gm = torch.zeros_like(mask)
    if gb is None:
        gb = torch.zeros_like(bias)
    return gi, gw, goff, gm, gb


@deform_conv2d_backward.register_fake
def _backward_fake(grad, input, weight, offset, mask, bias, stride_h, stride_w, pad_h, pad_w, dilation_h,
                   dilation_w, groups, offset_groups, use_mask):
    return (input.new_empty(input.shape), weight.new_empty(weight.shape), offset.new_empty(offset.shape),
            mask.new_empty(mask.shape), bias.new_empty(bias.shape))


def _setup_context(ctx, inputs, output):
    input, weight, offset, mask, bias = inputs[:5]
    ctx.save_for_backward(input, weight, offset, mask, bias)
    ctx.geom = inputs[5:]


def _forward_backward(ctx, grad):
    input, weight, offset, mask, bias = ctx.saved_tensors
    gi, gw, goff, gm, gb = torch.ops.mps_deform_conv.deform_conv2d_backward(
        grad, input, weight, offset, mask, bias, *ctx.geom)
    return (gi, gw, goff, gm, gb) + (None,) * len(ctx.geom)


deform_conv2d_forward.register_autograd(_forward_backward, setup_context=_setup_context)


def traced_deform_conv2d(input: Tensor, offset: Tensor, weight: Tensor, bias, stride, padding, dilation, mask,
                         n_weight_grps: int, n_offset_grps: int) -> Tensor:
    """deform_conv2d through the registered operator (arguments validated by the caller)."""
    empty = input.new_empty((0,))
    return torch.ops.mps_deform_conv.deform_conv2d_forward(
        input, weight, offset, mask if mask is not None else empty, bias if bias is not None else empty,
        stride[0], stride[1], padding[0], padding[1], dilation[0], dilation[1], n_weight_grps, n_offset_grps,
        mask is not None)
