"""Serve torchvision's deformable-convolution operators with the B200 kernels.

After ``register_torchvision_ops()``, ``torchvision.ops.deform_conv2d`` (and
``torchvision.ops.DeformConv2d``) on CUDA tensors run on this package's
kernels: the CUDA implementations of ``torchvision::deform_conv2d`` and
``torchvision::_deform_conv2d_backward`` are replaced, keeping torchvision's
own autograd wiring.  The two schemas are argument-for-argument those of the
native functions (input, weight, offset, mask, bias, stride_h, stride_w, pad_h,
pad_w, dilation_h, dilation_w, groups, offset_groups, use_mask), so no argument
is translated.  CPU tensors keep torchvision's CPU kernels.
"""
from __future__ import annotations

import threading

import torch

_lock = threading.Lock()
_library = None


def _forward_cuda(input, weight, offset, mask, bias, stride_h, stride_w, pad_h, pad_w,
                  dilation_h, dilation_w, groups, offset_groups, use_mask):
    from mps_deform_conv import _get_lib
    return _get_lib().deform_conv2d_forward(input, weight, offset, mask, bias, stride_h, stride_w,
                                            pad_h, pad_w, dilation_h, dilation_w, groups,
                                            offset_groups, use_mask)


def _backward_cuda(grad, input, weight, offset, mask, bias, stride_h, stride_w, pad_h, pad_w,
                   dilation_h, dilation_w, groups, offset_groups, use_mask):
    from mps_deform_conv import _get_lib
    gi, gw, goff, gm, gb = _get_lib().deform_conv2d_backward(
        grad, input, weight, offset, mask, bias, stride_h, stride_w, pad_h, pad_w, dilation_h,
        dilation_w, groups, offset_groups, use_mask, [True] * 5, None)
    # torchvision's autograd expects every gradient defined
    if gm is None:
        gm = torch.zeros_like(mask)
    if gb is None:
        gb = torch.zeros_like(bias)
    return gi, gw, goff, gm, gb


def register_torchvision_ops() -> None:
    """Make torchvision's deform_conv2d CUDA kernels these kernels (idempotent)."""
    global _library
    with _lock:
        if _library is not None:
            return
        import torchvision  # noqa: F401  (registers the torchvision operator schemas)
        import warnings

        lib = torch.library.Library("torchvision", "IMPL")
        with warnings.catch_warnings():
            warnings.simplefilter("ignore")  # "overriding a previously registered kernel"
            lib.impl("deform_conv2d", _forward_cuda, "CUDA")
            lib.impl("_deform_conv2d_backward", _backward_cuda, "CUDA")
        _library = lib


def registered() -> bool:
    return _library is not None
