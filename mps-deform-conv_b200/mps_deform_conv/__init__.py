"""
B200 Deformable Convolution -- torchvision.ops.deform_conv2d for NVIDIA B200 (sm_100a).

Drop-in for the Python API of mps-deform-conv (``deform_conv2d``,
``DeformConv2d``, ``ModulatedDeformConv2d``, ``is_available``) with the same
signatures, validation and error messages, running on CUDA devices instead of
MPS.  The native module ``_C`` is a thin PyTorch layer over ``libdcn_b200.so``
(C ABI in ``include/dcn_b200.h``); there is no CPU fallback.

Reference: mps_deform_conv/__init__.py (v0.2.2).
"""

import math
import threading
import weakref
from typing import Optional, Tuple

import torch
from torch import Tensor, nn

from . import ops as _ops

__version__ = "0.2.2"

# Thread-safe library loading (reference __init__.py:17-55)
_lib_lock = threading.Lock()

# Kept for compatibility with code that sets it (reference __init__.py:21, tests:161);
# B200 runs bf16 natively, so nothing is ever converted or warned about.
_bf16_warned = False

# Training cache: when the weight needs a gradient, the forward keeps its
# gathered column tiles and the channels-last input copy on the device for
# the backward (about B*Ho*Wo*C*kh*kw*2 bytes per layer between forward and
# backward), so the backward neither re-lays-out the input nor gathers the
# columns again.  The reference rebuilds its column buffer in the backward
# instead (mps_deform_conv/__init__.py:266-273).
_training_cache = True


def set_training_cache(enabled: bool) -> None:
    """Keep (True, default) or drop (False) the forward's column tiles for the backward.

    Dropping them saves device memory between forward and backward at the
    cost of a second bilinear gather in the weight-gradient pass."""
    global _training_cache
    _training_cache = bool(enabled)


# Weight images of forward-only calls.  The tensor-core forward reads its
# weights as a pre-swizzled tile image that each call otherwise rebuilds from
# the weight.  With the cache on, a forward that keeps no state for a backward
# reuses the image built for the same weight tensor, as long as the tensor's
# version counter, shape, dtype, device and group split are unchanged.
# In-place updates through the tensor (optimizer steps, ``copy_``,
# ``load_state_dict``) bump the version counter and rebuild the image; writes
# through ``weight.data`` bypass the counter, which is why the cache is off by
# default.  Entries are keyed by the weight tensor's identity and dropped when
# the tensor is freed.
_weight_images = None
_EMPTY = torch.empty(0, dtype=torch.uint8)  # "no image" argument of the forward


def set_weight_image_cache(enabled: bool) -> None:
    """Reuse (True) or rebuild per call (False, default) the forward weight image
    of forward-only calls.  Turn it on for inference with weights that change
    only through in-place operations on the weight tensor itself."""
    global _weight_images
    _weight_images = {} if enabled else None


def _weight_image(lib, input, weight, geo):
    """Forward weight image of `weight` (an empty tensor when the problem is
    not on the tensor cores), from the cache when it is on and current."""
    cache = _weight_images
    key = (tuple(weight.shape), weight.dtype, weight.device, geo[-3])
    if cache is not None:
        hit = cache.get(id(weight))
        if hit is not None and hit[0]() is weight and hit[1] == weight._version and hit[2] == key:
            return hit[3]
    img = lib.weight_image(input, weight, *geo)
    if cache is not None and img.numel() > 0:
        wid = id(weight)
        drop = lambda _ref, c=cache, k=wid: c.pop(k, None)  # the weight was freed
        cache[wid] = (weakref.ref(weight, drop), weight._version, key, img)
    return img


# ModulatedDeformConv2d reads its offset convolution's output in place (offsets
# and mask logits, sigmoid inside the kernels) when the problem allows it, or
# slices it and applies the sigmoid in PyTorch first as the reference does
# (mps_deform_conv/__init__.py:500-511).
_head_fusion = True


def set_head_fusion(enabled: bool) -> None:
    """Fuse (True, default) or compose (False) ModulatedDeformConv2d's offset/mask head."""
    global _head_fusion
    _head_fusion = bool(enabled)


# Called as hook(grad_weight, grad_bias) during each backward, as soon as those
# two gradients are enqueued on the current stream (either may be None).  On
# the tensor-core path the final layout passes of the input / offset / mask
# gradients are enqueued after the hook returns, so work the hook starts on
# another stream -- typically the data-parallel all-reduce of the parameter
# gradients -- runs alongside them.
# Work on another stream must wait for an event recorded on the current stream
# inside the hook, and the caller joins that stream before reading the
# gradients.  No reference counterpart (its backward returns all gradients at
# once, mps_deform_conv/__init__.py:245-322).
_param_grad_hook = None


def set_param_grad_hook(hook) -> None:
    """Install (or clear, with None) the parameter-gradient hook of the backward."""
    global _param_grad_hook
    if hook is not None and not callable(hook):
        raise TypeError("hook must be callable or None")
    _param_grad_hook = hook


def _load_library():
    """Load the native extension; fail loudly when it is missing."""
    try:
        from mps_deform_conv import _C as _lib
    except ImportError as e:  # no silent fallback: the CUDA kernels are the product
        raise ImportError(
            "mps_deform_conv._C is not built or cannot load libdcn_b200.so "
            "(build it with: python mps-deform-conv_b200/build.py): " + str(e)
        ) from e
    return _lib


_lib_cache = None


def _get_lib():
    """Thread-safe library loading (double-checked lock)."""
    global _lib_cache
    if _lib_cache is None:
        with _lib_lock:
            if _lib_cache is None:
                _lib_cache = _load_library()
    return _lib_cache


def _validate_conv_params(
    stride: Tuple[int, int],
    padding: Tuple[int, int],
    dilation: Tuple[int, int],
    kernel_h: int,
    kernel_w: int,
) -> None:
    """Validate convolution parameters (reference __init__.py:58-84)."""
    stride_h, stride_w = stride
    pad_h, pad_w = padding
    dilation_h, dilation_w = dilation
    if stride_h <= 0 or stride_w <= 0:
        raise ValueError(f"stride must be positive, got stride=({stride_h}, {stride_w})")
    if dilation_h <= 0 or dilation_w <= 0:
        raise ValueError(f"dilation must be positive, got dilation=({dilation_h}, {dilation_w})")
    if pad_h < 0 or pad_w < 0:
        raise ValueError(f"padding must be non-negative, got padding=({pad_h}, {pad_w})")
    if kernel_h <= 0 or kernel_w <= 0:
        raise ValueError(f"kernel_size must be positive, got kernel=({kernel_h}, {kernel_w})")


def _validate_groups(
    in_channels: int,
    out_channels: int,
    offset_channels: int,
    kernel_h: int,
    kernel_w: int,
    weight_in_channels: int,
) -> Tuple[int, int]:
    """Infer and check (n_weight_grps, n_offset_grps) (reference __init__.py:87-121)."""
    if weight_in_channels <= 0:
        raise ValueError(f"weight in_channels must be positive, got {weight_in_channels}")
    if in_channels % weight_in_channels != 0:
        raise ValueError(
            f"in_channels ({in_channels}) must be divisible by weight in_channels ({weight_in_channels})"
        )
    n_weight_grps = in_channels // weight_in_channels
    if out_channels % n_weight_grps != 0:
        raise ValueError(
            f"out_channels ({out_channels}) must be divisible by n_weight_grps ({n_weight_grps})"
        )
    offset_per_position = 2 * kernel_h * kernel_w
    if offset_per_position <= 0:
        raise ValueError(f"Invalid kernel size: {kernel_h}x{kernel_w}")
    if offset_channels % offset_per_position != 0:
        raise ValueError(
            f"offset channels ({offset_channels}) must be divisible by 2*kernel_h*kernel_w ({offset_per_position})"
        )
    n_offset_grps = offset_channels // offset_per_position
    if n_offset_grps == 0 or in_channels % n_offset_grps != 0:
        raise ValueError(
            f"in_channels ({in_channels}) must be divisible by n_offset_grps ({n_offset_grps})"
        )
    return n_weight_grps, n_offset_grps


def _check_tensor_device(tensor: Tensor, name: str, expected_device: torch.device) -> None:
    """Reference __init__.py:124-129."""
    if tensor.device != expected_device:
        raise ValueError(
            f"{name} must be on same device as input ({expected_device}), got {tensor.device}"
        )


def _check_overflow(values: list, names: list, limit: int = 2**31 - 1) -> None:
    """int32 guard on the dispatch size (reference __init__.py:145-154)."""
    product = 1
    for val, name in zip(values, names):
        product *= val
        if product > limit:
            raise ValueError(
                f"Tensor size overflow: product of {names[:names.index(name)+1]} = {product} exceeds {limit}. "
                f"Reduce batch size or spatial dimensions."
            )


def _pair(v):
    return (v, v) if isinstance(v, int) else tuple(v)


class _DeformConv2dFunction(torch.autograd.Function):
    """Autograd function with the fused CUDA backward (reference __init__.py:157-322)."""

    @staticmethod
    def forward(
        ctx,
        input: Tensor,
        offset: Tensor,
        weight: Tensor,
        bias: Optional[Tensor],
        stride: Tuple[int, int],
        padding: Tuple[int, int],
        dilation: Tuple[int, int],
        mask: Optional[Tensor],
        n_weight_grps: int,
        n_offset_grps: int,
        use_mask: bool,
    ) -> Tensor:
        lib = _get_lib()
        stride, padding, dilation = _pair(stride), _pair(padding), _pair(dilation)
        stride_h, stride_w = stride
        pad_h, pad_w = padding
        dilation_h, dilation_w = dilation

        expected_device = input.device
        _check_tensor_device(weight, "weight", expected_device)
        _check_tensor_device(offset, "offset", expected_device)
        if bias is not None:
            _check_tensor_device(bias, "bias", expected_device)
        if mask is not None:
            _check_tensor_device(mask, "mask", expected_device)

        batch_sz = input.size(0)
        n_in_channels = input.size(1)
        in_h, in_w = input.size(2), input.size(3)
        kernel_h, kernel_w = weight.size(2), weight.size(3)
        out_h = (in_h + 2 * pad_h - (dilation_h * (kernel_h - 1) + 1)) // stride_h + 1
        out_w = (in_w + 2 * pad_w - (dilation_w * (kernel_w - 1) + 1)) // stride_w + 1
        if out_h <= 0 or out_w <= 0:
            raise ValueError(
                f"Invalid output dimensions: out_h={out_h}, out_w={out_w}. "
                f"Check stride/padding/dilation values."
            )
        _check_overflow(
            [n_in_channels, kernel_h, kernel_w, batch_sz, out_h, out_w],
            ["channels", "kernel_h", "kernel_w", "batch", "out_h", "out_w"],
        )

        bias_t = bias if bias is not None else torch.empty(0, device=input.device, dtype=input.dtype)
        mask_t = mask if mask is not None else torch.empty(0, device=input.device, dtype=input.dtype)

        # a channels_last input gives a channels_last output (read and written in
        # place by the tensor-core kernels)
        keep = bool(_training_cache and ctx.needs_input_grad[2])
        image = _EMPTY
        if not keep and _weight_images is not None:
            image = _weight_image(lib, input, weight, (stride_h, stride_w, pad_h, pad_w, dilation_h, dilation_w,
                                                       n_weight_grps, n_offset_grps, use_mask))
        output, saved = lib.deform_conv2d_forward_ex(
            input, weight, offset, mask_t, bias_t,
            stride_h, stride_w, pad_h, pad_w,
            dilation_h, dilation_w,
            n_weight_grps, n_offset_grps, use_mask, keep, image,
        )
        if saved.numel() == 0:
            saved = None

        ctx.save_for_backward(input, offset, weight, mask_t if use_mask else None, saved)
        ctx.bias_exists = bias is not None
        ctx.stride = stride
        ctx.padding = padding
        ctx.dilation = dilation
        ctx.n_weight_grps = n_weight_grps
        ctx.n_offset_grps = n_offset_grps
        ctx.use_mask = use_mask
        return output

    @staticmethod
    def backward(ctx, grad_output: Tensor):
        input, offset, weight, mask, saved = ctx.saved_tensors
        stride_h, stride_w = ctx.stride
        pad_h, pad_w = ctx.padding
        dilation_h, dilation_w = ctx.dilation
        use_mask = ctx.use_mask and mask is not None
        lib = _get_lib()
        mask_t = mask if use_mask else torch.empty(0, device=input.device, dtype=input.dtype)
        bias_t = (torch.empty(weight.size(0), device=input.device, dtype=input.dtype)
                  if ctx.bias_exists else torch.empty(0, device=input.device, dtype=input.dtype))
        needs = ctx.needs_input_grad
        output_mask = [bool(needs[0]), bool(needs[2]), bool(needs[1]),
                       bool(use_mask and needs[7]), bool(ctx.bias_exists and needs[3])]
        grad_input, grad_weight, grad_offset, grad_mask, grad_bias = lib.deform_conv2d_backward(
            grad_output, input, weight, offset, mask_t, bias_t,
            stride_h, stride_w, pad_h, pad_w, dilation_h, dilation_w,
            ctx.n_weight_grps, ctx.n_offset_grps, use_mask, output_mask,
            saved, _param_grad_hook,
        )
        return (grad_input, grad_offset, grad_weight, grad_bias,
                None, None, None, grad_mask, None, None, None)


class _DeformConv2dHeadFunction(torch.autograd.Function):
    """deform_conv2d reading offsets and mask logits in place from a DCNv2 head
    output [B, 3*og*kh*kw, Ho, Wo] (offsets first); the mask is the sigmoid of
    the logits.  Its backward returns the gradient of that head output."""

    @staticmethod
    def forward(ctx, input, offset_mask, weight, bias, stride, padding, dilation, n_weight_grps, n_offset_grps):
        lib = _get_lib()
        bias_t = bias if bias is not None else torch.empty(0, device=input.device, dtype=input.dtype)
        keep = _training_cache and ctx.needs_input_grad[2]
        output, saved = lib.deform_conv2d_forward_head(
            input, weight, offset_mask, bias_t, stride[0], stride[1], padding[0], padding[1],
            dilation[0], dilation[1], n_weight_grps, n_offset_grps, keep)
        ctx.save_for_backward(input, offset_mask, weight, saved)
        ctx.geom = (stride, padding, dilation, n_weight_grps, n_offset_grps)
        ctx.bias_exists = bias is not None
        return output

    @staticmethod
    def backward(ctx, grad_output):
        input, offset_mask, weight, saved = ctx.saved_tensors
        (sh, sw), (ph, pw), (dh, dw), n_weight_grps, n_offset_grps = ctx.geom
        needs = ctx.needs_input_grad
        bias_t = (torch.empty(weight.size(0), device=input.device, dtype=input.dtype) if ctx.bias_exists
                  else torch.empty(0, device=input.device, dtype=input.dtype))
        output_mask = [bool(needs[0]), bool(needs[2]), bool(needs[1]), bool(ctx.bias_exists and needs[3])]
        grad_input, grad_weight, grad_offset_mask, grad_bias = _get_lib().deform_conv2d_backward_head(
            grad_output, input, weight, offset_mask, bias_t, sh, sw, ph, pw, dh, dw, n_weight_grps,
            n_offset_grps, output_mask, saved if saved.numel() > 0 else None)
        if _param_grad_hook is not None:  # no overlap on this path: called once all gradients are enqueued
            _param_grad_hook(grad_weight, grad_bias)
        return grad_input, grad_offset_mask, grad_weight, grad_bias, None, None, None, None, None


def deform_conv2d(
    input: Tensor,
    offset: Tensor,
    weight: Tensor,
    bias: Optional[Tensor] = None,
    stride: Tuple[int, int] = (1, 1),
    padding: Tuple[int, int] = (0, 0),
    dilation: Tuple[int, int] = (1, 1),
    mask: Optional[Tensor] = None,
) -> Tensor:
    """
    Deformable 2D convolution (reference __init__.py:325-386).

    Args:
        input: Input tensor (N, C_in, H, W)
        offset: Offset tensor (N, 2*K*K*offset_groups, H_out, W_out)
        weight: Weight tensor (C_out, C_in/groups, K, K)
        bias: Optional bias (C_out,)
        stride: Convolution stride (must be positive)
        padding: Input padding (must be non-negative)
        dilation: Kernel dilation (must be positive)
        mask: Optional DCNv2 mask (N, K*K*offset_groups, H_out, W_out)

    Returns:
        Output tensor (N, C_out, H_out, W_out)

    Raises:
        ValueError: If input is not on a CUDA device or parameters are invalid.

    While a compiler traces it, or on meta tensors, the call goes through the
    registered operators of ``mps_deform_conv.ops`` (fake implementations for
    shapes, autograd wired to the fused backward).
    """
    traced = input.device.type == "meta" or torch.compiler.is_compiling()
    if not (input.device.type == "cuda" or traced):
        raise ValueError(f"Input must be on CUDA device, got {input.device}")
    stride, padding, dilation = _pair(stride), _pair(padding), _pair(dilation)
    kernel_h, kernel_w = weight.size(2), weight.size(3)
    in_channels = input.size(1)
    out_channels = weight.size(0)
    offset_channels = offset.size(1)
    weight_in_channels = weight.size(1)
    _validate_conv_params(stride, padding, dilation, kernel_h, kernel_w)
    n_weight_grps, n_offset_grps = _validate_groups(
        in_channels, out_channels, offset_channels, kernel_h, kernel_w, weight_in_channels
    )
    use_mask = mask is not None
    if traced:
        return _ops.traced_deform_conv2d(input, offset, weight, bias, stride, padding, dilation, mask,
                                         n_weight_grps, n_offset_grps)
    return _DeformConv2dFunction.apply(
        input, offset, weight, bias,
        stride, padding, dilation, mask,
        n_weight_grps, n_offset_grps, use_mask,
    )


class DeformConv2d(nn.Module):
    """Deformable 2D Convolution Module (reference __init__.py:389-437)."""

    def __init__(
        self,
        in_channels: int,
        out_channels: int,
        kernel_size: int,
        stride: int = 1,
        padding: int = 0,
        dilation: int = 1,
        groups: int = 1,
        offset_groups: int = 1,
        bias: bool = True,
    ):
        super().__init__()
        self.in_channels = in_channels
        self.out_channels = out_channels
        self.kernel_size = (kernel_size, kernel_size) if isinstance(kernel_size, int) else kernel_size
        self.stride = (stride, stride) if isinstance(stride, int) else stride
        self.padding = (padding, padding) if isinstance(padding, int) else padding
        self.dilation = (dilation, dilation) if isinstance(dilation, int) else dilation
        self.groups = groups
        self.offset_groups = offset_groups
        self.weight = nn.Parameter(torch.empty(out_channels, in_channels // groups, *self.kernel_size))
        if bias:
            self.bias = nn.Parameter(torch.empty(out_channels))
        else:
            self.register_parameter("bias", None)
        self.reset_parameters()

    def reset_parameters(self):
        nn.init.kaiming_uniform_(self.weight, a=math.sqrt(5))
        if self.bias is not None:
            fan_in, _ = nn.init._calculate_fan_in_and_fan_out(self.weight)
            bound = 1 / math.sqrt(fan_in) if fan_in > 0 else 0
            nn.init.uniform_(self.bias, -bound, bound)

    def forward(self, input: Tensor, offset: Tensor, mask: Optional[Tensor] = None) -> Tensor:
        return deform_conv2d(
            input, offset, self.weight, self.bias,
            self.stride, self.padding, self.dilation, mask,
        )


class ModulatedDeformConv2d(nn.Module):
    """Modulated Deformable Convolution (DCNv2) with built-in offset prediction
    (reference __init__.py:440-511)."""

    def __init__(
        self,
        in_channels: int,
        out_channels: int,
        kernel_size: int,
        stride: int = 1,
        padding: int = 0,
        dilation: int = 1,
        groups: int = 1,
        offset_groups: int = 1,
        bias: bool = True,
    ):
        super().__init__()
        self.in_channels = in_channels
        self.out_channels = out_channels
        self.kernel_size = (kernel_size, kernel_size) if isinstance(kernel_size, int) else kernel_size
        self.stride = (stride, stride) if isinstance(stride, int) else stride
        self.padding = (padding, padding) if isinstance(padding, int) else padding
        self.dilation = (dilation, dilation) if isinstance(dilation, int) else dilation
        self.groups = groups
        self.offset_groups = offset_groups
        self.weight = nn.Parameter(torch.empty(out_channels, in_channels // groups, *self.kernel_size))
        if bias:
            self.bias = nn.Parameter(torch.empty(out_channels))
        else:
            self.register_parameter("bias", None)
        kernel_h, kernel_w = self.kernel_size
        offset_channels = 2 * kernel_h * kernel_w * offset_groups
        mask_channels = kernel_h * kernel_w * offset_groups
        self.offset_conv = nn.Conv2d(
            in_channels,
            offset_channels + mask_channels,
            kernel_size=self.kernel_size,
            stride=self.stride,
            padding=self.padding,
            dilation=self.dilation,
            bias=True,
        )
        self.reset_parameters()

    def reset_parameters(self):
        nn.init.kaiming_uniform_(self.weight, a=math.sqrt(5))
        if self.bias is not None:
            fan_in, _ = nn.init._calculate_fan_in_and_fan_out(self.weight)
            bound = 1 / math.sqrt(fan_in) if fan_in > 0 else 0
            nn.init.uniform_(self.bias, -bound, bound)
        nn.init.zeros_(self.offset_conv.weight)
        nn.init.zeros_(self.offset_conv.bias)

    def _fused_head(self, input: Tensor, offset_mask: Tensor) -> bool:
        if torch.compiler.is_compiling():  # traced: the composition below, through the registered operators
            return False
        if not (_head_fusion and input.is_cuda and input.dim() == 4 and
                input.dtype == offset_mask.dtype == self.weight.dtype and
                (self.bias is None or self.bias.dtype == input.dtype)):
            return False
        return bool(_get_lib().head_supported(
            input, self.weight, self.stride[0], self.stride[1], self.padding[0], self.padding[1],
            self.dilation[0], self.dilation[1], self.groups, self.offset_groups))

    def forward(self, input: Tensor) -> Tensor:
        kernel_h, kernel_w = self.kernel_size
        offset_channels = 2 * kernel_h * kernel_w * self.offset_groups
        offset_mask = self.offset_conv(input)
        if self._fused_head(input, offset_mask):
            return _DeformConv2dHeadFunction.apply(
                input, offset_mask, self.weight, self.bias, tuple(self.stride), tuple(self.padding),
                tuple(self.dilation), self.groups, self.offset_groups)
        offset = offset_mask[:, :offset_channels]
        mask = torch.sigmoid(offset_mask[:, offset_channels:])
        return deform_conv2d(
            input, offset, self.weight, self.bias,
            self.stride, self.padding, self.dilation, mask,
        )


def is_available() -> bool:
    """True when a CUDA device is present (the reference checks MPS, __init__.py:514-516)."""
    return torch.cuda.is_available()


__all__ = ["deform_conv2d", "DeformConv2d", "ModulatedDeformConv2d", "is_available", "__version__",
           "set_training_cache", "set_param_grad_hook", "set_head_fusion", "set_weight_image_cache"]
