"""ctypes binding of the C ABI in include/dcn_b200.h (libdcn_b200.so).

For callers that want the kernels without the PyTorch extension: every entry
point takes device pointers, a ``DcnConvDesc`` and a CUDA stream handle.
``call_*`` helpers accept torch CUDA tensors and allocate outputs/workspace
with torch, then call straight into the C ABI.
"""
from __future__ import annotations

import ctypes
import os
from typing import Optional

LIB_PATH = os.path.join(os.path.dirname(os.path.abspath(__file__)), "lib", "libdcn_b200.so")
# The same library built with -DDCN_DEBUG_BOUNDS: index checks in the gather
# and scatter kernels (build.py builds both).
BOUNDS_LIB_PATH = os.path.join(os.path.dirname(os.path.abspath(__file__)), "lib", "libdcn_b200_bounds.so")

DCN_FLOAT32, DCN_FLOAT16, DCN_BFLOAT16 = 0, 1, 2
DCN_OK = 0
DCN_ERR_INVALID_ARGUMENT = 1
DCN_ERR_UNSUPPORTED = 2
DCN_ERR_CUDA = 3
DCN_ERR_WORKSPACE = 4
DCN_ERR_DEVICE_TIMEOUT = 5


class DcnConvDesc(ctypes.Structure):
    """Mirror of ``dcn_conv_desc``."""
    _fields_ = [
        ("dtype", ctypes.c_int32), ("use_mask", ctypes.c_int32),
        ("batch", ctypes.c_int64), ("in_channels", ctypes.c_int64),
        ("in_h", ctypes.c_int64), ("in_w", ctypes.c_int64),
        ("out_channels", ctypes.c_int64), ("kernel_h", ctypes.c_int64), ("kernel_w", ctypes.c_int64),
        ("stride_h", ctypes.c_int64), ("stride_w", ctypes.c_int64),
        ("pad_h", ctypes.c_int64), ("pad_w", ctypes.c_int64),
        ("dilation_h", ctypes.c_int64), ("dilation_w", ctypes.c_int64),
        ("n_weight_grps", ctypes.c_int64), ("n_offset_grps", ctypes.c_int64),
    ]


class DcnBoundsRecord(ctypes.Structure):
    """Mirror of ``dcn_bounds_record``."""
    _fields_ = [("count", ctypes.c_uint64), ("index", ctypes.c_int64), ("extent", ctypes.c_int64),
                ("site", ctypes.c_int32), ("width", ctypes.c_int32)]


# name -> (restype, argtypes); the exported surface of include/dcn_b200.h
_D = ctypes.POINTER(DcnConvDesc)
DCN_LAYOUT_NCHW = 0
DCN_LAYOUT_NHWC = 1
DCN_EX_WEIGHT_IMAGE = 1


class DcnExOptions(ctypes.Structure):
    """dcn_ex_options of include/dcn_b200.h."""
    _fields_ = [("input_layout", ctypes.c_int32), ("output_layout", ctypes.c_int32), ("head", ctypes.c_int32),
                ("flags", ctypes.c_int32)]


_O = ctypes.POINTER(DcnExOptions)
# void (*dcn_params_ready_fn)(void* user_data)
PARAMS_READY_FN = ctypes.CFUNCTYPE(None, ctypes.c_void_p)
_V = ctypes.c_void_p
_SZ = ctypes.c_size_t
SIGNATURES = {
    "dcn_abi_version": (ctypes.c_int, []),
    "dcn_last_error": (ctypes.c_char_p, []),
    "dcn_launch_count": (ctypes.c_uint64, []),
    "dcn_profile_enable": (None, [ctypes.c_int]),
    "dcn_profile_summary": (ctypes.c_int, [ctypes.c_int, ctypes.c_char_p, ctypes.c_size_t,
                                           ctypes.POINTER(ctypes.c_uint64), ctypes.POINTER(ctypes.c_double)]),
    "dcn_output_size": (ctypes.c_int, [_D, ctypes.POINTER(ctypes.c_int64), ctypes.POINTER(ctypes.c_int64)]),
    "dcn_validate": (ctypes.c_int, [_D]),
    "dcn_forward_workspace_size": (_SZ, [_D]),
    "dcn_deform_conv2d_forward": (ctypes.c_int, [_D, _V, _V, _V, _V, _V, _V, _V, _SZ, _V]),
    "dcn_deformable_im2col": (ctypes.c_int, [_D, _V, _V, _V, _V, _V]),
    "dcn_backward_input_workspace_size": (_SZ, [_D]),
    "dcn_deform_conv2d_backward_input": (ctypes.c_int, [_D, _V, _V, _V, _V, _V, _SZ, _V]),
    "dcn_deform_conv2d_backward_input_noalloc": (ctypes.c_int, [_D, _V, _V, _V, _V, _V]),
    "dcn_deform_conv2d_backward_offset_mask": (ctypes.c_int, [_D, _V, _V, _V, _V, _V, _V, _V]),
    "dcn_backward_workspace_size": (_SZ, [_D]),
    "dcn_deform_conv2d_backward": (ctypes.c_int, [_D, _V, _V, _V, _V, _V, _V, _V, _V, _V, _V, _V, _SZ, _V]),
    "dcn_saved_state_bytes": (_SZ, [_D]),
    "dcn_deform_conv2d_forward_train": (ctypes.c_int, [_D, _V, _V, _V, _V, _V, _V, _V, _SZ, _V, _SZ, _V]),
    "dcn_deform_conv2d_backward_train": (ctypes.c_int, [_D, _V, _V, _V, _V, _V, _V, _SZ, _V, _V, _V, _V, _V,
                                                        _V, _SZ, _V]),
    "dcn_deform_conv2d_backward_overlap": (ctypes.c_int, [_D, _V, _V, _V, _V, _V, _V, _SZ, _V, _V, _V, _V, _V,
                                                          _V, _SZ, _V, PARAMS_READY_FN, _V]),
    "dcn_head_supported": (ctypes.c_int, [_D]),
    "dcn_ex_supported": (ctypes.c_int, [_D, _O, ctypes.c_int]),
    "dcn_weight_image_bytes": (_SZ, [_D]),
    "dcn_weight_image": (ctypes.c_int, [_D, _V, _V, _SZ, _V]),
    "dcn_deform_conv2d_forward_ex": (ctypes.c_int, [_D, _O, _V, _V, _V, _V, _V, _V, _V, _SZ, _V, _SZ, _V]),
    "dcn_deform_conv2d_backward_ex": (ctypes.c_int, [_D, _O, _V, _V, _V, _V, _V, _V, _SZ, _V, _V, _V, _V, _V, _V,
                                                     _SZ, _V]),
    "dcn_deform_conv2d_forward_head": (ctypes.c_int, [_D, _V, _V, _V, _V, _V, _V, _SZ, _V, _SZ, _V]),
    "dcn_deform_conv2d_backward_head": (ctypes.c_int, [_D, _V, _V, _V, _V, _V, _SZ, _V, _V, _V, _V, _V, _SZ,
                                                       _V]),
    "dcn_device_status": (ctypes.c_int, [_V]),
    "dcn_uses_tensor_cores": (ctypes.c_int, [_D]),
    "dcn_debug_bounds_enabled": (ctypes.c_int, []),
    "dcn_debug_bounds_read": (ctypes.c_int, [ctypes.POINTER(DcnBoundsRecord), ctypes.c_int]),
}

_libs = {}


def load(path: str = LIB_PATH) -> ctypes.CDLL:
    """Load libdcn_b200.so (or another build of it at `path`) once and declare
    every exported signature."""
    if path not in _libs:
        lib = ctypes.CDLL(path)
        for name, (res, args) in SIGNATURES.items():
            f = getattr(lib, name)
            f.restype = res
            f.argtypes = args
        _libs[path] = lib
    return _libs[path]


def load_bounds() -> ctypes.CDLL:
    """The bounds-checked build (libdcn_b200_bounds.so)."""
    return load(BOUNDS_LIB_PATH)


def bounds_record(lib: Optional[ctypes.CDLL] = None, reset: bool = True) -> DcnBoundsRecord:
    """Synchronise the device and read (and by default clear) the library's
    out-of-bounds index record; all zero unless indices left their tensors."""
    lib = lib or load_bounds()
    rec = DcnBoundsRecord()
    check(lib.dcn_debug_bounds_read(ctypes.byref(rec), 1 if reset else 0), lib)
    return rec


class DcnError(RuntimeError):
    def __init__(self, code: int, msg: str):
        super().__init__(f"[dcn error {code}] {msg}")
        self.code = code


def check(rc: int, lib: Optional[ctypes.CDLL] = None) -> None:
    if rc != DCN_OK:
        raise DcnError(rc, (lib or load()).dcn_last_error().decode())


def make_desc(dtype: int, input_shape, weight_shape, stride=(1, 1), padding=(0, 0),
              dilation=(1, 1), n_weight_grps=1, n_offset_grps=1, use_mask=False) -> DcnConvDesc:
    d = DcnConvDesc()
    d.dtype = dtype
    d.use_mask = 1 if use_mask else 0
    d.batch, d.in_channels, d.in_h, d.in_w = input_shape
    d.out_channels, _, d.kernel_h, d.kernel_w = weight_shape
    d.stride_h, d.stride_w = stride
    d.pad_h, d.pad_w = padding
    d.dilation_h, d.dilation_w = dilation
    d.n_weight_grps = n_weight_grps
    d.n_offset_grps = n_offset_grps
    return d


def profile_enable(on: bool) -> None:
    load().dcn_profile_enable(1 if on else 0)


def profile_summary(max_entries: int = 64):
    """[(kernel name, launches, total device ms)] recorded since profile_enable(True)."""
    lib = load()
    stride = 64
    names = ctypes.create_string_buffer(max_entries * stride)
    launches = (ctypes.c_uint64 * max_entries)()
    ms = (ctypes.c_double * max_entries)()
    n = lib.dcn_profile_summary(max_entries, names, stride, launches, ms)
    if n < 0:
        raise DcnError(DCN_ERR_CUDA, "profile summary failed")
    out = []
    for i in range(min(n, max_entries)):
        nm = names.raw[i * stride:(i + 1) * stride].split(b"\0", 1)[0].decode()
        out.append((nm, int(launches[i]), float(ms[i])))
    return out


def launch_count() -> int:
    return int(load().dcn_launch_count())


def output_size(d: DcnConvDesc, lib: Optional[ctypes.CDLL] = None):
    lib = lib or load()
    oh, ow = ctypes.c_int64(), ctypes.c_int64()
    check(lib.dcn_output_size(ctypes.byref(d), ctypes.byref(oh), ctypes.byref(ow)), lib)
    return oh.value, ow.value


# ---------------------------------------------------------------- torch helpers
def _torch_dtype_code(t) -> int:
    import torch
    return {torch.float32: DCN_FLOAT32, torch.float16: DCN_FLOAT16, torch.bfloat16: DCN_BFLOAT16}[t.dtype]


def _ptr(t) -> Optional[int]:
    return None if t is None else t.data_ptr()


def _stream(t) -> int:
    import torch
    return torch.cuda.current_stream(t.device).cuda_stream


def desc_for(input, weight, offset, stride=(1, 1), padding=(0, 0), dilation=(1, 1), mask=None):
    kh, kw = weight.shape[2], weight.shape[3]
    return make_desc(_torch_dtype_code(input), tuple(input.shape), tuple(weight.shape), stride,
                     padding, dilation, input.shape[1] // weight.shape[1],
                     offset.shape[1] // (2 * kh * kw), mask is not None)


def call_forward(input, offset, weight, bias=None, stride=(1, 1), padding=(0, 0), dilation=(1, 1),
                 mask=None, lib: Optional[ctypes.CDLL] = None):
    """Forward through the C ABI; tensors must be contiguous CUDA tensors.
    `lib`: another build of the library (default libdcn_b200.so)."""
    import torch
    lib = lib or load()
    d = desc_for(input, weight, offset, stride, padding, dilation, mask)
    oh, ow = output_size(d, lib)
    out = torch.empty((d.batch, d.out_channels, oh, ow), device=input.device, dtype=input.dtype)
    wsz = lib.dcn_forward_workspace_size(ctypes.byref(d))
    ws = torch.empty(max(wsz, 1), device=input.device, dtype=torch.uint8)
    check(lib.dcn_deform_conv2d_forward(ctypes.byref(d), _ptr(input), _ptr(weight), _ptr(offset),
                                        _ptr(mask), _ptr(bias), _ptr(out), _ptr(ws), wsz,
                                        _stream(input)), lib)
    return out


def call_backward(grad_output, input, offset, weight, stride=(1, 1), padding=(0, 0),
                  dilation=(1, 1), mask=None, with_bias=True, lib: Optional[ctypes.CDLL] = None):
    """All five gradients through the C ABI: (gI, gOff, gW, gB, gMask).
    `lib`: another build of the library (default libdcn_b200.so)."""
    import torch
    lib = lib or load()
    d = desc_for(input, weight, offset, stride, padding, dilation, mask)
    gi = torch.empty_like(input)
    goff = torch.empty_like(offset)
    gw = torch.empty_like(weight)
    gb = torch.empty(weight.shape[0], device=input.device, dtype=input.dtype) if with_bias else None
    gm = torch.empty_like(mask) if mask is not None else None
    wsz = lib.dcn_backward_workspace_size(ctypes.byref(d))
    ws = torch.empty(max(wsz, 1), device=input.device, dtype=torch.uint8)
    check(lib.dcn_deform_conv2d_backward(ctypes.byref(d), _ptr(grad_output), _ptr(input),
                                         _ptr(weight), _ptr(offset), _ptr(mask), _ptr(gi), _ptr(gw),
                                         _ptr(goff), _ptr(gm), _ptr(gb), _ptr(ws), wsz,
                                         _stream(input)), lib)
    return gi, goff, gw, gb, gm
