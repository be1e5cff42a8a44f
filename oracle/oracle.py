"""CPU parity oracle for deform_conv2d (forward and backward), float64.

TEST INFRASTRUCTURE ONLY.  Used by tests/, by ``__graft_entry__.smoke()`` and by
the CPU-baseline leg of ``bench.py`` as the checker; never by the product path.
It wraps ``oracle/dcn_oracle.c`` (a restatement of the reference's Metal
kernels in ``mps_deform_conv/csrc/deform_conv2d_mps.mm``) through ctypes.

The restatement is pinned against ``torchvision.ops.deform_conv2d`` on CPU in
float64 by the fixtures in ``tests/golden/`` (see ``tests/test_oracle_golden.py``).
"""
from __future__ import annotations

import ctypes
import os
import subprocess
from typing import Optional

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "_build", "libdcn_oracle.so")
_lib = None


class _Shape(ctypes.Structure):
    _fields_ = [(n, ctypes.c_int64) for n in (
        "B", "C", "H", "W", "Co", "kh", "kw", "sh", "sw", "ph", "pw", "dh", "dw",
        "groups", "og", "use_mask", "Ho", "Wo")]


def build() -> str:
    """Compile the oracle shared library (gcc) if it is missing or stale."""
    src = os.path.join(_HERE, "dcn_oracle.c")
    if (not os.path.exists(_LIB_PATH)) or os.path.getmtime(_LIB_PATH) < os.path.getmtime(src):
        subprocess.check_call(["make", "-s", "-C", _HERE])
    return _LIB_PATH


def _load():
    global _lib
    if _lib is None:
        build()
        lib = ctypes.CDLL(_LIB_PATH)
        P = ctypes.POINTER(ctypes.c_double)
        S = ctypes.POINTER(_Shape)
        lib.dcn_oracle_im2col.argtypes = [S, P, P, P, P]
        lib.dcn_oracle_col2im.argtypes = [S, P, P, P, P]
        lib.dcn_oracle_col2im_coord.argtypes = [S, P, P, P, P, P, P]
        lib.dcn_oracle_forward.argtypes = [S, P, P, P, P, P, P]
        lib.dcn_oracle_backward.argtypes = [S, P, P, P, P, P, P, P, P, P, P]
        for f in (lib.dcn_oracle_im2col, lib.dcn_oracle_col2im, lib.dcn_oracle_col2im_coord,
                  lib.dcn_oracle_forward, lib.dcn_oracle_backward):
            f.restype = None
        _lib = lib
    return _lib


def _arr(a) -> np.ndarray:
    if a is None:
        return None
    if hasattr(a, "detach"):  # torch tensor
        a = a.detach().to("cpu").double().numpy()
    return np.ascontiguousarray(np.asarray(a, dtype=np.float64))


def _ptr(a: Optional[np.ndarray]):
    if a is None:
        return ctypes.POINTER(ctypes.c_double)()
    return a.ctypes.data_as(ctypes.POINTER(ctypes.c_double))


def make_shape(input_shape, weight_shape, stride=(1, 1), padding=(0, 0), dilation=(1, 1),
               offset_groups=1, use_mask=False) -> _Shape:
    B, C, H, W = input_shape
    Co, cig, kh, kw = weight_shape
    s = _Shape()
    s.B, s.C, s.H, s.W = B, C, H, W
    s.Co, s.kh, s.kw = Co, kh, kw
    s.sh, s.sw = stride
    s.ph, s.pw = padding
    s.dh, s.dw = dilation
    s.groups = C // cig
    s.og = offset_groups
    s.use_mask = 1 if use_mask else 0
    s.Ho = (H + 2 * s.ph - (s.dh * (kh - 1) + 1)) // s.sh + 1
    s.Wo = (W + 2 * s.pw - (s.dw * (kw - 1) + 1)) // s.sw + 1
    return s


def _pair(v):
    return (v, v) if isinstance(v, int) else tuple(v)


def _og_of(offset, weight):
    kh, kw = weight.shape[2], weight.shape[3]
    return offset.shape[1] // (2 * kh * kw)


def forward(input, offset, weight, bias=None, stride=(1, 1), padding=(0, 0), dilation=(1, 1),
            mask=None) -> np.ndarray:
    """float64 forward with the reference's argument order."""
    x, off, w = _arr(input), _arr(offset), _arr(weight)
    b, m = _arr(bias), _arr(mask)
    s = make_shape(x.shape, w.shape, _pair(stride), _pair(padding), _pair(dilation),
                   _og_of(off, w), m is not None)
    out = np.zeros((s.B, s.Co, s.Ho, s.Wo), dtype=np.float64)
    _load().dcn_oracle_forward(ctypes.byref(s), _ptr(x), _ptr(off), _ptr(m), _ptr(w), _ptr(b), _ptr(out))
    return out


def backward(grad_out, input, offset, weight, stride=(1, 1), padding=(0, 0), dilation=(1, 1),
             mask=None, with_bias=True):
    """float64 gradients (grad_input, grad_offset, grad_weight, grad_bias, grad_mask)."""
    go, x, off, w, m = _arr(grad_out), _arr(input), _arr(offset), _arr(weight), _arr(mask)
    s = make_shape(x.shape, w.shape, _pair(stride), _pair(padding), _pair(dilation),
                   _og_of(off, w), m is not None)
    gi = np.zeros_like(x)
    goff = np.zeros_like(off)
    gw = np.zeros_like(w)
    gb = np.zeros((s.Co,), dtype=np.float64) if with_bias else None
    gm = np.zeros_like(m) if m is not None else None
    _load().dcn_oracle_backward(ctypes.byref(s), _ptr(go), _ptr(x), _ptr(off), _ptr(m), _ptr(w),
                                _ptr(gi), _ptr(goff), _ptr(gm), _ptr(gw), _ptr(gb))
    return gi, goff, gw, gb, gm


def im2col(input, offset, mask, kernel_h, kernel_w, stride=(1, 1), padding=(0, 0),
           dilation=(1, 1), offset_groups=1) -> np.ndarray:
    """Column buffer [C*kh*kw, B*Ho*Wo] (the reference's deformable_im2col)."""
    x, off, m = _arr(input), _arr(offset), _arr(mask)
    s = make_shape(x.shape, (1, x.shape[1], kernel_h, kernel_w), _pair(stride), _pair(padding),
                   _pair(dilation), offset_groups, m is not None)
    cols = np.zeros((s.C * kernel_h * kernel_w, s.B * s.Ho * s.Wo), dtype=np.float64)
    _load().dcn_oracle_im2col(ctypes.byref(s), _ptr(x), _ptr(off), _ptr(m), _ptr(cols))
    return cols


def col2im(grad_columns, input_shape, offset, mask, kernel_h, kernel_w, stride=(1, 1),
           padding=(0, 0), dilation=(1, 1), offset_groups=1) -> np.ndarray:
    """grad_input from a column gradient (the reference's backward_input)."""
    gc, off, m = _arr(grad_columns), _arr(offset), _arr(mask)
    s = make_shape(tuple(input_shape), (1, input_shape[1], kernel_h, kernel_w), _pair(stride),
                   _pair(padding), _pair(dilation), offset_groups, m is not None)
    gi = np.zeros(tuple(input_shape), dtype=np.float64)
    _load().dcn_oracle_col2im(ctypes.byref(s), _ptr(gc), _ptr(off), _ptr(m), _ptr(gi))
    return gi


def col2im_coord(grad_columns, input, offset, mask, kernel_h, kernel_w, stride=(1, 1),
                 padding=(0, 0), dilation=(1, 1), offset_groups=1):
    """(grad_offset, grad_mask) from a column gradient (backward_offset_mask)."""
    gc, x, off, m = _arr(grad_columns), _arr(input), _arr(offset), _arr(mask)
    s = make_shape(x.shape, (1, x.shape[1], kernel_h, kernel_w), _pair(stride), _pair(padding),
                   _pair(dilation), offset_groups, m is not None)
    goff = np.zeros_like(off)
    gm = np.zeros_like(m) if m is not None else None
    _load().dcn_oracle_col2im_coord(ctypes.byref(s), _ptr(gc), _ptr(x), _ptr(off), _ptr(m),
                                    _ptr(goff), _ptr(gm))
    return goff, gm


def param_grads(grad_out, input, offset, weight, stride=(1, 1), padding=(0, 0), dilation=(1, 1),
                mask=None):
    """float64 (grad_weight, grad_bias) for problems too large for the scalar
    loops of dcn_oracle_backward.  Same arithmetic, per weight group
    (mps_deform_conv/__init__.py:266-286, with the per-group products the
    forward's grouped bmm implies): the columns come from the C restatement of
    deformable_im2col, grad_weight_g = grad_out_g . columns_g^T is a float64
    numpy (BLAS) product and grad_bias is the sum of grad_out over batch and
    pixels."""
    x, off, w, m = _arr(input), _arr(offset), _arr(weight), _arr(mask)
    go = _arr(grad_out)
    Co, cig, kh, kw = w.shape
    G = x.shape[1] // cig
    og = _og_of(off, w)
    cols = im2col(x, off, m, kh, kw, _pair(stride), _pair(padding), _pair(dilation), og)
    P = cols.shape[1]
    go2 = np.ascontiguousarray(go.transpose(1, 0, 2, 3).reshape(Co, P))
    K = cig * kh * kw
    cog = Co // G
    gw = np.empty((Co, K), dtype=np.float64)
    for g in range(G):
        gw[g * cog:(g + 1) * cog] = go2[g * cog:(g + 1) * cog] @ cols[g * K:(g + 1) * K].T
    return gw.reshape(w.shape), go2.sum(axis=1)
