"""Forward weight images of forward-only calls (dcn_weight_image,
DCN_EX_WEIGHT_IMAGE, mps_deform_conv.set_weight_image_cache): a forward from
a prebuilt or cached image is bitwise the forward that rebuilds it, a cache
hit skips the rebuild (one launch fewer), and the cache follows in-place
weight updates through the tensor's version counter."""
import ctypes

import numpy as np
import pytest
import torch

from _util import assert_close
from oracle import oracle

pytestmark = pytest.mark.gpu

DTYPES = {"float16": torch.float16, "bfloat16": torch.bfloat16}


def _inputs(dev, dt, B=2, C=128, H=11, W=10, Co=128, G=2, og=2, seed=0):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(B, C, H, W, generator=g).to(dev, dt)
    w = (torch.randn(Co, C // G, 3, 3, generator=g) / np.sqrt(C // G * 9)).to(dev, dt)
    off = (torch.randn(B, 2 * og * 9, H, W, generator=g) * 2).to(dev, dt)
    m = torch.sigmoid(torch.randn(B, og * 9, H, W, generator=g)).to(dev, dt)
    b = (torch.randn(Co, generator=g) * 0.1).to(dev, dt)
    return x, w, off, m, b


@pytest.fixture
def image_cache():
    import mps_deform_conv as mdc
    mdc.set_weight_image_cache(True)
    yield mdc
    mdc.set_weight_image_cache(False)


@pytest.mark.parametrize("dtype", list(DTYPES))
@pytest.mark.parametrize("channels_last", [False, True])
def test_cached_image_forward_is_bitwise_and_skips_rebuild(dtype, channels_last, cuda, image_cache):
    mdc = image_cache
    from mps_deform_conv import _abi
    x, w, off, m, b = _inputs(cuda, DTYPES[dtype])
    if channels_last:
        x = x.contiguous(memory_format=torch.channels_last)
    with torch.no_grad():
        mdc.set_weight_image_cache(False)
        ref = mdc.deform_conv2d(x, off, w, b, 1, 1, 1, m)
        mdc.set_weight_image_cache(True)
        n0 = _abi.launch_count()
        first = mdc.deform_conv2d(x, off, w, b, 1, 1, 1, m)
        n1 = _abi.launch_count()
        second = mdc.deform_conv2d(x, off, w, b, 1, 1, 1, m)
        n2 = _abi.launch_count()
    torch.cuda.synchronize()
    assert torch.equal(first, ref) and torch.equal(second, ref)
    assert n2 - n1 == (n1 - n0) - 1, (n1 - n0, n2 - n1)
    cast = [t.double() for t in (x, off, w, b, m)]
    assert_close(second, oracle.forward(cast[0], cast[1], cast[2], cast[3], 1, 1, 1, cast[4]), dtype, "out")


@pytest.mark.parametrize("dtype", list(DTYPES))
def test_cache_follows_in_place_weight_updates(dtype, cuda, image_cache):
    mdc = image_cache
    x, w, off, m, b = _inputs(cuda, DTYPES[dtype], seed=1)
    with torch.no_grad():
        before = mdc.deform_conv2d(x, off, w, b, 1, 1, 1, m)
        w.mul_(-0.5)  # bumps w._version
        after = mdc.deform_conv2d(x, off, w, b, 1, 1, 1, m)
        mdc.set_weight_image_cache(False)
        expect = mdc.deform_conv2d(x, off, w, b, 1, 1, 1, m)
    torch.cuda.synchronize()
    assert torch.equal(after, expect)
    assert not torch.equal(after, before)


def test_training_forward_ignores_the_cache(cuda, image_cache):
    """A forward that keeps state for the backward builds both images itself."""
    mdc = image_cache
    x, w, off, m, b = _inputs(cuda, torch.bfloat16, seed=2)
    with torch.no_grad():
        mdc.deform_conv2d(x, off, w, b, 1, 1, 1, m)  # fills the cache
    wl = w.clone().requires_grad_(True)
    out = mdc.deform_conv2d(x, off, wl, b, 1, 1, 1, m)
    gw, = torch.autograd.grad(out, [wl], torch.ones_like(out))
    mdc.set_weight_image_cache(False)
    wl2 = w.clone().requires_grad_(True)
    out2 = mdc.deform_conv2d(x, off, wl2, b, 1, 1, 1, m)
    gw2, = torch.autograd.grad(out2, [wl2], torch.ones_like(out2))
    assert torch.equal(out, out2) and torch.equal(gw, gw2)


@pytest.mark.parametrize("dtype", list(DTYPES))
def test_abi_weight_image_forward(dtype, cuda):
    """dcn_weight_image + dcn_deform_conv2d_forward_ex(flags = DCN_EX_WEIGHT_IMAGE)
    equals the plain forward bitwise; backward options reject the flag."""
    from mps_deform_conv import _abi
    lib = _abi.load()
    x, w, off, m, b = _inputs(cuda, DTYPES[dtype], seed=3)
    ref = _abi.call_forward(x, off, w, b, (1, 1), (1, 1), (1, 1), m)
    d = _abi.desc_for(x, w, off, (1, 1), (1, 1), (1, 1), m)
    nbytes = lib.dcn_weight_image_bytes(ctypes.byref(d))
    assert nbytes == w.numel() * w.element_size()
    img = torch.empty(nbytes, device=cuda, dtype=torch.uint8)
    st = torch.cuda.current_stream(cuda).cuda_stream
    _abi.check(lib.dcn_weight_image(ctypes.byref(d), w.data_ptr(), img.data_ptr(), nbytes, st))
    opt = _abi.DcnExOptions(_abi.DCN_LAYOUT_NCHW, _abi.DCN_LAYOUT_NCHW, 0, _abi.DCN_EX_WEIGHT_IMAGE)
    assert lib.dcn_ex_supported(ctypes.byref(d), ctypes.byref(opt), 1) == 0
    out = torch.empty_like(ref)
    wsz = lib.dcn_forward_workspace_size(ctypes.byref(d))
    ws = torch.empty(max(wsz, 1), device=cuda, dtype=torch.uint8)
    _abi.check(lib.dcn_deform_conv2d_forward_ex(ctypes.byref(d), ctypes.byref(opt), x.data_ptr(), img.data_ptr(),
                                                off.data_ptr(), m.data_ptr(), b.data_ptr(), out.data_ptr(), None, 0,
                                                ws.data_ptr(), wsz, st))
    torch.cuda.synchronize()
    assert torch.equal(out, ref)
