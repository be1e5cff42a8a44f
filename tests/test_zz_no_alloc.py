"""The allocation-free input-gradient entry point
(dcn_deform_conv2d_backward_input_noalloc), called through the C ABI.

It serves callers that cannot allocate device memory (plugin interfaces that
pass a kernel library only input/output pointers, real-time loops that forbid
allocation after start-up), so its fp32 accumulator for fp16/bf16 data is a
fixed array inside the library instead of a caller workspace.  This file
checks, on the GPU, that calls in a row agree with the workspace-based
dcn_deform_conv2d_backward_input within the parity tolerance (1e-4 fp32,
1e-2 fp16/bf16, normwise relative):
  * two calls in a row, with and without a mask (the second call proves the
    array is cleared between calls);
  * a bf16 problem of exactly 2,097,152 grad_input elements (the whole array);
  * a large call followed by a smaller one with different data.
On the host it checks that fp16/bf16 problems above the array's size are
refused and that fp32 problems, which never use the array, are not.

The file name sorts last so that a run stopping at the first failure has
already run every other test.
"""
import ctypes

import pytest
import torch

from _util import TOL, rel_err, to_np

DTYPES = {"float32": torch.float32, "float16": torch.float16, "bfloat16": torch.bfloat16}
MAX_ELEMS = 2 * 1024 * 1024


def _problem(dev, dtype, shape=(2, 64, 40, 36), og=2, seed=0, use_mask=True):
    g = torch.Generator().manual_seed(seed)
    B, C, H, W = shape
    k = 3
    oh, ow = H, W  # pad 1, stride 1
    off = (torch.randn(B, 2 * og * k * k, oh, ow, generator=g) * 2.0).to(dev, dtype)
    mask = torch.sigmoid(torch.randn(B, og * k * k, oh, ow, generator=g)).to(dev, dtype) if use_mask else None
    gcol = torch.randn(C * k * k, B * oh * ow, generator=g).to(dev, dtype)
    return shape, off, mask, gcol, og


def _desc(shape, dtype, og, use_mask=True):
    from mps_deform_conv import _abi
    code = {torch.float32: _abi.DCN_FLOAT32, torch.float16: _abi.DCN_FLOAT16,
            torch.bfloat16: _abi.DCN_BFLOAT16}[dtype]
    return _abi.make_desc(code, shape, (1, shape[1], 3, 3), (1, 1), (1, 1), (1, 1), 1, og, use_mask)


def _workspace_path(lib, d, shape, dt, gcol, off, mask, dev, stream):
    from mps_deform_conv import _abi
    ref = torch.empty(shape, device=dev, dtype=dt)
    wsz = lib.dcn_backward_input_workspace_size(ctypes.byref(d))
    ws = torch.empty(max(wsz, 1), device=dev, dtype=torch.uint8)
    _abi.check(lib.dcn_deform_conv2d_backward_input(ctypes.byref(d), gcol.data_ptr(), off.data_ptr(),
                                                    mask.data_ptr() if mask is not None else None,
                                                    ref.data_ptr(), ws.data_ptr(), wsz, stream))
    return ref


def _noalloc(lib, d, shape, dt, gcol, off, mask, dev, stream):
    from mps_deform_conv import _abi
    out = torch.full(shape, float("nan"), device=dev, dtype=dt)
    _abi.check(lib.dcn_deform_conv2d_backward_input_noalloc(
        ctypes.byref(d), gcol.data_ptr(), off.data_ptr(), mask.data_ptr() if mask is not None else None,
        out.data_ptr(), stream))
    return out


@pytest.mark.gpu
@pytest.mark.parametrize("use_mask", [True, False])
@pytest.mark.parametrize("dtype", list(DTYPES))
def test_noalloc_matches_workspace_entry_point_twice(dtype, use_mask, cuda):
    from mps_deform_conv import _abi
    lib = _abi.load()
    dt = DTYPES[dtype]
    shape, off, mask, gcol, og = _problem(cuda, dt, use_mask=use_mask)
    d = _desc(shape, dt, og, use_mask)
    stream = torch.cuda.current_stream(cuda).cuda_stream
    ref = _workspace_path(lib, d, shape, dt, gcol, off, mask, cuda, stream)
    outs = [_noalloc(lib, d, shape, dt, gcol, off, mask, cuda, stream) for _ in range(2)]
    torch.cuda.synchronize()
    for out in outs:
        assert torch.isfinite(out).all()
        assert rel_err(to_np(out), to_np(ref)) <= TOL[dtype]


@pytest.mark.gpu
def test_noalloc_at_the_array_size_then_a_smaller_call(cuda):
    """A bf16 problem whose grad_input fills the whole array (B*C*H*W =
    2,097,152: the `>` limit admits it), then a smaller problem with other
    data: the second result must not keep anything of the first."""
    from mps_deform_conv import _abi
    lib = _abi.load()
    dt = torch.bfloat16
    stream = torch.cuda.current_stream(cuda).cuda_stream
    big = (2, 64, 128, 128)
    assert big[0] * big[1] * big[2] * big[3] == MAX_ELEMS
    small = (1, 32, 24, 20)
    for shape, og, seed in ((big, 4, 1), (small, 2, 2)):
        shape, off, mask, gcol, og = _problem(cuda, dt, shape=shape, og=og, seed=seed)
        d = _desc(shape, dt, og)
        ref = _workspace_path(lib, d, shape, dt, gcol, off, mask, cuda, stream)
        out = _noalloc(lib, d, shape, dt, gcol, off, mask, cuda, stream)
        torch.cuda.synchronize()
        assert torch.isfinite(out).all()
        assert rel_err(to_np(out), to_np(ref)) <= TOL["bfloat16"], shape


@pytest.mark.parametrize("dtype", ["float16", "bfloat16"])
def test_noalloc_refuses_16bit_problems_above_its_array(dtype):
    from mps_deform_conv import _abi
    lib = _abi.load()
    d = _desc((1, 64, 256, 256), DTYPES[dtype], 1)  # 4,194,304 elements > 2,097,152
    rc = lib.dcn_deform_conv2d_backward_input_noalloc(ctypes.byref(d), None, None, None, None, None)
    assert rc == _abi.DCN_ERR_UNSUPPORTED
    msg = lib.dcn_last_error().decode()
    assert "2097152" in msg and "workspace" in msg


def test_noalloc_fp32_has_no_array_limit():
    """fp32 accumulates in grad_input itself, so a problem above the array's
    size passes the size check (the NULL pointers are what is refused here)."""
    from mps_deform_conv import _abi
    lib = _abi.load()
    d = _desc((1, 64, 256, 256), torch.float32, 1)
    rc = lib.dcn_deform_conv2d_backward_input_noalloc(ctypes.byref(d), None, None, None, None, None)
    assert rc == _abi.DCN_ERR_INVALID_ARGUMENT
    assert "NULL" in lib.dcn_last_error().decode()
