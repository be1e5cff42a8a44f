"""The allocation-free input-gradient entry point
(dcn_deform_conv2d_backward_input_noalloc), called through the C ABI.

It serves callers that cannot allocate device memory (plugin interfaces that
pass a kernel library only input/output pointers, real-time loops that forbid
allocation after start-up), so its fp32 accumulator is a fixed array inside the
library instead of a caller workspace.  This file checks, on the GPU, that two
calls in a row agree with the workspace-based dcn_deform_conv2d_backward_input
within the parity tolerance (1e-4 fp32, 1e-2 fp16/bf16, normwise relative) --
the second call also proves the array is cleared between calls -- and, on the
host, that problems above the array's size are refused.

The file name sorts last so that a run stopping at the first failure has
already run every other test.
"""
import ctypes

import pytest
import torch

from _util import TOL, rel_err, to_np

DTYPES = {"float32": torch.float32, "float16": torch.float16, "bfloat16": torch.bfloat16}
MAX_ELEMS = 2 * 1024 * 1024


def _problem(dev, dtype, seed=0):
    g = torch.Generator().manual_seed(seed)
    B, C, H, W, og, k = 2, 64, 40, 36, 2, 3
    oh, ow = H, W  # pad 1, stride 1
    off = (torch.randn(B, 2 * og * k * k, oh, ow, generator=g) * 2.0).to(dev, dtype)
    mask = torch.sigmoid(torch.randn(B, og * k * k, oh, ow, generator=g)).to(dev, dtype)
    gcol = torch.randn(C * k * k, B * oh * ow, generator=g).to(dev, dtype)
    return (B, C, H, W), off, mask, gcol, og


def _desc(shape, dtype, og, use_mask=True):
    from mps_deform_conv import _abi
    code = {torch.float32: _abi.DCN_FLOAT32, torch.float16: _abi.DCN_FLOAT16,
            torch.bfloat16: _abi.DCN_BFLOAT16}[dtype]
    return _abi.make_desc(code, shape, (1, shape[1], 3, 3), (1, 1), (1, 1), (1, 1), 1, og, use_mask)


@pytest.mark.gpu
@pytest.mark.parametrize("dtype", list(DTYPES))
def test_noalloc_matches_workspace_entry_point_twice(dtype, cuda):
    from mps_deform_conv import _abi
    lib = _abi.load()
    dt = DTYPES[dtype]
    shape, off, mask, gcol, og = _problem(cuda, dt)
    d = _desc(shape, dt, og)
    stream = torch.cuda.current_stream(cuda).cuda_stream

    ref = torch.empty(shape, device=cuda, dtype=dt)
    wsz = lib.dcn_backward_input_workspace_size(ctypes.byref(d))
    ws = torch.empty(max(wsz, 1), device=cuda, dtype=torch.uint8)
    _abi.check(lib.dcn_deform_conv2d_backward_input(ctypes.byref(d), gcol.data_ptr(), off.data_ptr(),
                                                    mask.data_ptr(), ref.data_ptr(), ws.data_ptr(),
                                                    wsz, stream))
    outs = []
    for _ in range(2):  # two calls in a row share the library's array
        out = torch.full(shape, float("nan"), device=cuda, dtype=dt)
        _abi.check(lib.dcn_deform_conv2d_backward_input_noalloc(
            ctypes.byref(d), gcol.data_ptr(), off.data_ptr(), mask.data_ptr(), out.data_ptr(), stream))
        outs.append(out)
    torch.cuda.synchronize()
    for out in outs:
        assert torch.isfinite(out).all()
        assert rel_err(to_np(out), to_np(ref)) <= TOL[dtype]


def test_noalloc_refuses_problems_above_its_array():
    from mps_deform_conv import _abi
    lib = _abi.load()
    d = _desc((1, 64, 256, 256), torch.bfloat16, 1)  # 4,194,304 elements > 2,097,152
    rc = lib.dcn_deform_conv2d_backward_input_noalloc(ctypes.byref(d), None, None, None, None, None)
    assert rc == _abi.DCN_ERR_UNSUPPORTED
    msg = lib.dcn_last_error().decode()
    assert "2097152" in msg and "workspace" in msg
