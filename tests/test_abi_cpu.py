"""The C ABI library loads, exports every declared symbol, and its host-side
checks behave like the reference's (no GPU needed: nothing here launches)."""
import ctypes
import os
import re

import pytest

from conftest import REPO

HEADER = os.path.join(REPO, "include", "dcn_b200.h")


def declared_functions():
    src = open(HEADER).read()
    return sorted(set(re.findall(r"DCN_API\s+[\w\s\*]+?\b(dcn_\w+)\s*\(", src)))


def test_library_loads_and_exports_every_declared_symbol():
    from mps_deform_conv import _abi
    lib = _abi.load()
    names = declared_functions()
    assert len(names) >= 14
    for n in names:
        assert hasattr(lib, n), f"libdcn_b200.so does not export {n}"
    # and the ctypes binding declares exactly the header's surface
    assert set(_abi.SIGNATURES) == set(names)


def test_bounds_library_exports_the_same_surface():
    """libdcn_b200_bounds.so (build.py, -DDCN_DEBUG_BOUNDS) exports the same
    symbols; only it reports the index checks as compiled in."""
    from mps_deform_conv import _abi
    assert os.path.exists(_abi.BOUNDS_LIB_PATH)
    blib = _abi.load_bounds()
    for n in declared_functions():
        assert hasattr(blib, n), f"libdcn_b200_bounds.so does not export {n}"
    assert blib.dcn_debug_bounds_enabled() == 1
    assert _abi.load().dcn_debug_bounds_enabled() == 0


def test_abi_version():
    from mps_deform_conv import _abi
    assert _abi.load().dcn_abi_version() >= 100


def _desc(**kw):
    from mps_deform_conv import _abi
    base = dict(dtype=_abi.DCN_FLOAT32, input_shape=(1, 4, 8, 8), weight_shape=(4, 4, 3, 3))
    base.update(kw)
    return _abi.make_desc(base.pop("dtype"), base.pop("input_shape"), base.pop("weight_shape"), **base)


@pytest.mark.parametrize("kw,needle", [
    (dict(stride=(0, 1)), "stride must be positive"),
    (dict(dilation=(1, 0)), "dilation must be positive"),
    (dict(padding=(-1, 0)), "padding must be non-negative"),
    (dict(n_weight_grps=3), "divisible"),
    (dict(n_offset_grps=3), "divisible"),
    (dict(input_shape=(1, 4, 4, 4), weight_shape=(4, 4, 5, 5), stride=(2, 2)), "Invalid output dimensions"),
    (dict(dtype=7), "dtype"),
    (dict(input_shape=(70000, 512, 64, 64)), "exceeds int32 limit"),
])
def test_validate_messages(kw, needle):
    from mps_deform_conv import _abi
    lib = _abi.load()
    d = _desc(**kw)
    rc = lib.dcn_validate(ctypes.byref(d))
    assert rc != _abi.DCN_OK
    assert needle in lib.dcn_last_error().decode()


def test_validate_ok_and_output_size():
    from mps_deform_conv import _abi
    lib = _abi.load()
    d = _desc(padding=(1, 1))
    assert lib.dcn_validate(ctypes.byref(d)) == _abi.DCN_OK
    assert _abi.output_size(d) == (8, 8)
    d = _desc(stride=(2, 2), dilation=(2, 2), padding=(2, 2), input_shape=(1, 4, 9, 8))
    assert _abi.output_size(d) == (5, 4)


def test_workspace_sizes_are_host_queries():
    from mps_deform_conv import _abi
    lib = _abi.load()
    d = _desc(dtype=_abi.DCN_BFLOAT16, input_shape=(2, 64, 16, 16), weight_shape=(64, 64, 3, 3),
              padding=(1, 1), use_mask=True)
    assert lib.dcn_backward_workspace_size(ctypes.byref(d)) > 0
    assert lib.dcn_backward_input_workspace_size(ctypes.byref(d)) == 2 * 64 * 16 * 16 * 4
    bad = _desc(stride=(0, 0))
    assert lib.dcn_backward_workspace_size(ctypes.byref(bad)) == 0
    # every query of every path, on every dtype, including an empty batch
    for dt in (_abi.DCN_FLOAT32, _abi.DCN_FLOAT16, _abi.DCN_BFLOAT16):
        for shape in ((0, 64, 16, 16), (1, 64, 16, 16), (2, 4, 5, 6)):
            q = _desc(dtype=dt, input_shape=shape, weight_shape=(64 if shape[1] == 64 else 4, shape[1], 3, 3),
                      padding=(1, 1), use_mask=True)
            for fn in ("dcn_forward_workspace_size", "dcn_backward_workspace_size",
                       "dcn_backward_input_workspace_size", "dcn_saved_state_bytes"):
                assert getattr(lib, fn)(ctypes.byref(q)) >= 0
            assert lib.dcn_head_supported(ctypes.byref(q)) in (0, 1)
    # the fp32 forward materializes its columns [C*T][P] (fp32) for the
    # tensor-core GEMM, in slices of whole images of at most 1 GiB
    small = _desc(input_shape=(1, 64, 16, 16), weight_shape=(64, 64, 3, 3), padding=(1, 1))
    assert lib.dcn_forward_workspace_size(ctypes.byref(small)) == 64 * 9 * 256 * 4
    big = _desc(input_shape=(4, 64, 512, 512), weight_shape=(64, 64, 3, 3), padding=(1, 1))
    per_image = 64 * 9 * 512 * 512 * 4  # 604 MB: one image per slice
    assert lib.dcn_forward_workspace_size(ctypes.byref(big)) == per_image
    # 2x128x64x64: both images in one slice; the GEMM writes the output
    # directly (no K-split partials)
    c2 = _desc(input_shape=(2, 128, 64, 64), weight_shape=(128, 128, 3, 3), padding=(1, 1), use_mask=True)
    assert lib.dcn_forward_workspace_size(ctypes.byref(c2)) == 128 * 9 * 8192 * 4


def test_forward_rejects_null_and_small_workspace_without_launching():
    from mps_deform_conv import _abi
    lib = _abi.load()
    d = _desc(padding=(1, 1))
    rc = lib.dcn_deform_conv2d_forward(ctypes.byref(d), None, None, None, None, None, None, None, 0, None)
    assert rc == _abi.DCN_ERR_INVALID_ARGUMENT
    assert "NULL" in lib.dcn_last_error().decode()
    bd = _desc(padding=(1, 1))
    rc = lib.dcn_deform_conv2d_backward(ctypes.byref(bd), ctypes.c_void_p(16), ctypes.c_void_p(16),
                                        ctypes.c_void_p(16), ctypes.c_void_p(16), None, None, None,
                                        None, None, None, None, 0, None)
    assert rc == _abi.DCN_ERR_WORKSPACE


def test_head_layout_support_query_and_rejection_without_launching():
    """The fused DCNv2 head layout is a tensor-core-only path: the query is a
    host computation, and an unsupported problem is rejected before any
    pointer is touched."""
    from mps_deform_conv import _abi
    lib = _abi.load()
    ok = _desc(dtype=_abi.DCN_BFLOAT16, input_shape=(2, 64, 16, 16), weight_shape=(64, 64, 3, 3), padding=(1, 1),
               use_mask=True)
    assert lib.dcn_head_supported(ctypes.byref(ok)) == 1
    for kw in (dict(dtype=_abi.DCN_FLOAT32),           # SIMT path
               dict(n_offset_grps=8),                   # 8 channels per offset group: 16-channel dgrad slabs
               dict(use_mask=False)):                   # the head layout carries a mask
        base = dict(dtype=_abi.DCN_BFLOAT16, input_shape=(2, 64, 16, 16), weight_shape=(64, 64, 3, 3),
                    padding=(1, 1), use_mask=True)
        base.update(kw)
        bad = _desc(**base)
        assert lib.dcn_head_supported(ctypes.byref(bad)) == 0
        rc = lib.dcn_deform_conv2d_forward_head(ctypes.byref(bad), ctypes.c_void_p(16), ctypes.c_void_p(16),
                                                ctypes.c_void_p(16), None, ctypes.c_void_p(16), None, 0, None, 0,
                                                None)
        assert rc == _abi.DCN_ERR_UNSUPPORTED
        assert "head layout" in lib.dcn_last_error().decode()


def test_ex_layout_options_checked_without_launching():
    """dcn_*_ex: channels-last layouts need the tensor-core path, channels-last
    pointers must be 16-byte aligned, and plain options behave like the
    training pair; every check here returns before anything is launched."""
    from mps_deform_conv import _abi
    lib = _abi.load()
    nhwc = _abi.DcnExOptions(_abi.DCN_LAYOUT_NHWC, _abi.DCN_LAYOUT_NHWC, 0, 0)
    plain = _abi.DcnExOptions(_abi.DCN_LAYOUT_NCHW, _abi.DCN_LAYOUT_NCHW, 0, 0)
    bad_layout = _abi.DcnExOptions(7, _abi.DCN_LAYOUT_NCHW, 0, 0)
    tc = _desc(dtype=_abi.DCN_BFLOAT16, input_shape=(2, 64, 16, 16), weight_shape=(64, 64, 3, 3), padding=(1, 1),
               use_mask=True)
    f32 = _desc(input_shape=(2, 64, 16, 16), weight_shape=(64, 64, 3, 3), padding=(1, 1), use_mask=True)
    assert lib.dcn_ex_supported(ctypes.byref(tc), ctypes.byref(nhwc), 0) == 1
    assert lib.dcn_ex_supported(ctypes.byref(tc), ctypes.byref(nhwc), 1) == 1
    assert lib.dcn_ex_supported(ctypes.byref(f32), ctypes.byref(nhwc), 0) == 0
    assert lib.dcn_ex_supported(ctypes.byref(f32), ctypes.byref(plain), 1) == 1   # any problem, any path
    assert lib.dcn_ex_supported(ctypes.byref(f32), None, 1) == 1
    assert lib.dcn_ex_supported(ctypes.byref(tc), ctypes.byref(bad_layout), 0) == 0
    p = ctypes.c_void_p(16)
    rc = lib.dcn_deform_conv2d_forward_ex(ctypes.byref(f32), ctypes.byref(nhwc), p, p, p, p, None, p, None, 0,
                                          None, 0, None)
    assert rc == _abi.DCN_ERR_UNSUPPORTED
    rc = lib.dcn_deform_conv2d_forward_ex(ctypes.byref(tc), ctypes.byref(nhwc), ctypes.c_void_p(18), p, p, p, None,
                                          p, None, 0, None, 0, None)
    assert rc == _abi.DCN_ERR_INVALID_ARGUMENT
    assert "16-byte aligned" in lib.dcn_last_error().decode()
    rc = lib.dcn_deform_conv2d_backward_ex(ctypes.byref(tc), ctypes.byref(nhwc), p, ctypes.c_void_p(34), p, p, p,
                                           None, 0, p, p, p, p, None, None, 0, None)
    assert rc == _abi.DCN_ERR_INVALID_ARGUMENT
    rc = lib.dcn_deform_conv2d_forward_ex(ctypes.byref(tc), None, None, None, None, None, None, None, None, 0,
                                          None, 0, None)
    assert rc == _abi.DCN_ERR_INVALID_ARGUMENT and "NULL" in lib.dcn_last_error().decode()


def test_weight_image_queries_and_flag_checks():
    """Forward weight images: the size query, and the options that accept or
    reject DCN_EX_WEIGHT_IMAGE (host logic, nothing launches)."""
    from mps_deform_conv import _abi
    lib = _abi.load()
    tc = _desc(dtype=_abi.DCN_BFLOAT16, input_shape=(2, 128, 16, 16), weight_shape=(64, 64, 3, 3),
               padding=(1, 1), use_mask=True, n_weight_grps=2)
    f32 = _desc(input_shape=(2, 64, 16, 16), weight_shape=(64, 64, 3, 3), padding=(1, 1), use_mask=True)
    assert lib.dcn_weight_image_bytes(ctypes.byref(tc)) == 64 * 64 * 9 * 2
    assert lib.dcn_weight_image_bytes(ctypes.byref(f32)) == 0
    img = _abi.DcnExOptions(_abi.DCN_LAYOUT_NCHW, _abi.DCN_LAYOUT_NCHW, 0, _abi.DCN_EX_WEIGHT_IMAGE)
    img_nhwc = _abi.DcnExOptions(_abi.DCN_LAYOUT_NHWC, _abi.DCN_LAYOUT_NHWC, 0, _abi.DCN_EX_WEIGHT_IMAGE)
    unknown = _abi.DcnExOptions(_abi.DCN_LAYOUT_NCHW, _abi.DCN_LAYOUT_NCHW, 0, 2)
    assert lib.dcn_ex_supported(ctypes.byref(tc), ctypes.byref(img), 0) == 1
    assert lib.dcn_ex_supported(ctypes.byref(tc), ctypes.byref(img_nhwc), 0) == 1
    assert lib.dcn_ex_supported(ctypes.byref(tc), ctypes.byref(img), 1) == 0      # forward only
    assert lib.dcn_ex_supported(ctypes.byref(f32), ctypes.byref(img), 0) == 0     # tensor-core problems only
    assert lib.dcn_ex_supported(ctypes.byref(tc), ctypes.byref(unknown), 0) == 0  # unknown flag bits
    p = ctypes.c_void_p(16)
    rc = lib.dcn_weight_image(ctypes.byref(f32), p, p, 1 << 20, None)
    assert rc == _abi.DCN_ERR_UNSUPPORTED
    rc = lib.dcn_weight_image(ctypes.byref(tc), p, p, 100, None)
    assert rc == _abi.DCN_ERR_WORKSPACE
    rc = lib.dcn_weight_image(ctypes.byref(tc), p, ctypes.c_void_p(24), 1 << 20, None)
    assert rc == _abi.DCN_ERR_INVALID_ARGUMENT and "16-byte" in lib.dcn_last_error().decode()
    # an image with saved state is refused before anything launches
    rc = lib.dcn_deform_conv2d_forward_ex(ctypes.byref(tc), ctypes.byref(img), p, p, p, p, None, p, p, 1 << 40,
                                          p, 1 << 40, None)
    assert rc == _abi.DCN_ERR_INVALID_ARGUMENT and "forward-only" in lib.dcn_last_error().decode()


@pytest.mark.parametrize("kw,expect", [
    (dict(), 1),                                                   # bf16, 64 -> 64, og 1
    (dict(dtype=0), 0),                                            # fp32: SIMT
    (dict(dtype=1), 1),                                            # fp16
    (dict(input_shape=(2, 96, 16, 16), weight_shape=(64, 96, 3, 3)), 0),   # C/G not a multiple of 64
    (dict(weight_shape=(48, 64, 3, 3)), 0),                        # C_out/G not a multiple of 32
    (dict(weight_shape=(512, 64, 3, 3)), 1),                       # C_out/G = 512: forward
    (dict(n_offset_grps=16), 0),                                   # 4 channels per offset group
    (dict(n_offset_grps=8), 1),                                    # 8 channels per offset group
    (dict(input_shape=(2, 128, 16, 16), weight_shape=(128, 64, 3, 3), n_weight_grps=2), 1),
])
def test_tensor_core_dispatch_rules(kw, expect):
    """The dispatch conditions of the tensor-core path (a host query)."""
    from mps_deform_conv import _abi
    lib = _abi.load()
    base = dict(dtype=_abi.DCN_BFLOAT16, input_shape=(2, 64, 16, 16), weight_shape=(64, 64, 3, 3), padding=(1, 1),
                use_mask=True)
    base.update(kw)
    d = _desc(**base)
    assert lib.dcn_uses_tensor_cores(ctypes.byref(d)) == expect


def test_torch_extension_imports():
    import mps_deform_conv
    lib = mps_deform_conv._get_lib()
    for f in ("deform_conv2d_forward", "deformable_im2col", "deform_conv2d_backward_input",
              "deform_conv2d_backward_offset_mask", "deform_conv2d_backward"):
        assert hasattr(lib, f)
    assert lib.abi_version() >= 100
