"""Host-side API behaviour that needs no GPU: validation messages (the reference's
validation tests, tests/test_deform_conv.py:18-138), module construction,
parameter names and the CUDA-only device rule."""
import pytest
import torch

import mps_deform_conv as mdc


def test_public_surface():
    for n in ("deform_conv2d", "DeformConv2d", "ModulatedDeformConv2d", "is_available", "__version__"):
        assert hasattr(mdc, n)
    assert mdc.__version__ == "0.2.2"


def test_cpu_input_rejected():
    x = torch.randn(1, 4, 8, 8)
    w = torch.randn(4, 4, 3, 3)
    off = torch.randn(1, 18, 6, 6)
    with pytest.raises(ValueError, match="Input must be on CUDA device"):
        mdc.deform_conv2d(x, off, w)


@pytest.mark.parametrize("kw,msg", [
    (dict(stride=(0, 1)), "stride must be positive"),
    (dict(dilation=(0, 1)), "dilation must be positive"),
    (dict(padding=(-1, 0)), "padding must be non-negative"),
])
def test_validate_conv_params(kw, msg):
    args = dict(stride=(1, 1), padding=(0, 0), dilation=(1, 1))
    args.update(kw)
    with pytest.raises(ValueError, match=msg):
        mdc._validate_conv_params(args["stride"], args["padding"], args["dilation"], 3, 3)


def test_validate_groups():
    assert mdc._validate_groups(512, 512, 72, 3, 3, 256) == (2, 4)
    with pytest.raises(ValueError, match="divisible"):
        mdc._validate_groups(4, 4, 18, 3, 3, 3)
    with pytest.raises(ValueError, match="divisible"):
        mdc._validate_groups(4, 4, 17, 3, 3, 4)
    with pytest.raises(ValueError, match="divisible"):
        mdc._validate_groups(6, 6, 72, 3, 3, 6)  # 4 offset groups do not divide 6 channels


def test_check_overflow():
    with pytest.raises(ValueError, match="Tensor size overflow"):
        mdc._check_overflow([512, 3, 3, 4096, 512, 512], ["channels", "kernel_h", "kernel_w", "batch", "out_h", "out_w"])


def test_modules_and_state_dict_names():
    m = mdc.DeformConv2d(8, 16, 3, padding=1, groups=2, offset_groups=2)
    assert tuple(m.weight.shape) == (16, 4, 3, 3)
    assert set(m.state_dict()) == {"weight", "bias"}
    mm = mdc.ModulatedDeformConv2d(8, 16, 3, padding=1, offset_groups=2)
    assert set(mm.state_dict()) == {"weight", "bias", "offset_conv.weight", "offset_conv.bias"}
    assert mm.offset_conv.out_channels == 3 * 9 * 2
    assert torch.count_nonzero(mm.offset_conv.weight) == 0


def test_torchvision_registration_keeps_cpu_kernels():
    """Registering the CUDA implementations leaves torchvision's CPU path intact."""
    import numpy as np
    from torchvision.ops import deform_conv2d as tv
    from mps_deform_conv.torchvision_ops import register_torchvision_ops, registered
    from oracle import oracle
    register_torchvision_ops()
    register_torchvision_ops()  # idempotent
    assert registered()
    g = torch.Generator().manual_seed(3)
    x = torch.randn(1, 4, 6, 6, generator=g, dtype=torch.float64)
    w = torch.randn(3, 4, 3, 3, generator=g, dtype=torch.float64)
    off = torch.randn(1, 18, 6, 6, generator=g, dtype=torch.float64)
    out = tv(x, off, w, padding=(1, 1))
    np.testing.assert_allclose(out.numpy(), oracle.forward(x, off, w, None, 1, 1, 1, None), rtol=1e-12, atol=1e-12)
