"""The reference's validation tests that need a device tensor
(tests/test_deform_conv.py:99-138): a tensor on another device than the input,
and an output size that is not positive, raise ValueError before any kernel
runs."""
import pytest
import torch

pytestmark = pytest.mark.gpu


def test_device_mismatch(cuda):
    import mps_deform_conv as mdc
    x = torch.randn(1, 4, 8, 8, device=cuda)
    w = torch.randn(4, 4, 3, 3)  # on the host
    off = torch.randn(1, 18, 6, 6, device=cuda) * 0.1
    with pytest.raises(ValueError, match="device"):
        mdc.deform_conv2d(x, off, w)


def test_invalid_output_dimensions(cuda):
    import mps_deform_conv as mdc
    x = torch.randn(1, 4, 4, 4, device=cuda)
    w = torch.randn(4, 4, 5, 5, device=cuda)
    off = torch.randn(1, 50, 1, 1, device=cuda) * 0.1
    with pytest.raises(ValueError, match="Invalid output dimensions"):
        mdc.deform_conv2d(x, off, w, stride=(2, 2))
