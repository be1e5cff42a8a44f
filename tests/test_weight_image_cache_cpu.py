"""Host logic of the forward weight-image cache (set_weight_image_cache): a
fake native layer stands in for the image builder, so nothing launches."""
import gc

import torch

import mps_deform_conv as mdc


class FakeLib:
    def __init__(self, supported=True):
        self.builds = 0
        self.supported = supported

    def weight_image(self, input, weight, *geo):
        self.builds += 1
        n = weight.numel() * weight.element_size() if self.supported else 0
        return torch.full((n,), self.builds, dtype=torch.uint8)


GEO = (1, 1, 1, 1, 1, 1, 1, 1, True)


def test_cache_hits_follow_identity_and_version():
    lib = FakeLib()
    x = torch.zeros(1, 64, 4, 4)
    w = torch.randn(64, 64, 3, 3)
    mdc.set_weight_image_cache(True)
    try:
        a = mdc._weight_image(lib, x, w, GEO)
        b = mdc._weight_image(lib, x, w, GEO)
        assert lib.builds == 1 and b is a
        w.mul_(2.0)  # in place: new version -> rebuilt
        c = mdc._weight_image(lib, x, w, GEO)
        assert lib.builds == 2 and c is not a
        w2 = w.clone()  # equal values, another tensor -> its own image
        mdc._weight_image(lib, x, w2, GEO)
        assert lib.builds == 3
        mdc._weight_image(lib, x, w, GEO[:-3] + (2,) + GEO[-2:])  # other group split -> rebuilt
        assert lib.builds == 4
        n = len(mdc._weight_images)
        del w2
        gc.collect()
        assert len(mdc._weight_images) == n - 1  # a freed weight's entry is dropped
    finally:
        mdc.set_weight_image_cache(False)


def test_cache_off_or_unsupported_builds_every_call():
    lib = FakeLib()
    x = torch.zeros(1, 64, 4, 4)
    w = torch.randn(64, 64, 3, 3)
    mdc.set_weight_image_cache(False)
    mdc._weight_image(lib, x, w, GEO)
    mdc._weight_image(lib, x, w, GEO)
    assert lib.builds == 2
    lib = FakeLib(supported=False)
    mdc.set_weight_image_cache(True)
    try:
        assert mdc._weight_image(lib, x, w, GEO).numel() == 0
        assert mdc._weight_image(lib, x, w, GEO).numel() == 0
        assert lib.builds == 2 and not mdc._weight_images  # nothing cached for the SIMT path
    finally:
        mdc.set_weight_image_cache(False)
