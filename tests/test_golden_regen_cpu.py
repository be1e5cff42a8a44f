"""The committed golden fixtures are what tests/golden/make_golden.py produces
from torchvision.ops.deform_conv2d (CPU, float64) today: every case is
regenerated and compared array by array."""
import importlib.util
import os

import numpy as np
import pytest

HERE = os.path.dirname(os.path.abspath(__file__))
GOLDEN = os.path.join(HERE, "golden")

torchvision = pytest.importorskip("torchvision")


def _make_golden():
    spec = importlib.util.spec_from_file_location("make_golden", os.path.join(GOLDEN, "make_golden.py"))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


MG = _make_golden()


@pytest.mark.parametrize("name", sorted(MG.CASES))
def test_fixture_regenerates(name):
    fresh = MG.case_arrays(MG.CASES[name], MG.seeds()[name])
    with np.load(os.path.join(GOLDEN, f"{name}.npz")) as z:
        assert sorted(z.files) == sorted(fresh)
        for k in z.files:
            np.testing.assert_allclose(fresh[k], z[k], rtol=1e-12, atol=1e-12, err_msg=k)
