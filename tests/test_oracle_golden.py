"""The CPU oracle against the torchvision float64 golden fixtures (pins the oracle)."""
import numpy as np
import pytest

from _util import golden_cases, load_golden
from oracle import oracle

CASES = golden_cases()


def test_fixture_set_complete():
    assert len(CASES) >= 11


@pytest.mark.parametrize("name", CASES)
def test_oracle_forward_matches_torchvision(name):
    d = load_golden(name)
    out = oracle.forward(d["input"], d["offset"], d["weight"], d.get("bias"), tuple(d["stride"]),
                         tuple(d["padding"]), tuple(d["dilation"]), d.get("mask"))
    assert out.shape == d["output"].shape
    np.testing.assert_allclose(out, d["output"], rtol=1e-12, atol=1e-12)


@pytest.mark.parametrize("name", [c for c in CASES if c != "empty_batch"])
def test_oracle_backward_matches_torchvision(name):
    d = load_golden(name)
    gi, goff, gw, gb, gm = oracle.backward(
        d["grad_output"], d["input"], d["offset"], d["weight"], tuple(d["stride"]),
        tuple(d["padding"]), tuple(d["dilation"]), d.get("mask"), "bias" in d)
    np.testing.assert_allclose(gi, d["grad_input"], rtol=1e-12, atol=1e-12)
    np.testing.assert_allclose(goff, d["grad_offset"], rtol=1e-12, atol=1e-12)
    np.testing.assert_allclose(gw, d["grad_weight"], rtol=1e-11, atol=1e-12)
    if "bias" in d:
        np.testing.assert_allclose(gb, d["grad_bias"], rtol=1e-12, atol=1e-12)
    if "mask" in d:
        np.testing.assert_allclose(gm, d["grad_mask"], rtol=1e-12, atol=1e-12)


@pytest.mark.parametrize("name", [c for c in CASES if c != "empty_batch"])
def test_oracle_param_grads_match_torchvision(name):
    """The BLAS-product path for large shards (oracle.param_grads) gives the
    torchvision grad_weight / grad_bias of every fixture."""
    d = load_golden(name)
    gw, gb = oracle.param_grads(d["grad_output"], d["input"], d["offset"], d["weight"], tuple(d["stride"]),
                                tuple(d["padding"]), tuple(d["dilation"]), d.get("mask"))
    np.testing.assert_allclose(gw, d["grad_weight"], rtol=1e-11, atol=1e-12)
    if "bias" in d:
        np.testing.assert_allclose(gb, d["grad_bias"], rtol=1e-12, atol=1e-12)


@pytest.mark.parametrize("name", ["mask_bias_g2_og2", "stride2_dil2", "integer_offsets"])
def test_oracle_column_pieces_compose(name):
    """im2col / col2im / col2im_coord compose to the same gradients (groups=1 slice)."""
    d = load_golden(name)
    x, off, w, m = d["input"], d["offset"], d["weight"], d.get("mask")
    kh, kw = w.shape[2], w.shape[3]
    og = off.shape[1] // (2 * kh * kw)
    st, pd, dl = tuple(d["stride"]), tuple(d["padding"]), tuple(d["dilation"])
    cols = oracle.im2col(x, off, m, kh, kw, st, pd, dl, og)
    B, C = x.shape[:2]
    G = C // w.shape[1]
    Co = w.shape[0]
    go = d["grad_output"]
    P = cols.shape[1]
    go_flat = go.transpose(1, 0, 2, 3).reshape(Co, P)
    # per-group column gradient
    K = cols.shape[0] // G
    gcol = np.zeros_like(cols)
    for g in range(G):
        wg = w[g * (Co // G):(g + 1) * (Co // G)].reshape(Co // G, K)
        gcol[g * K:(g + 1) * K] = wg.T @ go_flat[g * (Co // G):(g + 1) * (Co // G)]
    gi = oracle.col2im(gcol, x.shape, off, m, kh, kw, st, pd, dl, og)
    goff, gm = oracle.col2im_coord(gcol, x, off, m, kh, kw, st, pd, dl, og)
    np.testing.assert_allclose(gi, d["grad_input"], rtol=1e-12, atol=1e-12)
    np.testing.assert_allclose(goff, d["grad_offset"], rtol=1e-12, atol=1e-12)
    if m is not None:
        np.testing.assert_allclose(gm, d["grad_mask"], rtol=1e-12, atol=1e-12)


def test_oracle_linearity_in_weight():
    """forward is linear in the weight: f(a*w1 + w2) = a*f(w1) + f(w2) (no bias)."""
    rng = np.random.default_rng(0)
    x = rng.standard_normal((2, 4, 7, 6))
    off = rng.standard_normal((2, 18, 7, 6)) * 2
    w1 = rng.standard_normal((3, 4, 3, 3))
    w2 = rng.standard_normal((3, 4, 3, 3))
    f = lambda w: oracle.forward(x, off, w, None, 1, 1, 1, None)
    np.testing.assert_allclose(f(2.5 * w1 + w2), 2.5 * f(w1) + f(w2), rtol=1e-12, atol=1e-12)


def test_oracle_planted_mistake_is_caught():
    """A wrong offset-channel order (dx/dy swapped) must not pass the fixture check."""
    d = load_golden("basic_v1")
    off = d["offset"].copy()
    off[:, 0::2], off[:, 1::2] = d["offset"][:, 1::2], d["offset"][:, 0::2]
    out = oracle.forward(d["input"], off, d["weight"], None, tuple(d["stride"]),
                         tuple(d["padding"]), tuple(d["dilation"]), None)
    assert np.abs(out - d["output"]).max() > 1e-3
