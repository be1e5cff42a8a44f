"""Properties of the CPU oracle beyond the golden fixtures (float64, CPU).

* col2im is the adjoint of im2col in the input, and col2im_coord is the
  derivative of <im2col, G> in the offsets and the mask;
* the forward is W . im2col + bias, linear in the input and in the weight;
* the backward's gradients match central finite differences of
  L = <forward, grad_output> at sampling points away from grid lines (the
  reference's own tests check gradients by finite differences,
  tests/test_deform_conv.py:334-389).
"""
import numpy as np
import pytest

from oracle import oracle


def _problem(seed, B=2, C=6, H=7, W=8, Co=4, G=2, og=3, k=3, stride=1, pad=1, dil=1, frac=False):
    rng = np.random.default_rng(seed)
    Ho = (H + 2 * pad - (dil * (k - 1) + 1)) // stride + 1
    Wo = (W + 2 * pad - (dil * (k - 1) + 1)) // stride + 1
    x = rng.standard_normal((B, C, H, W))
    w = rng.standard_normal((Co, C // G, k, k)) / np.sqrt(C // G * k * k)
    if frac:  # integer part in [-1, 1], fractional part in [0.25, 0.75]: no grid line within 0.25
        off = rng.integers(-1, 2, (B, 2 * og * k * k, Ho, Wo)) + rng.uniform(0.25, 0.75, (B, 2 * og * k * k, Ho, Wo))
    else:
        off = rng.standard_normal((B, 2 * og * k * k, Ho, Wo)) * 1.5
    m = rng.uniform(0.1, 0.9, (B, og * k * k, Ho, Wo))
    b = rng.standard_normal(Co) * 0.1
    go = rng.standard_normal((B, Co, Ho, Wo))
    geo = dict(stride=(stride, stride), padding=(pad, pad), dilation=(dil, dil))
    return dict(x=x, w=w, off=off, m=m, b=b, go=go, geo=geo, k=k, og=og, G=G)


@pytest.mark.parametrize("seed", [0, 1])
def test_col2im_is_adjoint_of_im2col(seed):
    P = _problem(seed)
    k, geo = P["k"], P["geo"]
    cols = oracle.im2col(P["x"], P["off"], P["m"], k, k, offset_groups=P["og"], **geo)
    G = np.random.default_rng(seed + 100).standard_normal(cols.shape)
    gi = oracle.col2im(G, P["x"].shape, P["off"], P["m"], k, k, offset_groups=P["og"], **geo)
    lhs, rhs = float(np.sum(cols * G)), float(np.sum(P["x"] * gi))
    assert abs(lhs - rhs) <= 1e-12 * max(1.0, abs(lhs))


def test_forward_is_weight_times_columns_plus_bias():
    P = _problem(3, G=1)
    k, geo = P["k"], P["geo"]
    out = oracle.forward(P["x"], P["off"], P["w"], P["b"], mask=P["m"], **geo)
    cols = oracle.im2col(P["x"], P["off"], P["m"], k, k, offset_groups=P["og"], **geo)
    B, Co, Ho, Wo = out.shape
    ref = (P["w"].reshape(Co, -1) @ cols).reshape(Co, B, Ho, Wo).transpose(1, 0, 2, 3) + P["b"][None, :, None, None]
    np.testing.assert_allclose(out, ref, rtol=1e-12, atol=1e-12)


def test_forward_linear_in_input_and_weight():
    P = _problem(4)
    geo = P["geo"]
    f = lambda x, w: oracle.forward(x, P["off"], w, None, mask=P["m"], **geo)
    rng = np.random.default_rng(5)
    x2, w2 = rng.standard_normal(P["x"].shape), rng.standard_normal(P["w"].shape)
    np.testing.assert_allclose(f(2.0 * P["x"] - 3.0 * x2, P["w"]), 2.0 * f(P["x"], P["w"]) - 3.0 * f(x2, P["w"]),
                               rtol=1e-11, atol=1e-11)
    np.testing.assert_allclose(f(P["x"], 0.5 * P["w"] + w2), 0.5 * f(P["x"], P["w"]) + f(P["x"], w2),
                               rtol=1e-11, atol=1e-11)


@pytest.mark.parametrize("shape", [dict(), dict(stride=2, pad=1, dil=2, H=9, W=9), dict(G=1, og=1, C=4)])
def test_backward_matches_finite_differences(shape):
    P = _problem(7, frac=True, **shape)
    geo = P["geo"]

    def loss(x=None, off=None, w=None, m=None, b=None):
        out = oracle.forward(P["x"] if x is None else x, P["off"] if off is None else off,
                             P["w"] if w is None else w, P["b"] if b is None else b,
                             mask=P["m"] if m is None else m, **geo)
        return float(np.sum(out * P["go"]))

    gi, goff, gw, gb, gm = oracle.backward(P["go"], P["x"], P["off"], P["w"], mask=P["m"], with_bias=True, **geo)
    rng = np.random.default_rng(11)
    h = 1e-6
    for name, arr, grad in (("input", P["x"], gi), ("offset", P["off"], goff), ("weight", P["w"], gw),
                            ("mask", P["m"], gm), ("bias", P["b"], gb)):
        for _ in range(6):
            idx = tuple(int(rng.integers(0, s)) for s in arr.shape)
            plus, minus = arr.copy(), arr.copy()
            plus[idx] += h
            minus[idx] -= h
            key = {"input": "x", "offset": "off", "weight": "w", "mask": "m", "bias": "b"}[name]
            fd = (loss(**{key: plus}) - loss(**{key: minus})) / (2 * h)
            assert abs(fd - grad[idx]) <= 1e-6 * max(1.0, abs(fd)), (name, idx, fd, grad[idx])
