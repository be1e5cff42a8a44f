"""Fused DCNv2 offset/mask head: the operator reads ModulatedDeformConv2d's
offset convolution output [B, 3*og*kh*kw, Ho, Wo] in place (offsets, then
mask logits; sigmoid inside the kernels) and its backward returns the
gradient of that output.  Checked against the float64 oracle of the
reference's composition (slice, sigmoid, deform_conv2d) on the same 16-bit
inputs, and the module's fused route against its composed route.
Tolerance: normwise relative error <= 1e-2 (fp16/bf16)."""
import numpy as np
import pytest
import torch

from _util import TOL, assert_close, rel_err, to_np
from oracle import oracle

pytestmark = pytest.mark.gpu

DTYPES = {"float16": torch.float16, "bfloat16": torch.bfloat16}
# (B, C, H, W, Co, groups, og, k, stride, pad, dil)
SHAPES = {
    "c64_og1": (2, 64, 12, 10, 64, 1, 1, 3, 1, 1, 1),
    "c128_g2_og4_dil2": (2, 128, 10, 11, 128, 2, 4, 3, 1, 2, 2),
    "c128_og2_s2": (1, 128, 14, 13, 96, 1, 2, 3, 2, 1, 1),
}


def _inputs(spec, dtype, dev, seed):
    B, C, H, W, Co, G, og, k, s, p, d = spec
    g = torch.Generator().manual_seed(seed)
    Ho = (H + 2 * p - (d * (k - 1) + 1)) // s + 1
    Wo = (W + 2 * p - (d * (k - 1) + 1)) // s + 1
    T = k * k
    x = torch.randn(B, C, H, W, generator=g)
    w = torch.randn(Co, C // G, k, k, generator=g) / np.sqrt(C // G * T)
    b = torch.randn(Co, generator=g) * 0.1
    om = torch.cat([torch.randn(B, 2 * og * T, Ho, Wo, generator=g) * 2.0,   # offsets
                    torch.randn(B, og * T, Ho, Wo, generator=g) * 1.5], 1)    # mask logits
    go = torch.randn(B, Co, Ho, Wo, generator=g)
    cv = lambda t: t.to(dev, dtype)
    return dict(x=cv(x), w=cv(w), b=cv(b), om=cv(om), go=cv(go), geo=((s, s), (p, p), (d, d)), G=G, og=og, T=T)


@pytest.mark.parametrize("keep_saved", [True, False])
@pytest.mark.parametrize("dtype", list(DTYPES))
@pytest.mark.parametrize("name", list(SHAPES))
def test_head_forward_backward_vs_oracle(name, dtype, keep_saved, cuda):
    import mps_deform_conv as mdc
    lib = mdc._get_lib()
    I = _inputs(SHAPES[name], DTYPES[dtype], cuda, seed=31)
    (sh, sw), (ph, pw), (dh, dw) = I["geo"]
    assert lib.head_supported(I["x"], I["w"], sh, sw, ph, pw, dh, dw, I["G"], I["og"])
    out, saved = lib.deform_conv2d_forward_head(I["x"], I["w"], I["om"], I["b"], sh, sw, ph, pw, dh, dw, I["G"],
                                                I["og"], keep_saved)
    assert (saved.numel() > 0) == keep_saved
    gi, gw, gom, gb = lib.deform_conv2d_backward_head(I["go"], I["x"], I["w"], I["om"], I["b"], sh, sw, ph, pw,
                                                      dh, dw, I["G"], I["og"], [True] * 4,
                                                      saved if keep_saved else None)
    torch.cuda.synchronize()
    lib.device_status()
    # oracle: the reference's composition in float64 on the same 16-bit values
    n_off = 2 * I["og"] * I["T"]
    om64 = I["om"].double()
    off = om64[:, :n_off].contiguous()
    m = torch.sigmoid(om64[:, n_off:]).contiguous()
    st, pd, dl = I["geo"]
    ref = oracle.forward(I["x"], off, I["w"], I["b"], st, pd, dl, m)
    rgi, rgoff, rgw, rgb, rgm = oracle.backward(I["go"], I["x"], off, I["w"], st, pd, dl, m, True)
    m_np = to_np(m)
    rgom = np.concatenate([rgoff, rgm * m_np * (1.0 - m_np)], axis=1)
    tol = TOL[dtype]
    assert_close(out, ref, dtype, 'out')
    assert_close(gi, rgi, dtype, 'gi')
    assert_close(gw, rgw, dtype, 'gw')
    assert_close(gb, rgb, dtype, 'gb')
    assert_close(gom[:, :n_off], rgoff, dtype, 'gom[:, :n_off]')
    assert_close(gom[:, n_off:], rgom[:, n_off:], dtype, 'gom[:, n_off:]')


@pytest.mark.parametrize("name", ["c64_og1", "c128_g2_og4_dil2"])
def test_module_fused_head_matches_composed(name, cuda):
    """ModulatedDeformConv2d: the fused route and the reference's composition
    (slice + sigmoid + deform_conv2d) agree on the output and on every
    parameter and input gradient."""
    import mps_deform_conv as mdc
    B, C, H, W, Co, G, og, k, s, p, d = SHAPES[name]
    torch.manual_seed(5)
    mod = mdc.ModulatedDeformConv2d(C, Co, k, stride=s, padding=p, dilation=d, groups=G, offset_groups=og)
    with torch.no_grad():  # non-trivial offsets and masks
        mod.offset_conv.weight.normal_(0, 0.05)
        mod.offset_conv.bias.normal_(0, 0.5)
    mod = mod.to(cuda, torch.bfloat16)
    x0 = torch.randn(B, C, H, W, device=cuda, dtype=torch.bfloat16)
    res = {}
    for fused in (True, False):
        mdc.set_head_fusion(fused)
        try:
            mod.zero_grad(set_to_none=True)
            x = x0.clone().requires_grad_(True)
            out = mod(x)
            out.float().square().mean().backward()
        finally:
            mdc.set_head_fusion(True)
        res[fused] = [out.detach(), x.grad, mod.weight.grad, mod.bias.grad, mod.offset_conv.weight.grad,
                      mod.offset_conv.bias.grad]
    torch.cuda.synchronize()
    assert mod._fused_head(x0, mod.offset_conv(x0))
    for i, (a, b) in enumerate(zip(res[True], res[False])):
        assert rel_err(to_np(a), to_np(b)) <= 2e-2, i


def test_module_without_head_support_composes(cuda):
    """8 channels per offset group: no fused head; the module composes as the
    reference does and gives the same result with fusion on or off."""
    import mps_deform_conv as mdc
    torch.manual_seed(6)
    mod = mdc.ModulatedDeformConv2d(64, 64, 3, padding=1, offset_groups=8).to(cuda, torch.bfloat16)
    x = torch.randn(2, 64, 9, 11, device=cuda, dtype=torch.bfloat16)
    assert not mod._fused_head(x, mod.offset_conv(x))
    a = mod(x)
    mdc.set_head_fusion(False)
    try:
        b = mod(x)
    finally:
        mdc.set_head_fusion(True)
    torch.cuda.synchronize()
    assert torch.equal(a, b)
