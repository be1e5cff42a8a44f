"""Parity of the tensor-core (tcgen05) path: shapes whose channel counts the
tcgen05 kernels take (per-group input channels a multiple of 64), fp16 and
bf16, against the float64 oracle on the same rounded inputs.  Tolerance:
normwise relative error <= 1e-2 (tests/_util.rel_err)."""
import numpy as np
import pytest
import torch

from _util import TOL, assert_close, rel_err, to_np
from oracle import oracle

pytestmark = pytest.mark.gpu

DTYPES = {"float16": torch.float16, "bfloat16": torch.bfloat16}

# (B, C, H, W, Co, groups, og, k, stride, pad, dil, mask, bias, offset_scale)
SHAPES = {
    "c64_og1": (2, 64, 12, 10, 64, 1, 1, 3, 1, 1, 1, True, True, 2.0),
    "c64_og8_far": (2, 64, 9, 11, 64, 1, 8, 3, 1, 1, 1, True, False, 10.0),
    "c128_g2_og4_dil2": (2, 128, 10, 10, 128, 2, 4, 3, 1, 2, 2, True, True, 3.0),
    "c128_co256_s2": (1, 128, 14, 13, 256, 1, 1, 3, 2, 1, 1, True, False, 1.5),
    "c64_co512_nomask": (1, 64, 8, 9, 512, 1, 1, 3, 1, 1, 1, False, True, 1.0),
    "c192_co96_tail": (3, 192, 7, 9, 96, 1, 2, 3, 1, 1, 1, True, True, 2.0),
    "c64_og8_near_int": (2, 64, 10, 12, 64, 1, 8, 3, 1, 1, 1, True, True, "near_int"),
}


def _make(spec, dtype, dev, seed=0):
    B, C, H, W, Co, G, og, k, s, p, d, use_mask, use_bias, osc = spec
    g = torch.Generator().manual_seed(seed)
    Ho = (H + 2 * p - (d * (k - 1) + 1)) // s + 1
    Wo = (W + 2 * p - (d * (k - 1) + 1)) // s + 1
    x = torch.randn(B, C, H, W, generator=g)
    w = torch.randn(Co, C // G, k, k, generator=g) / np.sqrt(C // G * k * k)
    if osc == "near_int":  # within +-2e-6 of integers: exact-floor corner choice
        off = torch.randint(-3, 4, (B, 2 * og * k * k, Ho, Wo), generator=g).float()
        off += (torch.rand(B, 2 * og * k * k, Ho, Wo, generator=g) * 2 - 1) * 2e-6
    else:
        off = torch.randn(B, 2 * og * k * k, Ho, Wo, generator=g) * osc
    m = torch.sigmoid(torch.randn(B, og * k * k, Ho, Wo, generator=g)) if use_mask else None
    b = torch.randn(Co, generator=g) * 0.1 if use_bias else None
    go = torch.randn(B, Co, Ho, Wo, generator=g)
    cv = lambda t: None if t is None else t.to(dev, dtype)
    return dict(input=cv(x), weight=cv(w), offset=cv(off), mask=cv(m), bias=cv(b), grad_output=cv(go),
                stride=(s, s), padding=(p, p), dilation=(d, d))


@pytest.mark.parametrize("dtype", list(DTYPES))
@pytest.mark.parametrize("name", list(SHAPES))
def test_tc_forward_vs_oracle(name, dtype, cuda):
    import mps_deform_conv as mdc
    from mps_deform_conv import _abi
    T = _make(SHAPES[name], DTYPES[dtype], cuda)
    st, pd, dl = T["stride"], T["padding"], T["dilation"]
    lib = mdc._get_lib()
    G = T["input"].shape[1] // T["weight"].shape[1]
    og = T["offset"].shape[1] // 18
    assert lib.uses_tensor_cores(T["input"], T["weight"], st[0], st[1], pd[0], pd[1], dl[0], dl[1],
                                 G, og, T["mask"] is not None)
    out = _abi.call_forward(T["input"], T["offset"], T["weight"], T["bias"], st, pd, dl, T["mask"])
    torch.cuda.synchronize()
    lib.device_status()
    ref = oracle.forward(T["input"], T["offset"], T["weight"], T["bias"], st, pd, dl, T["mask"])
    assert_close(out, ref, dtype, 'out')
    # and through the public autograd API
    out2 = mdc.deform_conv2d(T["input"], T["offset"], T["weight"], T["bias"], st, pd, dl, T["mask"])
    assert_close(out2, ref, dtype, 'out2')


@pytest.mark.parametrize("dtype", list(DTYPES))
@pytest.mark.parametrize("name", list(SHAPES))
def test_tc_backward_vs_oracle(name, dtype, cuda):
    from mps_deform_conv import _abi
    T = _make(SHAPES[name], DTYPES[dtype], cuda, seed=1)
    st, pd, dl = T["stride"], T["padding"], T["dilation"]
    gi, goff, gw, gb, gm = _abi.call_backward(T["grad_output"], T["input"], T["offset"], T["weight"],
                                              st, pd, dl, T["mask"], with_bias=T["bias"] is not None)
    torch.cuda.synchronize()
    rgi, rgoff, rgw, rgb, rgm = oracle.backward(T["grad_output"], T["input"], T["offset"], T["weight"],
                                                st, pd, dl, T["mask"], T["bias"] is not None)
    tol = TOL[dtype]
    assert_close(gi, rgi, dtype, 'gi')
    assert_close(goff, rgoff, dtype, 'goff')
    assert_close(gw, rgw, dtype, 'gw')
    if T["bias"] is not None:
        assert_close(gb, rgb, dtype, 'gb')
    if T["mask"] is not None:
        assert_close(gm, rgm, dtype, 'gm')


def test_tc_forward_deterministic_and_batch_consistent(cuda):
    """Forward has no atomics: repeated runs are bitwise equal, and a batch
    slice gives the same rows as the full batch."""
    from mps_deform_conv import _abi
    T = _make(SHAPES["c128_g2_og4_dil2"], torch.bfloat16, cuda, seed=3)
    st, pd, dl = T["stride"], T["padding"], T["dilation"]
    a = _abi.call_forward(T["input"], T["offset"], T["weight"], T["bias"], st, pd, dl, T["mask"])
    b = _abi.call_forward(T["input"], T["offset"], T["weight"], T["bias"], st, pd, dl, T["mask"])
    c = _abi.call_forward(T["input"][1:].contiguous(), T["offset"][1:].contiguous(), T["weight"],
                          T["bias"], st, pd, dl, T["mask"][1:].contiguous())
    torch.cuda.synchronize()
    assert torch.equal(a, b)
    assert torch.equal(a[1:], c)


def _at_2_byte_offset(t):
    """The same values at a data pointer 2 bytes past a 4-byte boundary."""
    buf = torch.empty(t.numel() + 1, dtype=t.dtype, device=t.device)
    v = buf[1:].view(t.shape)
    v.copy_(t)
    assert v.data_ptr() % 4 == 2
    return v


@pytest.mark.parametrize("dtype", list(DTYPES))
def test_tc_layout_passes_unaligned_pointers(dtype, cuda):
    """The vectorized NCHW <-> channels-last passes need 4/16-byte aligned
    tensors; input and grad_output at a 2-byte offset take the scalar passes
    and give the same results (forward bitwise; gradients, accumulated with
    atomics in any order, within 1e-3)."""
    from mps_deform_conv import _abi
    T = _make(SHAPES["c128_g2_og4_dil2"], DTYPES[dtype], cuda, seed=21)  # 10x10 planes: vectorized when aligned
    st, pd, dl = T["stride"], T["padding"], T["dilation"]
    x_u, go_u = _at_2_byte_offset(T["input"]), _at_2_byte_offset(T["grad_output"])
    a = _abi.call_forward(T["input"], T["offset"], T["weight"], T["bias"], st, pd, dl, T["mask"])
    u = _abi.call_forward(x_u, T["offset"], T["weight"], T["bias"], st, pd, dl, T["mask"])
    ga = _abi.call_backward(T["grad_output"], T["input"], T["offset"], T["weight"], st, pd, dl, T["mask"],
                            with_bias=True)
    gu = _abi.call_backward(go_u, x_u, T["offset"], T["weight"], st, pd, dl, T["mask"], with_bias=True)
    torch.cuda.synchronize()
    assert torch.equal(a, u)
    for name, p, q in zip(("input", "offset", "weight", "bias", "mask"), ga, gu):
        assert rel_err(to_np(q), to_np(p)) <= 1e-3, name
    ref = oracle.forward(T["input"], T["offset"], T["weight"], T["bias"], st, pd, dl, T["mask"])
    assert_close(u, ref, dtype, 'u')


@pytest.mark.parametrize("name", ["c128_g2_og4_dil2", "c64_og8_near_int"])
@pytest.mark.parametrize("mask_sel", [(1, 0, 0, 0, 0), (0, 1, 0, 0, 1), (0, 0, 1, 1, 0), (0, 0, 1, 0, 0),
                                      (0, 0, 0, 1, 0)])
def test_tc_backward_output_subsets(mask_sel, name, cuda):
    """Only the requested gradients are computed and they match the full call
    (c64_og8_near_int takes the corner-quad epilogue, which writes the offset and
    mask gradients directly; c128_g2_og4_dil2 the 32-channel one)."""
    import mps_deform_conv as mdc
    lib = mdc._get_lib()
    spec = SHAPES[name]
    T = _make(spec, torch.bfloat16, cuda, seed=5)
    st, pd, dl = T["stride"], T["padding"], T["dilation"]
    args = (T["grad_output"], T["input"], T["weight"], T["offset"], T["mask"], T["bias"],
            st[0], st[1], pd[0], pd[1], dl[0], dl[1], spec[5], spec[6], True)
    full = lib.deform_conv2d_backward(*args, [True] * 5)
    part = lib.deform_conv2d_backward(*args, [bool(v) for v in mask_sel])
    torch.cuda.synchronize()
    for f, pz, sel in zip(full, part, mask_sel):
        if sel:
            assert rel_err(to_np(pz), to_np(f)) <= 1e-2
        else:
            assert pz is None


@pytest.mark.parametrize("cache", [True, False])
@pytest.mark.parametrize("name", ["c64_og8_far", "c128_g2_og4_dil2", "c192_co96_tail"])
def test_tc_autograd_training_cache(name, cache, cuda):
    """Autograd training step with the forward's saved state (column tiles +
    channels-last input) kept for the backward, and without it."""
    import mps_deform_conv as mdc
    T = _make(SHAPES[name], torch.bfloat16, cuda, seed=11)
    st, pd, dl = T["stride"], T["padding"], T["dilation"]
    leaves = {k: T[k].clone().requires_grad_(True) for k in ("input", "offset", "weight", "bias", "mask")
              if T[k] is not None}
    mdc.set_training_cache(cache)
    try:
        out = mdc.deform_conv2d(leaves["input"], leaves["offset"], leaves["weight"], leaves.get("bias"),
                                st, pd, dl, leaves.get("mask"))
        out.backward(T["grad_output"])
    finally:
        mdc.set_training_cache(True)
    torch.cuda.synchronize()
    ref_out = oracle.forward(T["input"], T["offset"], T["weight"], T["bias"], st, pd, dl, T["mask"])
    rgi, rgoff, rgw, rgb, rgm = oracle.backward(T["grad_output"], T["input"], T["offset"], T["weight"],
                                                st, pd, dl, T["mask"], T["bias"] is not None)
    tol = TOL["bfloat16"]
    assert_close(out, ref_out, "bfloat16", 'out')
    assert_close(leaves["input"].grad, rgi, "bfloat16", 'leaves["input"].grad')
    assert_close(leaves["offset"].grad, rgoff, "bfloat16", 'leaves["offset"].grad')
    assert_close(leaves["weight"].grad, rgw, "bfloat16", 'leaves["weight"].grad')
    if "bias" in leaves:
        assert_close(leaves["bias"].grad, rgb, "bfloat16", 'leaves["bias"].grad')
    if "mask" in leaves:
        assert_close(leaves["mask"].grad, rgm, "bfloat16", 'leaves["mask"].grad')


@pytest.mark.parametrize("cache", [True, False])
def test_tc_weight_grad_deterministic(cache, cuda):
    """grad_weight: each split of the pixel range stores its partial sum and
    the splits are added in a fixed order, so repeated backward passes are
    bitwise equal, with the saved column tiles and with the gathering wgrad."""
    import mps_deform_conv as mdc
    lib = mdc._get_lib()
    T = _make(SHAPES["c128_g2_og4_dil2"], torch.bfloat16, cuda, seed=17)
    T["input"] = T["input"].repeat(16, 1, 1, 1)  # 32 x 100 pixels: several pixel splits
    T["offset"] = T["offset"].repeat(16, 1, 1, 1)
    T["mask"] = T["mask"].repeat(16, 1, 1, 1)
    T["grad_output"] = T["grad_output"].repeat(16, 1, 1, 1)
    st, pd, dl = T["stride"], T["padding"], T["dilation"]
    args = (T["input"], T["weight"], T["offset"], T["mask"], T["bias"], st[0], st[1], pd[0], pd[1], dl[0], dl[1],
            2, 4, True)
    saved = lib.deform_conv2d_forward_train(*args)[1] if cache else None
    sel = [False, True, False, False, False]
    gw = [lib.deform_conv2d_backward(T["grad_output"], *args, sel, saved)[1] for _ in range(3)]
    torch.cuda.synchronize()
    lib.device_status()
    assert torch.equal(gw[0], gw[1]) and torch.equal(gw[0], gw[2])
    _, _, rgw, _, _ = oracle.backward(T["grad_output"][:2], T["input"][:2], T["offset"][:2], T["weight"], st, pd,
                                      dl, T["mask"][:2], False)
    assert torch.isfinite(gw[0]).all()
    assert_close(to_np(gw[0]) / 16.0, rgw, "bfloat16", "grad_weight / 16")


def test_abi_training_pair_matches_plain_calls(cuda):
    """dcn_deform_conv2d_forward_train / _backward_train through ctypes give the
    same results as the plain forward / backward."""
    import ctypes
    from mps_deform_conv import _abi
    lib = _abi.load()
    T = _make(SHAPES["c128_g2_og4_dil2"], torch.float16, cuda, seed=13)
    st, pd, dl = T["stride"], T["padding"], T["dilation"]
    d = _abi.desc_for(T["input"], T["weight"], T["offset"], st, pd, dl, T["mask"])
    nbytes = lib.dcn_saved_state_bytes(ctypes.byref(d))
    assert nbytes > 0
    saved = torch.empty(nbytes, dtype=torch.uint8, device=cuda)
    oh, ow = _abi.output_size(d)
    out = torch.empty((d.batch, d.out_channels, oh, ow), device=cuda, dtype=torch.float16)
    wsz = lib.dcn_forward_workspace_size(ctypes.byref(d))
    ws = torch.empty(max(wsz, 1), dtype=torch.uint8, device=cuda)
    stream = torch.cuda.current_stream(cuda).cuda_stream
    p = lambda t: None if t is None else t.data_ptr()
    _abi.check(lib.dcn_deform_conv2d_forward_train(ctypes.byref(d), p(T["input"]), p(T["weight"]),
                                                   p(T["offset"]), p(T["mask"]), p(T["bias"]), p(out),
                                                   p(saved), nbytes, p(ws), wsz, stream))
    grads = [torch.empty_like(T[k]) for k in ("input", "weight", "offset", "mask")] + \
        [torch.empty_like(T["bias"])]
    bsz = lib.dcn_backward_workspace_size(ctypes.byref(d))
    bws = torch.empty(max(bsz, 1), dtype=torch.uint8, device=cuda)
    _abi.check(lib.dcn_deform_conv2d_backward_train(ctypes.byref(d), p(T["grad_output"]), p(T["input"]),
                                                    p(T["weight"]), p(T["offset"]), p(T["mask"]), p(saved),
                                                    nbytes, *[p(g) for g in grads], p(bws), bsz, stream))
    ref_out = _abi.call_forward(T["input"], T["offset"], T["weight"], T["bias"], st, pd, dl, T["mask"])
    gi, goff, gw, gb, gm = _abi.call_backward(T["grad_output"], T["input"], T["offset"], T["weight"],
                                              st, pd, dl, T["mask"], with_bias=True)
    torch.cuda.synchronize()
    assert torch.equal(out, ref_out)
    for a_, b_ in zip(grads, (gi, gw, goff, gm, gb)):
        assert rel_err(to_np(a_), to_np(b_)) <= 1e-2
