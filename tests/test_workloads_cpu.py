"""The benchmark problems on the CPU: shapes, algorithmic FLOPs and bytes, and
the seeded generator.

bench.py divides these FLOPs and bytes by measured times, so they are pinned
here to the published per-layer figures: F_fwd = 2*Co*(Cin/g)*kh*kw*B*Ho*Wo,
three times that for a training step, and the unique tensor bytes of the
step (forward reads x, offset, mask, weight and writes out; the backward
reads grad_out, x, offset, mask, weight and writes their gradients).
"""
import math

import pytest
import torch

from mps_deform_conv.workloads import PROBLEMS, make_inputs

# name: (out H, W, K reduction, GFLOP per step, MB per step), as published:
# to three significant figures, MB to one decimal (C4's and C5's to the unit)
PUBLISHED = {
    "c1_dcnv1_fp32": ((32, 32), 576, 0.0755, 0.7),
    "c2_dcnv2_fp32": ((64, 64), 1152, 7.25, 25.4),
    "c3a_backbone_bf16": ((50, 68), 2304, 32.1, 30.5),
    "c3b_backbone_s2_bf16": ((50, 50), 2304, 47.2, 64.9),
    "c4_video_fp16": ((180, 320), 576, 203.8, 1784.0),
    "c5_train_bf16": ((38, 38), 2304, 654.1, 540.0),
}


@pytest.mark.parametrize("name", list(PUBLISHED))
def test_flops_and_bytes_match_published_figures(name):
    p = PROBLEMS[name]
    hw, k_red, gflop, mb = PUBLISHED[name]
    assert p.out_hw == hw
    assert p.k_red == k_red
    assert math.isclose(p.flops() / 1e9, gflop, rel_tol=2e-3)
    assert abs(p.min_hbm_bytes() / 1e6 - mb) <= (0.5 if mb >= 100 else 0.05)


def test_flops_and_bytes_scale_with_batch():
    for p in PROBLEMS.values():
        assert math.isclose(p.flops(batch=3 * p.batch), 3 * p.flops())
        es = torch.tensor([], dtype=p.dtype).element_size()
        # batch-independent: weight and bias (read once in each pass, their gradients written)
        fixed = es * (p.out_channels * p.k_red * (3 if p.training else 1)
                      + (p.out_channels * (2 if p.training else 1) if p.use_bias else 0))
        per = p.min_hbm_bytes(batch=2) - p.min_hbm_bytes(batch=1)
        assert per > 0 and math.isclose(p.min_hbm_bytes(batch=1), fixed + per, rel_tol=1e-12)
        assert math.isclose(p.min_hbm_bytes(batch=5) - p.min_hbm_bytes(batch=2), 3 * per, rel_tol=1e-12)


@pytest.mark.parametrize("name", ["c1_dcnv1_fp32", "c2_dcnv2_fp32"])
def test_make_inputs_shapes_and_dtypes(name):
    p = PROBLEMS[name]
    d = make_inputs(p)
    t, (ho, wo) = p.kernel ** 2, p.out_hw
    assert d["input"].shape == (p.batch, p.in_channels, p.height, p.width)
    assert d["offset"].shape == (p.batch, 2 * p.offset_groups * t, ho, wo)
    assert d["weight"].shape == (p.out_channels, p.in_channels // p.groups, p.kernel, p.kernel)
    assert d["grad_output"].shape == (p.batch, p.out_channels, ho, wo)
    assert (d["mask"] is not None) == p.use_mask and (d["bias"] is not None) == p.use_bias
    if p.use_mask:
        assert d["mask"].shape == (p.batch, p.offset_groups * t, ho, wo)
        assert float(d["mask"].min()) > 0 and float(d["mask"].max()) < 1
    for v in d.values():
        assert v is None or v.dtype == p.dtype


def test_make_inputs_is_seeded_and_shards_are_slices():
    p = PROBLEMS["c2_dcnv2_fp32"]
    full = make_inputs(p, batch=4)
    again = make_inputs(p, batch=4)
    for k, v in full.items():
        assert torch.equal(v, again[k]), k
    assert not torch.equal(make_inputs(p, batch=4, seed=1)["input"], full["input"])
    for first, nb in ((0, 1), (1, 2), (3, 1)):
        part = make_inputs(p, batch=nb, batch_offset=first)
        for k in ("input", "offset", "mask", "grad_output"):
            assert torch.equal(part[k], full[k][first:first + nb]), (k, first)
        for k in ("weight", "bias"):
            assert torch.equal(part[k], full[k]), k


def test_make_inputs_offset_distributions():
    """C4's offsets are uniform in +-10 px; the others normal with the listed std."""
    p4 = PROBLEMS["c4_video_fp16"]
    small = dict(batch=1)
    off = make_inputs(p4, **small)["offset"].float()
    assert float(off.abs().max()) <= 10.0 and float(off.abs().max()) > 9.9
    assert abs(float(off.std()) - 10 / math.sqrt(3)) < 0.05
    p2 = PROBLEMS["c2_dcnv2_fp32"]
    off2 = make_inputs(p2, batch=2)["offset"]
    assert abs(float(off2.std()) - 2.0) < 0.05
    d0 = make_inputs(PROBLEMS["c1_dcnv1_fp32"])
    assert abs(float(d0["weight"].std()) - 1 / 24) < 0.004


def test_empty_batch():
    p = PROBLEMS["c2_dcnv2_fp32"]
    d = make_inputs(p, batch=0)
    assert d["input"].shape[0] == 0 and d["offset"].shape[0] == 0 and d["grad_output"].shape[0] == 0
    assert p.flops(batch=0) == 0
