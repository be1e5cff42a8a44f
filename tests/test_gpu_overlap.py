"""Parameter-gradient hook of the backward (set_param_grad_hook, C ABI
dcn_deform_conv2d_backward_overlap): called exactly once per backward with
grad_weight / grad_bias, after their kernels are enqueued; work it starts on a
side stream is ordered after them and is visible once the caller joins the
side stream.  The data-parallel all-reduce built on it
(sharding.OverlappedParamAllReduce) is checked on 2 GPUs when present."""
import os
import subprocess
import sys

import pytest
import torch

from _util import TOL, rel_err, to_np
from test_gpu_tc import SHAPES, _make

pytestmark = pytest.mark.gpu

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _grads(T, leaves_keys=("input", "offset", "weight", "bias", "mask")):
    import mps_deform_conv as mdc
    st, pd, dl = T["stride"], T["padding"], T["dilation"]
    leaves = [T[k].detach().clone().requires_grad_(True) for k in leaves_keys if T[k] is not None]
    d = dict(zip([k for k in leaves_keys if T[k] is not None], leaves))
    out = mdc.deform_conv2d(d["input"], d["offset"], d["weight"], d.get("bias"), st, pd, dl, d.get("mask"))
    return dict(zip(d.keys(), torch.autograd.grad(out, leaves, T["grad_output"])))


@pytest.mark.parametrize("dtype,shape", [(torch.bfloat16, "c128_g2_og4_dil2"), (torch.float32, "c64_og1")])
def test_hook_side_stream_work_is_ordered_and_joined(dtype, shape, cuda):
    """The hook starts a slow side-stream op (about a millisecond of spinning,
    then grad_weight *= 2, grad_bias *= 2) while the backward continues on the
    main stream; after joining, the gradients carry the side-stream update and
    the other gradients are those of a plain backward."""
    import mps_deform_conv as mdc
    T = _make(SHAPES[shape], dtype, cuda, seed=23)
    ref = _grads(T)
    side = torch.cuda.Stream()
    calls = []

    def hook(gw, gb):
        calls.append((gw is not None, gb is not None))
        side.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(side):
            torch.cuda._sleep(2_000_000)
            gw.mul_(2)
            if gb is not None:
                gb.mul_(2)

    mdc.set_param_grad_hook(hook)
    try:
        got = _grads(T)
    finally:
        mdc.set_param_grad_hook(None)
    torch.cuda.current_stream().wait_stream(side)
    torch.cuda.synchronize()
    mdc._get_lib().device_status()
    assert calls == [(True, T["bias"] is not None)]
    # grad_weight is deterministic on the tensor-core path (and fp32 on the
    # other); the other gradients accumulate with fp32 atomics in
    # run-dependent order (last-bit flips after rounding to 16 bits), so they
    # are held to the dtype tolerance
    assert rel_err(to_np(got["weight"]), 2 * to_np(ref["weight"])) <= 1e-6
    tol = TOL["float32" if dtype == torch.float32 else "bfloat16"]
    if T["bias"] is not None:
        assert rel_err(to_np(got["bias"]), 2 * to_np(ref["bias"])) <= tol
    for k in ("input", "offset", "mask"):
        if k in ref:
            assert rel_err(to_np(got[k]), to_np(ref[k])) <= tol, k


def test_hook_exception_propagates_and_library_stays_usable(cuda):
    import mps_deform_conv as mdc
    T = _make(SHAPES["c64_og1"], torch.bfloat16, cuda, seed=29)

    def hook(gw, gb):
        raise RuntimeError("hook failed on purpose")

    mdc.set_param_grad_hook(hook)
    try:
        with pytest.raises(RuntimeError, match="hook failed on purpose"):
            _grads(T)
    finally:
        mdc.set_param_grad_hook(None)
    torch.cuda.synchronize()
    g = _grads(T)
    torch.cuda.synchronize()
    assert torch.isfinite(g["weight"]).all()


def test_hook_rejects_non_callable():
    import mps_deform_conv as mdc
    with pytest.raises(TypeError):
        mdc.set_param_grad_hook(3)


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_overlapped_allreduce_two_gpus_matches_full_batch():
    """2 ranks over NCCL, each with half the batch: the overlapped all-reduce
    gives the full-batch grad_weight / grad_bias, equal to the serial one."""
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node=2",
           "--master-addr", "127.0.0.1", "--master-port", "29631",
           os.path.join(REPO, "tests", "_overlap_worker.py")]
    r = subprocess.run(["timeout", "-k", "30", "300"] + cmd, env=env, capture_output=True, text=True, cwd=REPO)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
    assert "OVERLAP OK" in r.stdout
