"""Batch-sharded training logic on CPU: two gloo ranks each take half of a
global batch, compute parameter gradients with the CPU reference
(torchvision.ops.deform_conv2d, the parity ground truth) and all-reduce them
with mps_deform_conv.sharding; the result must equal the full-batch gradients.
Also checks that a rank which raises makes its peer's collective fail within
the process-group timeout instead of hanging."""
import datetime
import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

from mps_deform_conv.sharding import OverlappedParamAllReduce, allreduce_param_grads, shard_range


def test_shard_range_partitions():
    for gb in (0, 1, 7, 8, 64):
        for ws in (1, 2, 3, 4, 8):
            spans = [shard_range(gb, ws, r) for r in range(ws)]
            assert sum(c for _, c in spans) == gb
            pos = 0
            for s, c in spans:
                assert s == pos
                pos += c
            assert max(c for _, c in spans) - min(c for _, c in spans) <= 1
    with pytest.raises(ValueError):
        shard_range(8, 2, 2)


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _problem():
    g = torch.Generator().manual_seed(7)
    B, C, H, W, Co = 4, 8, 7, 6, 6
    x = torch.randn(B, C, H, W, generator=g, dtype=torch.float64)
    w = torch.randn(Co, C // 2, 3, 3, generator=g, dtype=torch.float64)
    b = torch.randn(Co, generator=g, dtype=torch.float64)
    off = torch.randn(B, 2 * 2 * 9, H, W, generator=g, dtype=torch.float64) * 2
    m = torch.sigmoid(torch.randn(B, 2 * 9, H, W, generator=g, dtype=torch.float64))
    go = torch.randn(B, Co, H, W, generator=g, dtype=torch.float64)
    return x, w, b, off, m, go


def _param_grads(x, w, b, off, m, go):
    from torchvision.ops import deform_conv2d
    w = w.clone().requires_grad_(True)
    b = b.clone().requires_grad_(True)
    out = deform_conv2d(x, off, w, b, padding=(1, 1), mask=m)
    out.backward(go)
    return w.grad, b.grad


def _worker(rank, world, port, q, mode="serial"):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    import torch.distributed as dist
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=30))
    try:
        x, w, b, off, m, go = _problem()
        s, c = shard_range(x.shape[0], world, rank)
        gw, gb = _param_grads(x[s:s + c], w, b, off[s:s + c], m[s:s + c], go[s:s + c])
        if mode == "hook":  # the backward's parameter-gradient hook, CPU tensors
            hook = OverlappedParamAllReduce()
            hook(gw, gb)
            hook.wait()
            assert hook.calls == 1
        else:
            allreduce_param_grads([gw, None, gb])
        q.put((rank, gw.numpy().copy(), gb.numpy().copy()))  # by value: the sender exits
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("mode", ["serial", "hook"])
def test_two_rank_gloo_allreduce_matches_full_batch(mode):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q, mode)) for r in range(2)]
    for p in procs:
        p.start()
    res = [q.get(timeout=120) for _ in range(2)]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    x, w, b, off, m, go = _problem()
    gw_full, gb_full = _param_grads(x, w, b, off, m, go)
    for _, gw, gb in res:
        torch.testing.assert_close(torch.from_numpy(gw), gw_full, rtol=1e-10, atol=1e-10)
        torch.testing.assert_close(torch.from_numpy(gb), gb_full, rtol=1e-10, atol=1e-10)


def _failing_worker(rank, world, port, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    import torch.distributed as dist
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=5))
    if rank == 1:
        q.put((rank, "raised"))
        raise SystemExit(3)  # this rank leaves before the step's collective
    try:
        allreduce_param_grads([torch.ones(4, dtype=torch.float64)])
        q.put((rank, "completed"))
    except Exception as e:  # the surviving rank sees an error, not a hang
        q.put((rank, "error: " + type(e).__name__))


def test_failed_rank_surfaces_as_error_not_hang():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_failing_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    got = dict(q.get(timeout=120) for _ in range(2))
    for p in procs:
        p.join(timeout=60)
    assert got[1] == "raised"
    assert got[0].startswith("error")
