"""Worker of test_gpu_overlap.test_overlapped_allreduce_two_gpus_matches_full_batch
(launched by torch.distributed.run, one process per GPU, NCCL).

Each rank takes 2 samples of a 4-sample c5-shaped training problem (512->512,
38x38, groups 2, offset groups 4, bf16).  grad_weight / grad_bias are
all-reduced once with the overlapped hook and once after the backward; both
must agree, and equal the single-GPU full-batch gradients within the bf16
tolerance.  Prints OVERLAP OK on rank 0.
"""
import os
import sys
from datetime import timedelta

import numpy as np
import torch
import torch.distributed as dist

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, os.path.join(REPO, "mps-deform-conv_b200"))

import mps_deform_conv as mdc  # noqa: E402
from mps_deform_conv.sharding import OverlappedParamAllReduce, allreduce_param_grads, shard_range  # noqa: E402
from mps_deform_conv.workloads import PROBLEMS, make_inputs  # noqa: E402


def rel(a, b):
    a = a.double().cpu().numpy()
    b = b.double().cpu().numpy()
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


def main():
    rank, world, local = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"]), int(os.environ["LOCAL_RANK"])
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", timeout=timedelta(seconds=60), device_id=dev)
    p = PROBLEMS["c5_train_bf16"]
    global_batch = 4
    first, nb = shard_range(global_batch, world, rank)
    st, pd, dl = (p.stride,) * 2, (p.padding,) * 2, (p.dilation,) * 2

    def run(batch, offset, mode):
        inp = make_inputs(p, dev, batch=batch, batch_offset=offset)
        leaves = [inp[k].clone().requires_grad_(True) for k in ("input", "offset", "weight", "bias", "mask")]
        ar = OverlappedParamAllReduce() if mode == "overlap" else None
        mdc.set_param_grad_hook(ar)
        try:
            out = mdc.deform_conv2d(leaves[0], leaves[1], leaves[2], leaves[3], st, pd, dl, leaves[4])
            g = torch.autograd.grad(out, leaves, inp["grad_output"])
        finally:
            mdc.set_param_grad_hook(None)
        gw, gb = g[2], g[3]
        if ar is not None:
            ar.wait()
        elif mode == "serial":
            allreduce_param_grads([gw, gb])
        torch.cuda.synchronize()
        return gw, gb

    gw_o, gb_o = run(nb, first, "overlap")
    gw_s, gb_s = run(nb, first, "serial")
    assert torch.equal(gw_o, gw_s), "grad_weight: overlapped and serial all-reduce differ"
    assert rel(gb_o, gb_s) <= 1e-3, "grad_bias: overlapped and serial all-reduce differ"
    if rank == 0:
        gw_f, gb_f = run(global_batch, 0, "single")
        assert rel(gw_o, gw_f) <= 1e-2, rel(gw_o, gw_f)
        assert rel(gb_o, gb_f) <= 1e-2, rel(gb_o, gb_f)
        print("OVERLAP OK", rel(gw_o, gw_f), rel(gb_o, gb_f), flush=True)
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
