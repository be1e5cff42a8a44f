"""Batch sharding across ranks for deformable-convolution layers.

Samples are independent in the forward pass and in grad_input / grad_offset /
grad_mask, so a global batch splits across ranks with no exchange; only the
parameter gradients (grad_weight, grad_bias) sum over the batch.  This module
holds the two host-side pieces of that scheme:

* ``shard_range`` -- which contiguous samples of the global batch a rank owns;
* ``allreduce_param_grads`` -- one all-reduce (sum) of the parameter gradients
  packed into a single flat bucket, so a step issues one collective instead of
  one per tensor.  Works on any torch.distributed backend (NCCL over NVLink on
  GPUs, gloo on CPU).
* ``OverlappedParamAllReduce`` -- the same all-reduce started from the
  backward's parameter-gradient hook (``set_param_grad_hook``) on a side
  stream, so it runs while the backward finishes the input / offset / mask
  gradients.
"""
from __future__ import annotations

from typing import List, Optional, Sequence, Tuple

import torch


def shard_range(global_batch: int, world_size: int, rank: int) -> Tuple[int, int]:
    """(first sample, sample count) of `rank`'s shard; shards differ by at most one sample."""
    if world_size <= 0 or not (0 <= rank < world_size):
        raise ValueError(f"invalid rank {rank} for world size {world_size}")
    base, extra = divmod(global_batch, world_size)
    start = rank * base + min(rank, extra)
    return start, base + (1 if rank < extra else 0)


def allreduce_param_grads(grads: Sequence[Optional[torch.Tensor]], group=None,
                          average: bool = False) -> List[Optional[torch.Tensor]]:
    """Sum (or average) the given gradients over all ranks in one flat-bucket all-reduce.

    The gradients are packed into one contiguous buffer of their common dtype,
    reduced in place, and copied back into the original tensors, which are
    returned.  ``None`` entries are passed through.
    """
    import torch.distributed as dist

    present = [g for g in grads if g is not None]
    if not present or not dist.is_initialized() or dist.get_world_size(group) == 1:
        return list(grads)
    with torch.cuda.nvtx.range("dcn_param_allreduce"):
        flat = torch.cat([g.reshape(-1) for g in present])
        dist.all_reduce(flat, op=dist.ReduceOp.SUM, group=group)
        if average:
            flat /= dist.get_world_size(group)
        off = 0
        for g in present:
            n = g.numel()
            g.copy_(flat[off:off + n].view_as(g))
            off += n
    return list(grads)


class OverlappedParamAllReduce:
    """Parameter-gradient hook that all-reduces grad_weight / grad_bias on a
    side stream while the rest of the backward runs.

    Install with ``mps_deform_conv.set_param_grad_hook(h)``; after the backward
    returns, call ``h.wait()`` before reading the parameter gradients (it makes
    the current stream wait for the side stream; on CPU the reduction already
    ran inside the hook).  The gradients are reduced in place, so the caller
    keeps them alive until ``wait()`` and reads them only after it: with
    ``loss.backward()`` the parameters' ``.grad`` must be None before the
    backward (``zero_grad(set_to_none=True)``, the default), since autograd
    would otherwise add the new gradient into the old one on the current
    stream before the side-stream reduction ends.  Every rank must run the same
    layers in the same order, as for any collective.
    """

    def __init__(self, group=None, average: bool = False, stream=None):
        self.group = group
        self.average = average
        self._stream = stream
        self.calls = 0

    def _side_stream(self):
        if self._stream is None:
            self._stream = torch.cuda.Stream()
        return self._stream

    def __call__(self, grad_weight, grad_bias):
        self.calls += 1
        grads = [grad_weight, grad_bias]
        dev = next((g.device for g in grads if g is not None), None)
        if dev is None or dev.type != "cuda":
            allreduce_param_grads(grads, self.group, self.average)
            return
        side = self._side_stream()
        side.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(side):
            allreduce_param_grads(grads, self.group, self.average)

    def wait(self) -> None:
        if self._stream is not None:
            torch.cuda.current_stream().wait_stream(self._stream)
