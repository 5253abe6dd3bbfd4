"""Data-parallel training over the GPUs of one node (no reference counterpart: the reference is single-GPU).

Work is partitioned by spatial ownership: rank r of N trains the model of row
band r of the image (its own grid tables, its own coordinates), so coordinates
and table gradients never cross GPUs.  Only the shared heads (router / gate MLP
and decoder) are replicated: every rank starts from rank 0's weights and, each
step, applies the sum of all ranks' head gradients (one all-reduce of
head_count fp32 values, NCCL over NVLink on GPUs, gloo in the CPU tests).
Every rank issues the same collectives in the same order.
"""
import numpy as np
import torch
import torch.distributed as dist


def band_rows(height, rank, ranks):
    """Image rows [first, last) of rank's band: contiguous, covering every row once across ranks."""
    rows = np.array_split(np.arange(height), ranks)[rank]
    return int(rows[0]), int(rows[-1]) + 1


def broadcast_heads(model, src=0, group=None):
    """Make every rank's shared heads equal to rank src's."""
    for head in (model.gate, model.decoder):
        if head is not None:
            dist.broadcast(head.params.data, src, group=group)


def head_gradient_buffer(model, device='cuda'):
    """The fp32 buffer the runtime accumulates the head gradients into (gate | decoder), shared with NCCL."""
    count = (model.gate.params.numel() if model.gate is not None else 0) + model.decoder.params.numel()
    return torch.zeros(count, dtype=torch.float32, device=device)


class DataParallelStep:
    """One training step: local forward/backward + grid update, all-reduce of the head gradients, head update.

    runtime: an object with step_grads(ids) (writes this rank's head gradient into head_grad) and step_heads().
    """

    def __init__(self, runtime, head_grad, group=None):
        self.runtime, self.head_grad, self.group = runtime, head_grad, group
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1

    def __call__(self, ids):
        self.runtime.step_grads(ids)
        if self.world > 1:
            dist.all_reduce(self.head_grad, op=dist.ReduceOp.SUM, group=self.group)
        self.runtime.step_heads()


class NativeRuntime:
    """step_grads / step_heads of a NativeOptimizer through the C-ABI (odie_step_grads, odie_step_heads)."""

    def __init__(self, optimizer):
        self.opt = optimizer

    def step_grads(self, ids):
        self.opt.check(self.opt.lib.odie_step_grads(self.opt.handle, ids.data_ptr(), ids.numel(), 1))

    def step_heads(self):
        self.opt.check(self.opt.lib.odie_step_heads(self.opt.handle))
