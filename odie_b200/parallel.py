"""Data-parallel training over the GPUs of one node (no reference counterpart: the reference is single-GPU).

Work is partitioned by spatial ownership: rank r of N trains the expert tables of
its own row band of the image on its own coordinates, so coordinates and table
gradients never cross GPUs.  Only the shared parameters (router / gate MLP,
decoder and, for the gigapixel model, the coarse router grid) are replicated:
every rank starts from rank 0's weights and, each step, applies the sum of all
ranks' gradients of them (one all-reduce of fp32 values, NCCL over NVLink on
GPUs, gloo in the CPU tests).  Every rank issues the same collectives in the
same order.
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


def head_gradient_buffer(model, device='cuda', router_grid=False):
    """The fp32 buffer of the gradients summed across ranks, shared with NCCL: the heads (gate | decoder), then,
    with router_grid, the shared router grid's gradient (routed experts whose router grid is one model across
    ranks).  Returns (buffer, head view, router-grid view or None)."""
    heads = (model.gate.params.numel() if model.gate is not None else 0) + model.decoder.params.numel()
    extra = model.router_grid.numel() if router_grid else 0
    buffer = torch.zeros(heads + extra, dtype=torch.float32, device=device)
    return buffer, buffer[:heads], (buffer[heads:] if router_grid else None)


class DataParallelStep:
    """One training step: local forward/backward + grid update, all-reduce of the shared gradients, head update.

    runtime: an object with step_grads(ids) (writes this rank's shared gradients into `grads`) and step_heads().
    overlap_stream (CUDA only): the stream on which the runtime computes the shared gradients (its side branch);
    the all-reduce is issued there, so that it runs while the runtime's main stream still scatters into and
    updates the rank's own expert tables, and the main stream waits for the sum only before step_heads.
    """

    def __init__(self, runtime, grads, group=None, overlap_stream=None):
        self.runtime, self.grads, self.group, self.overlap_stream = runtime, grads, group, overlap_stream
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1

    def __call__(self, ids):
        self.runtime.step_grads(ids)
        if self.world > 1:
            if self.overlap_stream is not None:
                with torch.cuda.stream(self.overlap_stream):
                    work = dist.all_reduce(self.grads, op=dist.ReduceOp.SUM, group=self.group, async_op=True)
                work.wait()  # the caller's (training) stream waits for the sum
            else:
                dist.all_reduce(self.grads, op=dist.ReduceOp.SUM, group=self.group)
        self.runtime.step_heads()


class NativeRuntime:
    """step_grads / step_heads of a NativeOptimizer through the C-ABI (odie_step_grads, odie_step_heads)."""

    def __init__(self, optimizer):
        self.opt = optimizer

    def side_stream(self):
        """The runtime's side branch as a torch stream (routed experts), or None."""
        handle = int(self.opt.pointers.get('side_stream', 0))
        return torch.cuda.ExternalStream(handle) if handle else None

    def step_grads(self, ids):
        self.opt.check(self.opt.lib.odie_step_grads(self.opt.handle, ids.data_ptr(), ids.numel(), 1))

    def step_heads(self):
        self.opt.check(self.opt.lib.odie_step_heads(self.opt.handle))
