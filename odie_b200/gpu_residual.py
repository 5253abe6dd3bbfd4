"""Live residual scoring and exact greedy selection on the GPU (the stage boundary of odie/gpu_residual.py).

The image's pixels map to the next level's R x R cells through the exact fp32 cell thresholds
(selection.axis_buckets); a ResidualAccumulator keeps one fp64 total per cell on the device and adds each
chunk of predictions to it with score_chunk (raster order within a cell, bit-identical to the CPU
reference).  select_live decodes the whole image chunk by chunk -- through the fused native decode
(odie_decode) into one reused buffer when a training runtime is attached to the model, else through the
module's forward -- and then runs the exact greedy on the device totals (selection_init / selection_chunk);
only the chosen support and node masks come back to the host.
"""
import math
import time
import weakref

import numpy as np
import torch

from . import _lib
from . import selection as host
from .evaluation import coordinates


class ResidualAccumulator:
    """Per-cell fp64 residual totals of an R x R level over a (height, width) image, on the current device.

    Each axis of the image is cut into R buckets of consecutive pixels (the cells whose fp32 geometry the
    pixels' endpoint coordinates fall in); `counts` holds the pixels of every cell."""

    def __init__(self, shape, resolution):
        height, width = shape
        self.shape, self.resolution = shape, resolution
        self.row_cell = host.axis_buckets(height, resolution)
        column_cell = host.axis_buckets(width, resolution)
        cut = np.arange(resolution + 1)
        x_edges = np.searchsorted(column_cell, cut).astype(np.int32)  # first pixel column of each cell
        y_edges = np.searchsorted(self.row_cell, cut).astype(np.int32)
        self.counts = np.outer(np.diff(y_edges).astype(np.int64), np.diff(x_edges)).reshape(-1)
        self.x_edges = torch.from_numpy(x_edges).cuda()
        self.y_edges = torch.from_numpy(y_edges).cuda()
        self.totals = torch.zeros(resolution * resolution, dtype=torch.float64, device='cuda')

    def accumulate(self, prediction, target_rows, first_pixel):
        """Add the residual of fp32 predictions [n, 3] for pixels [first_pixel, first_pixel + n); target_rows:
        the same pixels' u8 (or fp32) RGB."""
        prediction, target_rows = prediction.contiguous(), target_rows.contiguous()  # read as packed [n, 3] rows
        width = self.shape[1]
        last_pixel = first_pixel + prediction.shape[0]
        top = int(self.row_cell[first_pixel // width])
        bottom = int(self.row_cell[(last_pixel - 1) // width])
        cells = (bottom - top + 1) * self.resolution  # only the cell rows the chunk's pixel rows touch
        _lib.check(_lib.library().score_chunk(
            prediction.data_ptr(), target_rows.data_ptr(), first_pixel, last_pixel, width, self.resolution, top, cells,
            self.x_edges.data_ptr(), self.y_edges.data_ptr(), self.totals.data_ptr(),
            target_rows.dtype == torch.uint8, torch.cuda.current_stream().cuda_stream), 'score_chunk')


def attach_runtime(model, runtime):
    """Let the stage boundary decode `model` through its training runtime (a NativeOptimizer), held weakly."""
    model._odie_runtime = weakref.ref(runtime)


def attached_runtime(model):
    ref = getattr(model, '_odie_runtime', None)
    runtime = ref() if ref is not None else None
    return runtime if runtime is not None and getattr(runtime, 'handle', None) else None


def fused_chunks(runtime, pixels, chunk):
    """(first pixel, fp32 predictions [n, 3]) over the image through odie_decode, one reused device buffer."""
    buffer = torch.empty((chunk, 3), dtype=torch.float32, device='cuda')
    for first in range(0, pixels, chunk):
        count = min(chunk, pixels - first)
        runtime.decode(first, count, rgb=buffer[:count])
        yield first, buffer[:count]


def module_chunks(model, shape, pixels, chunk):
    """The same through the module's forward (a model without a training runtime)."""
    for first in range(0, pixels, chunk):
        ids = torch.arange(first, min(first + chunk, pixels), device='cuda')
        yield first, model(coordinates(shape, ids)).float()


def select_device(scores, n, resolution, cap, normalized=True, chunk=4096, launches_per_check=8, trace=None):
    """Exact greedy B2 (normalized) / E on device fp64 scores [n] (selection_init / selection_chunk); the host
    polls the device status every `launches_per_check` launches.  Returns (support, record)."""
    lib = _lib.library()
    device, stream = scores.device, torch.cuda.current_stream().cuda_stream
    points = host.align8(n)
    level_sizes, level_offsets, tree_entries = host.tree_shape(n)
    buffers = dict(missing=torch.empty(n, dtype=torch.int32, device=device),
                   chosen=torch.empty(n, dtype=torch.uint8, device=device),
                   nodes=torch.empty(points, dtype=torch.uint8, device=device),
                   tree=torch.empty(tree_entries, dtype=torch.int32, device=device),
                   offsets=torch.from_numpy(level_offsets).to(device), sizes=torch.from_numpy(level_sizes).to(device),
                   stats=torch.zeros(4, dtype=torch.int64, device=device))
    b = {k: v.data_ptr() for k, v in buffers.items()}
    started = time.perf_counter()
    _lib.check(lib.selection_init(scores.data_ptr(), n, points, b['missing'], b['chosen'], b['nodes'], b['tree'],
                                  b['stats'], level_offsets.ctypes.data, level_sizes.ctypes.data, len(level_sizes),
                                  stream), 'selection_init')
    launches, stats = 0, np.zeros(4, dtype=np.int64)
    # every launch either makes `chunk` choices or finishes, so n / chunk launches (plus a check's worth) suffice
    budget = (n + chunk) // chunk + launches_per_check
    while not (stats[2] or stats[3]):
        if launches >= budget:
            raise RuntimeError('greedy selection did not finish within its iteration bound')
        for _ in range(launches_per_check):
            _lib.check(lib.selection_chunk(scores.data_ptr(), n, points, resolution, cap, bool(normalized),
                                           b['missing'], b['chosen'], b['nodes'], b['tree'], b['offsets'], b['sizes'],
                                           len(level_sizes), chunk, b['stats'], _lib.ptr(trace), stream),
                       'selection_chunk')
        launches += launches_per_check
        stats = buffers['stats'].cpu().numpy()
    if stats[3]:
        raise AssertionError('CUDA marginal-cost invariant failed')
    policy = ('B2 GPU residual / exact newly added closure-node parameters' if normalized
              else 'E GPU residual; exact node capacity constraint')
    support, record = host.result_record(buffers['chosen'].cpu().numpy().astype(bool),
                                         buffers['nodes'].cpu().numpy().astype(bool), resolution, cap, policy,
                                         int(stats[1]))
    if record['closure_nodes'] != int(stats[0]):
        raise AssertionError('Device and host closure counts differ')
    record.update(cuda_end_to_end_seconds=time.perf_counter() - started, launches=launches,
                  score_gpu_to_cpu_copies=0, score_cpu_to_gpu_copies=0,
                  selection_backend='cuda_device_residual_exact_greedy')
    return support, record


@torch.no_grad()
def select_live(model, target, shape, resolution, cap, dim, batch_size, validate_scores=False, optimizer=None):
    """Score the live model over the whole image on the GPU, then choose the next level's support with the exact
    greedy (the stage boundary of odie/gpu_residual.py:131).  The decode runs through `optimizer` (a NativeOptimizer)
    or the runtime attached to the model (attach_runtime) in chunks of max(batch_size, its capacity); without one,
    through the module.  Returns (metrics, support, record, cell pixel counts, timing, scores or None)."""
    runtime = optimizer if optimizer is not None else attached_runtime(model)
    data = getattr(target, 'data', target)
    pixels = data.shape[0]
    torch.cuda.synchronize()
    started = time.perf_counter()
    was_training = model.training
    model.eval()
    try:
        residual = ResidualAccumulator(shape, resolution)
        squared = torch.zeros((), dtype=torch.float64, device='cuda')
        if runtime is not None:
            chunk = max(batch_size, runtime.batch)
            chunks = fused_chunks(runtime, pixels, chunk)
        else:
            chunks = module_chunks(model, shape, pixels, batch_size)
        for first, prediction in chunks:
            last = first + prediction.shape[0]
            rows = data[first:last]
            truth = rows.float() / 255. if rows.dtype == torch.uint8 else rows
            squared += (prediction - truth).square().sum(dtype=torch.float64)
            # u8 targets go to the scorer as bytes: it divides by 255 with correct rounding, as the CPU reference does
            residual.accumulate(prediction, rows if rows.dtype == torch.uint8 else truth, first)
        torch.cuda.synchronize()
        scoring_seconds = time.perf_counter() - started
        mse = float(squared.item() / (pixels * 3))
        if not math.isfinite(mse) or not bool(torch.isfinite(residual.totals).all()):
            raise FloatingPointError('GPU live RGB residual is nonfinite')
        support, record = select_device(residual.totals, resolution * resolution, resolution, cap)
        record.update(plane_dim=dim, normalize_by_cost=True)
        downloaded = residual.totals.cpu().numpy() if validate_scores else None
        torch.cuda.synchronize()
        timing = dict(pipeline_seconds=time.perf_counter() - started, inference_and_scoring_seconds=scoring_seconds,
                      greedy_seconds=record['cuda_end_to_end_seconds'], prediction_gpu_to_cpu_copies=0,
                      gt_gpu_to_cpu_copies=0, validation_only_score_download=bool(validate_scores),
                      decode_path='fused odie_decode' if runtime is not None else 'module forward')
        metrics = {'mse': mse, 'psnr_db': -10 * math.log10(mse) if mse else None}
        return metrics, support, record, residual.counts, timing, downloaded
    finally:
        model.train(was_training)
