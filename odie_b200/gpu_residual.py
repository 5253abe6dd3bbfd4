"""Live residual scoring and exact greedy selection on the GPU (odie/gpu_residual.py).

DeviceScores streams model predictions into per-cell fp64 residual totals
(score_chunk); select_device runs the exact greedy (selection_init /
selection_chunk) on those totals without moving them to the host, and only the
selected support and node masks come back.  Buffers are torch tensors on the
current device; kernels run on the current stream.
"""
import math
import time

import numpy as np
import torch

from . import _lib
from . import selection as host
from .evaluation import coordinates


class DeviceScores:
    def __init__(self, shape, resolution):
        self.shape, self.resolution = shape, resolution
        height, width = shape
        xmap = host.axis_buckets(width, resolution)
        self.ymap = host.axis_buckets(height, resolution)
        bounds = np.arange(resolution + 1)
        xb = np.searchsorted(xmap, bounds).astype(np.int32)
        yb = np.searchsorted(self.ymap, bounds).astype(np.int32)
        self.counts = (np.diff(yb).astype(np.int64)[:, None] * np.diff(xb)[None, :]).reshape(-1)
        self.xb, self.yb = torch.from_numpy(xb).cuda(), torch.from_numpy(yb).cuda()
        self.totals = torch.zeros(resolution * resolution, dtype=torch.float64, device='cuda')

    def add(self, prediction, target, begin):
        """Accumulate the residual of predictions for pixel ids [begin, begin + len(prediction))."""
        prediction, target = prediction.contiguous(), target.contiguous()
        end, width = begin + prediction.shape[0], self.shape[1]
        first_y = int(self.ymap[begin // width])
        active = (int(self.ymap[(end - 1) // width]) - first_y + 1) * self.resolution
        _lib.check(_lib.library().score_chunk(
            prediction.data_ptr(), target.data_ptr(), begin, end, width, self.resolution, first_y, active,
            self.xb.data_ptr(), self.yb.data_ptr(), self.totals.data_ptr(), target.dtype == torch.uint8,
            torch.cuda.current_stream().cuda_stream), 'score_chunk')


def select_device(scores, n, resolution, cap, normalized=True, chunk=4096, launches_per_check=8, trace=None):
    """Exact greedy B2 (normalized) / E on device fp64 scores [n]; returns (support, record)."""
    lib = _lib.library()
    points = host.align8(n)
    sizes, offsets, tree_size = host.tree_shape(n)
    device = scores.device
    missing = torch.empty(n, dtype=torch.int32, device=device)
    chosen = torch.empty(n, dtype=torch.uint8, device=device)
    nodes = torch.empty(points, dtype=torch.uint8, device=device)
    tree = torch.empty(tree_size, dtype=torch.int32, device=device)
    dev_offsets = torch.from_numpy(offsets).to(device)
    dev_sizes = torch.from_numpy(sizes).to(device)
    stats = torch.zeros(4, dtype=torch.int64, device=device)
    stream = torch.cuda.current_stream().cuda_stream
    started = time.perf_counter()
    _lib.check(lib.selection_init(scores.data_ptr(), n, points, missing.data_ptr(), chosen.data_ptr(),
                                  nodes.data_ptr(), tree.data_ptr(), stats.data_ptr(), offsets.ctypes.data,
                                  sizes.ctypes.data, len(sizes), stream), 'selection_init')
    launches = 0
    status = np.zeros(4, dtype=np.int64)
    limit = n + 1  # every launch either selects chunk cells or finishes
    while not status[2] and not status[3]:
        for _ in range(launches_per_check):
            _lib.check(lib.selection_chunk(scores.data_ptr(), n, points, resolution, cap, bool(normalized),
                                           missing.data_ptr(), chosen.data_ptr(), nodes.data_ptr(), tree.data_ptr(),
                                           dev_offsets.data_ptr(), dev_sizes.data_ptr(), len(sizes), chunk,
                                           stats.data_ptr(), _lib.ptr(trace), stream), 'selection_chunk')
            launches += 1
        status = stats.cpu().numpy()
        if launches * chunk > limit + chunk * launches_per_check:
            raise RuntimeError('greedy selection did not finish within its iteration bound')
    if status[3]:
        raise AssertionError('CUDA marginal-cost invariant failed')
    selected = chosen.cpu().numpy().astype(bool)
    node_mask = nodes.cpu().numpy().astype(bool)
    policy = ('B2 GPU residual / exact newly added closure-node parameters' if normalized
              else 'E GPU residual; exact node capacity constraint')
    support, record = host.result_record(selected, node_mask, resolution, cap, policy, int(status[1]))
    if record['closure_nodes'] != int(status[0]):
        raise AssertionError('Device and host closure counts differ')
    record.update(cuda_end_to_end_seconds=time.perf_counter() - started, launches=launches,
                  score_gpu_to_cpu_copies=0, score_cpu_to_gpu_copies=0,
                  selection_backend='cuda_device_residual_exact_greedy')
    return support, record


@torch.no_grad()
def select_live(model, target, shape, resolution, cap, dim, batch_size, validate_scores=False):
    """Score the live model on the whole image, then select the next level's support (odie/gpu_residual.py:130-179)."""
    torch.cuda.synchronize()
    started = time.perf_counter()
    was_training = model.training
    model.eval()
    try:
        scores = DeviceScores(shape, resolution)
        total = torch.zeros((), dtype=torch.float64, device='cuda')
        data = getattr(target, 'data', target)
        pixels = data.shape[0]
        for begin in range(0, pixels, batch_size):
            ids = torch.arange(begin, min(begin + batch_size, pixels), device='cuda')
            prediction = model(coordinates(shape, ids)).float()
            truth = target[ids]
            total += (prediction - truth).square().double().sum()
            scores.add(prediction, data[begin:begin + ids.numel()] if data.dtype == torch.uint8 else truth, begin)
        torch.cuda.synchronize()
        scoring_seconds = time.perf_counter() - started
        mse = float(total.item() / (pixels * 3))
        if not math.isfinite(mse) or not bool(torch.isfinite(scores.totals).all()):
            raise FloatingPointError('GPU live RGB residual is nonfinite')
        support, record = select_device(scores.totals, resolution * resolution, resolution, cap)
        record.update(plane_dim=dim, normalize_by_cost=True)
        downloaded = scores.totals.cpu().numpy() if validate_scores else None
        torch.cuda.synchronize()
        timing = dict(pipeline_seconds=time.perf_counter() - started, inference_and_scoring_seconds=scoring_seconds,
                      greedy_seconds=record['cuda_end_to_end_seconds'], prediction_gpu_to_cpu_copies=0,
                      gt_gpu_to_cpu_copies=0, validation_only_score_download=bool(validate_scores))
        return ({'mse': mse, 'psnr_db': -10 * math.log10(mse) if mse else None},
                support, record, scores.counts, timing, downloaded)
    finally:
        model.train(was_training)
