"""Host-side helpers of live-residual allocation (odie/selection.py).

native_thresholds maps each cell boundary of an R-cell axis to the smallest
fp32 endpoint coordinate x whose fused fmaf(R-1, x, 0.5) rounds to at least
that boundary, using exact rational arithmetic; pixel_cells, closure_nodes and
the result validation follow the reference's contract.  The selection itself
runs on the GPU (gpu_residual.select_device).
"""
from fractions import Fraction
from functools import lru_cache
import struct

import numpy as np

from .layout import align8


def _bits(x):
    return struct.unpack('<I', struct.pack('<f', x))[0]


def _float(bits):
    return struct.unpack('<f', struct.pack('<I', bits))[0]


@lru_cache(maxsize=128)
def native_thresholds(resolution):
    """Smallest fp32 x in [0, 1] with floor(fl(fmaf(R-1, x, 0.5))) >= k, for k = 1..R-1 (odie/selection.py:16-42)."""
    if type(resolution) is not int or not 2 <= resolution <= 2**23:
        raise ValueError('Resolution must be an integer between 2 and 2^23')
    scale = resolution - 1
    one = _bits(1.0)
    out = []
    for k in range(1, resolution):
        kb = _bits(float(k))
        below = Fraction(_float(kb - 1))
        # fl(v) >= k  <=>  v > midpoint(prev(k), k), or v == midpoint when k wins the tie (even significand)
        need = (below + k) / 2 - Fraction(1, 2)
        tie_ok = kb % 2 == 0

        def ok(bits):
            value = scale * Fraction(_float(bits))
            return value > need or (tie_ok and value == need)

        guess = min(max(_bits(float(need / scale)) if need > 0 else 0, 0), one)
        bits = guess
        while bits > 0 and ok(bits - 1):
            bits -= 1
        while bits < one and not ok(bits):
            bits += 1
        out.append(_float(bits))
    return tuple(out)


def axis_buckets(length, resolution):
    """Cell index of each pixel along one axis: endpoint coordinates i/(length-1) in fp32."""
    thresholds = np.asarray(native_thresholds(resolution), dtype=np.float32)
    coords = np.arange(length, dtype=np.float32) / np.float32(length - 1)
    return np.searchsorted(thresholds, coords, side='right')


def pixel_cells(shape, resolution):
    height, width = shape
    if min(height, width) < 2:
        raise ValueError('Endpoint image axes must each contain at least two pixels')
    return (axis_buckets(height, resolution)[:, None] * resolution + axis_buckets(width, resolution)[None, :]).reshape(-1)


def closure_nodes(cells, resolution):
    cells = np.asarray(cells, dtype=np.int64)
    points = align8(resolution * resolution)
    present = np.zeros(points, dtype=bool)
    for delta in (0, 1, resolution, resolution + 1):
        present[(cells + delta) % points] = True
    return np.flatnonzero(present)


def validate_scores(scores, resolution, cap):
    scores = np.asarray(scores, dtype=np.float64)
    if scores.shape != (resolution**2,) or not np.isfinite(scores).all() or (scores < 0).any():
        raise ValueError('Scores must be a finite nonnegative R^2 vector')
    if type(cap) is not int or cap % 8 or not 0 <= cap <= align8(resolution**2):
        raise ValueError('Node cap must be 8-aligned and within the native plane')
    return scores


def result_record(selected, nodes, resolution, cap, policy, iterations):
    """Closure/cap validation and the selection record (odie/selection.py:91-105)."""
    closure = closure_nodes(np.flatnonzero(selected), resolution)
    if not np.array_equal(closure, np.flatnonzero(nodes)) or len(closure) > cap:
        raise AssertionError('Selection must preserve its complete node closure')
    used = int(nodes.sum())
    return selected, {
        'policy': policy, 'selected_cells': int(selected.sum()), 'closure_nodes': used, 'node_capacity': cap,
        'unused_allocated_node_slots': int(cap - used), 'aligned_used_node_slots': align8(used),
        'node_capacity_utilization': float(used / cap) if cap else 0.,
        'aligned_capacity_utilization': float(align8(used) / cap) if cap else 0.,
        'complete_interpolation_closure': True, 'tie_order': 'descending score, ascending native cell ID',
        'iterations': iterations}


def tree_shape(n):
    """Level sizes and offsets of the 32-ary, 5-category tournament tree (odie/gpu_residual.py:79-90)."""
    sizes, offsets, total, children = [], [], 0, n
    while True:
        parents = (children + 31) // 32
        sizes.append(parents)
        offsets.append(total)
        total += parents * 5
        if parents == 1:
            break
        children = parents
    return np.asarray(sizes, dtype=np.int32), np.asarray(offsets, dtype=np.int32), total
