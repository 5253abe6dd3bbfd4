"""Seeded test cases shared by the GPU parity tests (small enough for the oracle)."""
import math

import numpy as np
import torch

from odie_b200 import layout as host_layout


def plane_config(resolutions, dims, initial, seed=1729, router=True, k=0, activation='sigmoid'):
    levels = len(resolutions)
    width = (sum(dims) + 15) // 16 * 16
    return dict(resolutions=list(resolutions), n_levels=levels, representation='xy_planes', coarse_levels=k,
                gate_coarse_levels_K=k, gate_topology='shared', gate_position='feature', initial_active_prefix=initial,
                router_enabled=router, router_output_activation=activation, seed=seed, feature_init_std=1e-3,
                gate_parameters=(width * 32 + 32 * 16) if router else 0,
                decoder_parameters=width * 64 + 64 * 64 + 64 * 16, grid_lr=1e-2, gate_lr=1e-3, decoder_lr=1e-3,
                batch_size=1024)


def plane_case(seed=7, levels=16, dims=None, dense=10, packed=4, base=4, finest=96, fraction=.3):
    """Config + supports + caps: `dense` full-cover levels, `packed` sparse levels, the rest empty."""
    rng = np.random.default_rng(seed)
    resolutions = [int(round(base * (finest / base) ** (i / (levels - 1)))) for i in range(levels)]
    dims = dims or [2] * levels
    supports, caps = [], []
    for level, r in enumerate(resolutions):
        points = host_layout.align8(r * r)
        if level < dense:
            support = np.ones(r * r, dtype=bool)
            cap = points
        elif level < dense + packed:
            support = rng.random(r * r) < fraction
            cap = host_layout.align8(host_layout.plane_closure(support, r).numel()) + 8
        else:
            support = np.zeros(r * r, dtype=bool)
            cap = min(points, 64)
        supports.append(torch.from_numpy(support))
        caps.append(min(cap, points))
    return resolutions, dims, supports, caps


def layout_numpy(lay):
    return dict(descriptors=lay['descriptors'].numpy(), node_bitmap=lay['node_bitmap'].numpy(),
                node_prefix=lay['node_prefix'].numpy(), bitmap=lay['bitmap'].numpy())


def coordinates_with_edges(n, seed):
    """Uniform coordinates plus the exact corners and edges of the unit square."""
    rng = np.random.default_rng(seed)
    xy = rng.random((n, 2), dtype=np.float32)
    edges = np.array([[0, 0], [1, 1], [0, 1], [1, 0], [.5, .5], [1, .25], [.75, 0]], dtype=np.float32)
    xy[:len(edges)] = edges
    return xy


def random_image(height, width, seed):
    rng = np.random.default_rng(seed)
    return rng.integers(0, 256, (height * width, 3), dtype=np.uint8)


FP16_QUANTUM = 2.0 ** -24  # spacing of the fp16 subnormals: one step of an fp16-rounded value near zero


def close(actual, expected, rtol, floor=None, what='', quantum=0.0):
    """Per-element relative tolerance with a small stated floor:
        |a - e| <= rtol * |e| + max(floor * rms(e), quantum),
    rms over the nonzero expected values (floor defaults to rtol / 2; floor 0: purely relative).  The floor
    only matters for elements far below the tensor's typical magnitude (cancellation in a sum, a gradient
    through a near-zero activation); `quantum` (FP16_QUANTUM for values rounded to fp16) admits one step of
    the fp16 grid where values fall in its subnormal range.  Returns the worst relative error over the
    elements above the floor."""
    actual = np.asarray(actual, dtype=np.float64)
    expected = np.asarray(expected, dtype=np.float64)
    floor = rtol / 2 if floor is None else floor
    nonzero = expected[expected != 0]
    rms = np.sqrt(np.mean(nonzero * nonzero)) if nonzero.size else 0.0
    atol = max(floor * rms, quantum)
    diff = np.abs(actual - expected)
    bad = ~(diff <= rtol * np.abs(expected) + atol)
    big = np.abs(expected) > (atol / rtol if rtol else 0.0)
    worst = float((diff[big] / np.abs(expected[big])).max()) if big.any() else 0.0
    assert not bad.any(), (f'{what}: {bad.sum()} of {bad.size} outside rtol={rtol} + max({floor} x rms, '
                           f'{quantum:.1e}); worst |d|={diff.max():.3e}, worst relative {worst:.3e}, rms {rms:.3e}')
    return worst


def scatter_bound(backward, values, value_rtol=0.0, value_floor=0.0, quantum=0.0, sum_rtol=1e-5):
    """Per-parameter tolerance of a gradient scatter grad = sum_k w_k v_k (bilinear weights w >= 0), given
    backward(upstream), the oracle's fp64 scatter (linear in the upstream):
      * the fp32 summation of the terms in any order: sum_rtol x sum_k w_k |v_k| (1e-5: the rounding of up to
        ~160 fp32 additions, far more than any entry here receives in the worst case);
      * the tolerance of the values themselves, value_rtol |v| + max(value_floor x rms(v), quantum), carried
        through the weights: value_rtol x sum w |v| + that absolute part x sum w."""
    v = np.asarray(values, dtype=np.float32)
    magnitude = backward(np.abs(v).astype(np.float16))
    nonzero = v[v != 0].astype(np.float64)
    atol = max(value_floor * (np.sqrt(np.mean(nonzero * nonzero)) if nonzero.size else 0.0), quantum)
    bound = (sum_rtol + value_rtol) * magnitude
    if atol:
        bound = bound + atol * backward(np.ones(v.shape, dtype=np.float16))
    return bound


def close_bound(actual, expected, bound, what=''):
    """|a - e| <= bound element by element; returns the worst |a - e| / bound."""
    actual = np.asarray(actual, dtype=np.float64)
    expected = np.asarray(expected, dtype=np.float64)
    diff = np.abs(actual - expected)
    bad = diff > bound
    ratio = float(np.max(np.where(bound > 0, diff / np.where(bound > 0, bound, 1), np.where(diff > 0, np.inf, 0))))
    assert not bad.any(), f'{what}: {bad.sum()} of {bad.size} outside the bound; worst |d| / bound = {ratio:.3e}'
    return ratio
