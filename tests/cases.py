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


def close(actual, expected, rtol, scale_atol=None, what=''):
    """|a - e| <= rtol * |e| + atol with atol = rtol * max|e| (a tolerance relative to the tensor's scale)."""
    actual = np.asarray(actual, dtype=np.float64)
    expected = np.asarray(expected, dtype=np.float64)
    atol = (scale_atol if scale_atol is not None else rtol) * (np.abs(expected).max() if expected.size else 0)
    bad = np.abs(actual - expected) > rtol * np.abs(expected) + atol
    assert not bad.any(), (f'{what}: {bad.sum()} of {bad.size} outside rtol={rtol}; worst |d|='
                           f'{np.abs(actual - expected).max():.3e}, max|e|={np.abs(expected).max():.3e}')
