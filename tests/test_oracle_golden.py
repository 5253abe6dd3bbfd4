"""CPU: the oracle and the product's host logic against the reference's own outputs.

The golden vectors were produced by running the reference's CPU code
(odie/selection.py, odie/model.py, odie/config.py) in the build container
(tests/golden/make_golden.py).  Every comparison here is exact.
"""
import json

import numpy as np
import pytest
import torch

from oracle import oracle
from odie_b200 import layout, selection


# ---------------------------------------------------------------- a17/a18: selection and scoring
def greedy_cases(g):
    keys = sorted({k.rsplit('_scores', 1)[0] for k in g if k.endswith('_scores')})
    for key in keys:
        parts = key.split('_')
        r, cap = int(parts[-2][1:]), int(parts[-1][1:])
        yield key, r, cap


def test_greedy_b2_e_bit_exact(golden):
    g = golden('greedy.npz')
    cases = list(greedy_cases(g))
    assert len(cases) >= 10
    for key, r, cap in cases:
        scores = g[f'{key}_scores']
        for tag, normalized in (('B2', True), ('E', False)):
            chosen, nodes, iterations, used = oracle.select_benefit_cost(scores, r, cap, normalized)
            assert np.array_equal(chosen, g[f'{key}_{tag}_selected'].astype(bool)), (key, tag)
            assert np.array_equal(nodes, g[f'{key}_{tag}_nodes'].astype(bool)), (key, tag)
            assert iterations == int(g[f'{key}_{tag}_iterations']), (key, tag)
            assert used == int(nodes.sum()) <= cap


def test_greedy_b1_bit_exact(golden):
    g = golden('greedy.npz')
    for key, r, cap in greedy_cases(g):
        chosen, _ = oracle.select_mean_rank(np.abs(g[f'{key}_scores']), r, cap)
        assert np.array_equal(chosen, g[f'{key}_B1_selected'].astype(bool)), key


@pytest.mark.parametrize('key', ['37x53_8', '64x48_13', '101x77_100'])
def test_residual_scores_bit_exact(golden, key):
    """The C restatement of accumulate (one chunk = whole image) equals residual_scores' fp64 totals."""
    g = golden('residual.npz')
    pred, u8, total = g[f'res_pred_{key}'], g[f'res_u8_{key}'], g[f'res_total_{key}']
    h, w = map(int, key.split('_')[0].split('x'))
    r = int(key.split('_')[1])
    buckets_x = selection.axis_buckets(w, r)
    buckets_y = selection.axis_buckets(h, r)
    xb = np.searchsorted(buckets_x, np.arange(r + 1)).astype(np.int32)
    yb = np.searchsorted(buckets_y, np.arange(r + 1)).astype(np.int32)
    totals = np.zeros(r * r)
    oracle.score_chunk(pred, u8, 0, h * w, w, r, 0, r * r, xb, yb, totals, True)
    assert np.array_equal(totals, total)
    counts = (np.diff(yb).astype(np.int64)[:, None] * np.diff(xb)[None, :]).reshape(-1)
    assert np.array_equal(counts, g[f'res_counts_{key}'])


def test_residual_scores_in_chunks(golden):
    """Streaming the image in arbitrary pixel chunks gives the same totals (raster order kept)."""
    g = golden('residual.npz')
    key = '101x77_100'
    pred, u8, total = g[f'res_pred_{key}'], g[f'res_u8_{key}'], g[f'res_total_{key}']
    h, w, r = 101, 77, 100
    xmap, ymap = selection.axis_buckets(w, r), selection.axis_buckets(h, r)
    xb = np.searchsorted(xmap, np.arange(r + 1)).astype(np.int32)
    yb = np.searchsorted(ymap, np.arange(r + 1)).astype(np.int32)
    totals = np.zeros(r * r)
    for begin in range(0, h * w, 1013):
        end = min(begin + 1013, h * w)
        first_y = int(ymap[begin // w])
        active = (int(ymap[(end - 1) // w]) - first_y + 1) * r
        oracle.score_chunk(pred[begin:end], u8[begin:end], begin, end, w, r, first_y, active, xb, yb, totals, True)
    assert np.array_equal(totals, total)


# ---------------------------------------------------------------- host logic of the product
def test_thresholds_bit_exact(golden):
    g = golden('selection.npz')
    for key in (k for k in g if k.startswith('thr_')):
        r = int(key.split('_')[1])
        assert np.array_equal(np.asarray(selection.native_thresholds(r), dtype=np.float32), g[key]), r


def test_pixel_cells_bit_exact(golden):
    g = golden('selection.npz')
    for key in (k for k in g if k.startswith('cells_')):
        shape, r = key.split('_')[1], int(key.split('_')[2])
        h, w = map(int, shape.split('x'))
        assert np.array_equal(selection.pixel_cells((h, w), r), g[key]), key
    for key in (k for k in g if k.startswith('xbucket_')):
        shape, r = key.split('_')[1], int(key.split('_')[2])
        h, w = map(int, shape.split('x'))
        assert np.array_equal(selection.axis_buckets(w, r), g[key]), key
        assert np.array_equal(selection.axis_buckets(h, r), g[key.replace('xbucket', 'ybucket')]), key


def test_closures_and_node_index(golden):
    g = golden('layout.npz')
    for key in (k for k in g if k.startswith('clo_support_')):
        r = int(key.split('_')[-1])
        support = g[key]
        assert np.array_equal(selection.closure_nodes(np.flatnonzero(support), r), g[f'clo_nodes_{r}'])
        assert np.array_equal(layout.plane_closure(support, r).numpy(), g[f'clo_plane_{r}'])
    for key in (k for k in g if k.startswith('idx_nodes_')):
        points = int(key.split('_')[-1])
        bitmap, prefix = layout.make_node_index(torch.from_numpy(g[key]), points)
        assert np.array_equal(bitmap.numpy().view(np.int64), g[f'idx_bitmap_{points}'])
        assert np.array_equal(prefix.numpy(), g[f'idx_prefix_{points}'])


def test_make_layout_bit_exact(golden):
    g = golden('layout.npz')
    resolutions = [int(r) for r in g['lay_resolutions']]
    config = dict(resolutions=resolutions, n_levels=len(resolutions), representation='xy_planes', coarse_levels=0,
                  gate_topology='shared', gate_position='feature', initial_active_prefix=3)
    supports = [torch.from_numpy(g[f'lay_support_{l}']) for l in range(len(resolutions))]
    out = layout.make_layout(config, supports, [int(d) for d in g['lay_dims']], [int(c) for c in g['lay_caps']])
    assert np.array_equal(out['descriptors'].numpy(), g['lay_descriptors'])
    assert np.array_equal(out['node_bitmap'].numpy().view(np.int64), g['lay_node_bitmap'])
    assert np.array_equal(out['node_prefix'].numpy(), g['lay_node_prefix'])
    assert np.array_equal(out['bitmap'].numpy(), g['lay_bitmap'])
    assert out['params'] == int(g['lay_params']) and out['input_width'] == int(g['lay_input_width'])


def test_make_layout_rejects_bad_caps():
    config = dict(resolutions=[4, 4], n_levels=2, representation='xy_planes', coarse_levels=0,
                  gate_topology='shared', gate_position='feature', initial_active_prefix=2)
    supports = [torch.ones(16, dtype=torch.bool)] * 2
    with pytest.raises(ValueError):
        layout.make_layout(config, supports, [2, 2], [16, 12])   # cap below the closure
    with pytest.raises(ValueError):
        layout.make_layout(config, supports, [2, 3], [16, 16])   # F3 is not a native width


def test_hash_grid_layout(golden):
    g = golden('config.npz')
    encodings = {'c1': (19, 16, 1.5), 'c2': (16, 16, 1.5), 'tokyo': (21, 3, 1.841)}
    for name, (log2t, base, scale) in encodings.items():
        enc = dict(otype='HashGrid', n_levels=16, n_features_per_level=2, log2_hashmap_size=log2t,
                   base_resolution=base, per_level_scale=scale)
        _, res, caps = layout.hash_grid_layout(enc)
        assert res == list(g[f'hash_{name}_res']) and caps == list(g[f'hash_{name}_caps']), name


def test_gigapixel_plan_caps(golden):
    """The resolved gigapixel plan: its caps and resolutions are the layout the step runs on."""
    plan = json.loads(bytes(golden('config.npz')['plan_gigapixel_json']).decode())
    assert plan['n_levels'] == 16 and len(plan['cell_caps']) == 16
    assert plan['gate_parameters'] == 1536 and plan['decoder_parameters'] == 7168
    assert all(c % 8 == 0 for c in plan['cell_caps'])


# ---------------------------------------------------------------- oracle internals
def test_oracle_adam_matches_torch_adam():
    """The oracle's Adam (fp32 element math, fp64 scalars) tracks torch.optim.Adam to fp32 rounding."""
    rng = np.random.default_rng(3)
    p0 = rng.standard_normal(4096).astype(np.float32)
    param = torch.nn.Parameter(torch.from_numpy(p0.copy()))
    opt = torch.optim.Adam([param], lr=1e-2, betas=(.9, .999), eps=1e-15, foreach=False)
    p, m, v, steps = p0.copy(), np.zeros(4096, np.float32), np.zeros(4096, np.float32), np.zeros(4096, np.uint32)
    for _ in range(5):
        g = rng.standard_normal(4096).astype(np.float32)
        param.grad = torch.from_numpy(g.copy())
        opt.step()
        p, m, v, steps, _ = oracle.adam(p, m, v, steps, g * 128, 128., 1e-2, skip_zero=False)
    np.testing.assert_allclose(p, param.detach().numpy(), rtol=1e-5, atol=1e-7)
    assert (steps == 5).all()


def test_oracle_adam_skips_zero_gradients():
    p = np.ones(8, np.float32)
    g = np.array([0, 1, 0, -1, 0, 0, 2, 0], np.float32)
    p1, m1, v1, s1, _ = oracle.adam(p, np.zeros(8), np.zeros(8), np.zeros(8), g, 1., 1e-2, skip_zero=True)
    assert list(s1) == [0, 1, 0, 1, 0, 0, 1, 0]
    assert np.array_equal(p1[g == 0], p[g == 0])
    assert np.allclose(np.abs(p1[g != 0] - 1), 1e-2, rtol=1e-5)


def test_oracle_topk_ties_ascending_id():
    scores = np.array([1., 3., 3., 2., 3., 0.])
    assert list(oracle.topk(scores, 4)) == [1, 2, 4, 3]


def test_oracle_tile_scores_consistent_with_cells():
    rng = np.random.default_rng(5)
    h, w, tile = 70, 45, 16
    pred = rng.random((h * w, 3), dtype=np.float32)
    u8 = rng.integers(0, 256, (h * w, 3), dtype=np.uint8)
    scores = oracle.tile_scores(pred, u8, h, w, tile)
    d = pred.astype(np.float32) - (u8.astype(np.float32) / np.float32(255))
    per_pixel = (d * d).astype(np.float64).sum(1) / 3
    ty, tx = np.arange(h) // tile, np.arange(w) // tile
    tid = (ty[:, None] * ((w + tile - 1) // tile) + tx[None, :]).reshape(-1)
    np.testing.assert_allclose(scores, np.bincount(tid, per_pixel), rtol=1e-12)


def test_oracle_router_argmax_and_softmax():
    rng = np.random.default_rng(11)
    x = rng.standard_normal((64, 16)).astype(np.float16)
    w1 = (rng.standard_normal(32 * 16) * .3).astype(np.float16)
    w2 = (rng.standard_normal(32 * 32) * .3).astype(np.float16)
    w3 = (rng.standard_normal(16 * 32) * .3).astype(np.float16)
    expert, prob, logits = oracle.router(x, w1, w2, w3, 32, 16)
    z = logits.astype(np.float32)
    assert np.array_equal(expert, z.argmax(1))
    soft = np.exp(z - z.max(1, keepdims=True))
    np.testing.assert_allclose(prob, 1 / soft.sum(1), rtol=1e-5)


def test_oracle_routed_expert_step_consistency():
    """The routed-expert restatement: routing follows its logits, values follow p, scatters land in the chosen tables."""
    from odie_b200.layout import hash_levels
    rng = np.random.default_rng(4)
    enc = dict(n_levels=16, n_features_per_level=2, log2_hashmap_size=8, base_resolution=4, per_level_scale=1.5)
    renc = dict(n_levels=16, n_features_per_level=2, log2_hashmap_size=6, base_resolution=2, per_level_scale=1.2)
    records, stride = hash_levels(enc)
    rrecords, rtotal = hash_levels(renc)
    experts, shape = 3, (9, 11)
    tables = (rng.standard_normal(experts * stride) * .05).astype(np.float32)
    router_table = (rng.standard_normal(rtotal) * .5).astype(np.float32)
    router_params = (rng.standard_normal(32 * 32 + 32 * 32 + 16 * 32) * .2).astype(np.float32)
    decoder_params = (rng.standard_normal(32 * 64 + 64 * 64 + 16 * 64) * .1).astype(np.float32)
    rgb = rng.integers(0, 256, (shape[0] * shape[1], 3), dtype=np.uint8)
    ids = rng.integers(0, shape[0] * shape[1], 200)
    ref = oracle.reference_step_experts(rgb, ids, shape, tables, records, stride, experts, router_table, rrecords,
                                        router_params, decoder_params)
    z = ref['logits'].astype(np.float32)[:, :experts]
    assert np.array_equal(ref['expert'], z.argmax(1))
    assert ref['head_grad'].size == 32 * 32 + 32 * 32 + 16 * 32 + 32 * 64 + 64 * 64 + 16 * 64
    touched = np.nonzero(ref['grid_grad'])[0] // stride
    assert set(np.unique(touched)) <= set(np.unique(ref['expert']))
    assert np.isfinite(ref['router_grid_grad']).all() and np.abs(ref['router_grid_grad']).sum() > 0


def test_oracle_allocation_bitmap_hand_case():
    """4 x 4 image, 2 x 2 tiles, only the top-left tile allocated; a level of resolution 3 has cell centres at
    pixel columns/rows 0, 1.5 -> 2 (nearest, halves up) and 3, so only cell (0, 0) lies in the allocated tile."""
    tiles = np.array([[1, 0], [0, 0]], dtype=np.uint8)
    assert np.array_equal(oracle.allocation_bitmap(tiles, 2, 4, 4, 3), np.array([1, 0], dtype=np.uint8))
    assert np.array_equal(oracle.allocation_bitmap(np.ones((2, 2), np.uint8), 2, 4, 4, 3),
                          np.array([255, 1], dtype=np.uint8))


def test_stratified_sampler_restatement_properties():
    """The device sampler's restatement: ids inside the image, one per stratum, offsets spread over the strata."""
    shape, n = (1356, 2040), 1 << 14
    side = 128
    ids = oracle.stratified_ids(5, 9, shape[1], shape[0], n)
    assert ids.min() >= 0 and ids.max() < shape[0] * shape[1]
    j = np.arange(n)
    x, y = ids % shape[1], ids // shape[1]
    fx = (x + 0.5) * side / shape[1] - j % side
    fy = (y + 0.5) * side / shape[0] - j // side
    assert np.all((fx > -0.1) & (fx < 1.1)) and np.all((fy > -0.1) & (fy < 1.1))
    assert abs(fx.mean() - 0.5) < 0.02 and abs(fy.mean() - 0.5) < 0.02
    assert np.array_equal(ids, oracle.stratified_ids(5, 9, shape[1], shape[0], n))
    assert not np.array_equal(ids, oracle.stratified_ids(5, 10, shape[1], shape[0], n))
