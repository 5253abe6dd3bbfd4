"""The single fp32 hash grid's oracle (CPU): its per-coordinate backward against fp64 autograd of the same
network, its uniform sampler and bilinear targets, and the configuration's layout."""
import numpy as np
import torch

from odie_b200.data import blobs_and_gratings
from odie_b200.hashgrid32 import HEAD_PARAMS, c1_config, xavier_heads
from odie_b200.layout import hash_levels
from oracle import oracle


def c1_setup(n=600, grid_scale=0.3, seed=1729):
    config = c1_config(seed=seed)
    records, total = hash_levels(config['hash_encoding'])
    image = blobs_and_gratings(64, 48, seed).numpy()  # a small target keeps the test fast; shape is not special
    grid = ((torch.rand(total, generator=torch.Generator().manual_seed(seed)) * 2 - 1) * grid_scale).numpy()
    heads = xavier_heads(seed + 1).numpy()
    xy = oracle.uniform_xy(seed, 5, n)
    return records, total, image, grid, heads, xy


def test_layout_of_the_configuration():
    """T = 2^19, base 16, scale 1.5: resolutions 16 .. 7007, 10 dense then 6 hashed levels, 7 658 384 entries."""
    records, total = hash_levels(c1_config()['hash_encoding'])
    assert [r['resolution'] for r in records] == [16, 24, 36, 54, 81, 122, 183, 274, 411, 616, 923, 1384, 2076, 3114,
                                                  4671, 7007]
    assert [r['hashed'] for r in records] == [0] * 10 + [1] * 6
    assert total == 7658384 and HEAD_PARAMS == 6336


def test_uniform_coordinates():
    a = oracle.uniform_xy(1729, 0, 4096)
    assert a.dtype == np.float32 and a.shape == (4096, 2)
    assert a.min() >= 0.0 and a.max() < 1.0
    assert np.array_equal(a, oracle.uniform_xy(1729, 0, 4096))
    assert not np.array_equal(a, oracle.uniform_xy(1729, 1, 4096))
    assert np.array_equal(a[:100], oracle.uniform_xy(1729, 0, 100))  # slot i depends on i only
    assert abs(float(a.mean()) - 0.5) < 0.02


def test_bilinear_targets():
    image = np.random.default_rng(0).random((7, 5, 3), dtype=np.float32)
    corners = np.array([[0.0, 0.0], [1.0, 0.0], [0.0, 1.0], [1.0, 1.0]], dtype=np.float32)
    t = oracle.hg32_bilinear(image, corners)
    assert np.array_equal(t, image[[0, 0, 6, 6], [0, 4, 0, 4]])
    xy = np.random.default_rng(1).random((500, 2), dtype=np.float32)
    t = oracle.hg32_bilinear(image, xy)
    px, py = xy[:, 0].astype(np.float64) * 4, xy[:, 1].astype(np.float64) * 6
    x0, y0 = np.minimum(px.astype(int), 3), np.minimum(py.astype(int), 5)
    fx, fy = (px - x0)[:, None], (py - y0)[:, None]
    ref = (image[y0, x0] * (1 - fx) * (1 - fy) + image[y0, x0 + 1] * fx * (1 - fy) + image[y0 + 1, x0] * (1 - fx) * fy
           + image[y0 + 1, x0 + 1] * fx * fy)
    assert np.abs(t - ref).max() < 1e-6


def test_step_backward_against_fp64_autograd():
    """The oracle's fp32 forward/backward (and its fp64 weight and grid gradients) against torch fp64 autograd
    of the same network on the same features and targets: equal to fp32 rounding."""
    records, total, image, grid, heads, xy = c1_setup()
    r = oracle.hg32_step(image, xy, grid, heads, records)
    f = torch.tensor(r['features'], dtype=torch.float64, requires_grad=True)
    w = torch.tensor(heads, dtype=torch.float64, requires_grad=True)
    w1, w2, w3 = w[:2048].view(64, 32), w[2048:6144].view(64, 64), w[6144:].view(3, 64)
    h1 = torch.relu(f @ w1.T)
    h2 = torch.relu(h1 @ w2.T)
    y = torch.sigmoid(h2 @ w3.T)
    t = torch.tensor(r['target'], dtype=torch.float64)
    ((y - t) ** 2).mean().backward()

    def rel(a, b):
        b = np.asarray(b, dtype=np.float64)
        return np.abs(np.asarray(a, dtype=np.float64) - b).max() / np.abs(b).max()
    assert rel(r['h1'], h1.detach()) < 1e-5 and rel(r['h2'], h2.detach()) < 1e-5
    assert rel(r['y'], y.detach()) < 1e-6
    assert rel(r['squares'], ((y - t) ** 2).mean(1).detach()) < 1e-5
    assert rel(r['dx'], f.grad) < 1e-5
    assert rel(r['head_grad'], w.grad) < 1e-5
    assert rel(r['grid_grad'], oracle.hg32_scatter(xy, f.grad.numpy(), records, total)) < 1e-5
    # features: the fma chain of the four corners of every level, restated independently
    idx = np.empty((xy.shape[0], 16, 4), dtype=np.int32)
    wts = np.empty((xy.shape[0], 16, 4), dtype=np.float32)
    oracle.lib().oracle_hash_indices(oracle._p(xy), oracle.C.c_int64(xy.shape[0]), oracle._hash_levels(records), 16,
                                     oracle._p(idx), oracle._p(wts))
    for l, rec in enumerate(records[:3] + records[-2:]):
        level = records.index(rec)
        rows = rec['offset'] + 2 * idx[:, level, :].astype(np.int64)
        expect = (wts[:, level, :].astype(np.float64) * grid[rows].astype(np.float64)).sum(1)
        assert np.abs(r['features'][:, 2 * level] - expect).max() < 1e-6
