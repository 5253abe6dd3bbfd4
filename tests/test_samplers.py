"""Batch samplers of the benchmark workloads (host logic, CPU): the reference's stratified sampler
(odie/data.py:63-80) and the allocated-tile samplers of the on-demand allocation workload."""
import pytest
import torch

from odie_b200.data import stratified_batches
from odie_b200.workloads import allocated_ids, allocated_stratified_ids


def test_stratified_batches_one_sample_per_stratum():
    g = torch.Generator().manual_seed(0)
    shape, batch = (64, 96), 256
    ids = next(stratified_batches(shape, batch, g, device='cpu', steps=1))
    y, x = ids // shape[1], ids % shape[1]
    side = 16
    sx, sy = (x * side) // shape[1], (y * side) // shape[0]
    assert torch.equal(sy * side + sx, torch.arange(batch))
    with pytest.raises(ValueError):
        next(stratified_batches(shape, 200, g, device='cpu'))


@pytest.mark.parametrize('shape,grid,count', [((4096, 4096), (16, 16), 1 << 16), ((1356, 2040), (6, 8), 5000),
                                              ((300, 5), (2, 1), 77)])
def test_allocated_samplers_share_the_distribution(shape, grid, count):
    g = torch.Generator().manual_seed(sum(shape))
    tiles = torch.rand(grid, generator=g) < 0.4
    tiles.view(-1)[0] = True
    tile_px = -(-max(shape) // max(grid))
    for sampler in (allocated_ids, allocated_stratified_ids):
        ids = sampler(tiles, shape, count, g, tile_px=tile_px)
        assert ids.shape == (count,) and ids.dtype == torch.long
        assert int(ids.min()) >= 0 and int(ids.max()) < shape[0] * shape[1]
    ids = allocated_stratified_ids(tiles, shape, count, g, tile_px=tile_px)
    inside = int(round(count * 0.7))
    y, x = ids // shape[1], ids % shape[1]
    ty, tx = (y // tile_px).clamp(max=grid[0] - 1), (x // tile_px).clamp(max=grid[1] - 1)
    assert bool(tiles[ty[:inside], tx[:inside]].all()), 'the allocated share must land in allocated tiles'
    counts = torch.bincount((ty[:inside] * grid[1] + tx[:inside]), minlength=grid[0] * grid[1])[tiles.reshape(-1)]
    assert int(counts.max() - counts.min()) <= 1, 'the allocated share is spread evenly over the tiles'


def test_allocated_stratified_covers_each_stratum():
    g = torch.Generator().manual_seed(5)
    tiles = torch.ones((1, 1), dtype=torch.bool)
    ids = allocated_stratified_ids(tiles, (64, 64), 16 * 16, g, fraction=1.0, tile_px=64)
    y, x = ids // 64, ids % 64
    assert torch.equal((y // 4) * 16 + x // 4, torch.arange(256))
