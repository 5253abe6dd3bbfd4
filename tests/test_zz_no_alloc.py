"""GPU test of odie_tile_topk_noalloc, the allocation-free tile top-k entry point.

It keeps its row sums in a fixed array inside the library instead of a caller
buffer.  Two calls in a row on different images (the second one smaller, so the
array still holds the first call's larger row-sum range) must each match
odie_tile_topk on the same inputs, bit for bit: both run the same kernels, and
every row sum the second call reads is one it wrote itself.  The file name puts
it last in collection, so it runs both after the other GPU tests and alone.
"""
import numpy as np
import pytest
import torch

from odie_b200 import _lib

pytestmark = pytest.mark.gpu
MAX_ROW_SUMS = 1 << 18


def inputs(seed, h, w):
    rng = np.random.default_rng(seed)
    pred = torch.from_numpy(rng.random((h * w, 3), dtype=np.float32)).cuda()
    u8 = torch.from_numpy(rng.integers(0, 256, (h * w, 3), dtype=np.uint8)).cuda()
    return pred, u8


def outputs(tiles, k):
    return (torch.full((tiles,), float('nan'), dtype=torch.float64, device='cuda'),
            torch.full((k,), -1, dtype=torch.int64, device='cuda'),
            torch.full((tiles,), 7, dtype=torch.uint8, device='cuda'))


def run(noalloc, pred, u8, h, w, tile, k):
    lib, stream = _lib.library(), torch.cuda.current_stream().cuda_stream
    tiles = ((w + tile - 1) // tile) * ((h + tile - 1) // tile)
    scores, chosen, selected = outputs(tiles, k)
    if noalloc:
        _lib.check(lib.odie_tile_topk_noalloc(pred.data_ptr(), u8.data_ptr(), h, w, tile, k, scores.data_ptr(),
                                              chosen.data_ptr(), selected.data_ptr(), stream))
    else:
        row_sums = torch.empty(tiles * tile, dtype=torch.float64, device='cuda')
        _lib.check(lib.odie_tile_topk(pred.data_ptr(), u8.data_ptr(), h, w, tile, k, row_sums.data_ptr(),
                                      scores.data_ptr(), chosen.data_ptr(), selected.data_ptr(), stream))
    torch.cuda.synchronize()
    return scores.cpu().numpy(), chosen.cpu().numpy(), selected.cpu().numpy()


def test_noalloc_matches_tile_topk_twice_in_a_row(cuda):
    # first call: 12 x 11 tiles of 64 rows = 8448 row sums; second: 7 x 5 tiles of 48 rows
    for seed, (h, w, tile, k) in ((31, (700, 760, 64, 40)), (32, (231, 320, 48, 9))):
        pred, u8 = inputs(seed, h, w)
        expected = run(False, pred, u8, h, w, tile, k)
        got = run(True, pred, u8, h, w, tile, k)
        assert np.isfinite(got[0]).all()
        assert np.array_equal(got[0], expected[0]), 'tile scores differ'
        assert np.array_equal(got[1], expected[1]), 'chosen tiles differ'
        assert np.array_equal(got[2], expected[2]), 'selection mask differs'
        assert got[2].sum() == k


def test_noalloc_full_scratch_and_rejects_oversize(cuda):
    lib, stream = _lib.library(), torch.cuda.current_stream().cuda_stream
    # exactly the limit: 64 x 64 tiles of 64 rows = 262144 row sums
    h = w = 4096
    pred, u8 = inputs(33, h, w)
    expected = run(False, pred, u8, h, w, 64, 100)
    got = run(True, pred, u8, h, w, 64, 100)
    for a, b in zip(got, expected):
        assert np.array_equal(a, b)
    # one more tile row is rejected before anything is launched
    scores, chosen, selected = outputs(65 * 64, 1)
    status = lib.odie_tile_topk_noalloc(pred.data_ptr(), u8.data_ptr(), h + 1, w, 64, 1, scores.data_ptr(),
                                        chosen.data_ptr(), selected.data_ptr(), stream)
    assert status != 0
    assert 'exceed' in _lib.error() and str(MAX_ROW_SUMS) in _lib.error()
    torch.cuda.synchronize()
    assert torch.isnan(scores).all(), 'a rejected call must not write its outputs'
