"""GPU parity of the on-demand allocation of routed experts (the allocation benchmark).

Tile residuals and the top-k tile selection are bit-exact (tests/test_gpu_selection.py);
here: the per-level cell-visibility bitmaps built from the allocated tiles, the
expert gathers and scatters restricted to visible cells, and a full routed
training step with allocation, all against the CPU oracle.
"""
import numpy as np
import pytest
import torch

from oracle import oracle
from odie_b200 import _lib
from odie_b200.layout import hash_levels
from odie_b200.model import ExpertHashQuery, _hash_table, _stream
from tests.cases import close, close_bound, scatter_bound, FP16_QUANTUM
from tests.test_gpu_experts import SHAPE, read_rows, setup

pytestmark = pytest.mark.gpu


def device_bitmap(tiles, tile_px, height, width, res):
    t = torch.from_numpy(tiles.astype(np.uint8)).cuda()
    out = torch.zeros((res * res + 7) // 8, dtype=torch.uint8, device='cuda')
    _lib.check(_lib.library().odie_allocation_bitmap(t.data_ptr(), tiles.shape[1], tiles.shape[0], tile_px, height,
                                                     width, res, out.data_ptr(), _stream()))
    torch.cuda.synchronize()
    return out.cpu().numpy()


@pytest.mark.parametrize('height,width,tile_px', [(4096, 4096, 256), (61, 47, 8), (1356, 2040, 256), (5, 300, 64)])
def test_allocation_bitmap_matches_oracle(cuda, height, width, tile_px):
    rng = np.random.default_rng(height + width)
    tiles = rng.random((-(-height // tile_px), -(-width // tile_px))) < 0.3
    for res in (2, 3, 17, 36, 274, 1001):
        got = device_bitmap(tiles, tile_px, height, width, res)
        want = oracle.allocation_bitmap(tiles, tile_px, height, width, res)
        assert np.array_equal(got, want), f'res {res}'
    assert device_bitmap(np.ones_like(tiles), tile_px, height, width, 33).sum() > 0


def allocated_records(records, tiles, tile_px, shape, dense=9):
    out, bitmaps, offset = [], [], 0
    for r in records:
        r = dict(r)
        if r['resolution'] > dense:
            r['cells'] = offset
            b = oracle.allocation_bitmap(tiles, tile_px, shape[0], shape[1], r['resolution'])
            bitmaps.append(b)
            offset += b.size
        out.append(r)
    return out, np.concatenate(bitmaps) if bitmaps else np.zeros(1, np.uint8)


def test_expert_queries_touch_only_allocated_cells(cuda):
    rng = np.random.default_rng(3)
    encoding = dict(n_levels=16, n_features_per_level=2, log2_hashmap_size=10, base_resolution=4, per_level_scale=1.5)
    records, stride = hash_levels(encoding)
    tiles = rng.random((4, 4)) < 0.4
    records, bitmap = allocated_records(records, tiles, 16, (61, 61))
    experts, n = 3, 2500
    tables = (rng.standard_normal(experts * stride) * 0.1).astype(np.float32)
    xy = rng.random((n, 2), dtype=np.float32)
    xy[:4] = [[0, 0], [1, 1], [0, 1], [1, 0]]
    expert = rng.integers(0, experts, n).astype(np.int32)
    xy_d, tables_d, expert_d = (torch.from_numpy(a).cuda() for a in (xy, tables, expert))
    bitmap_d = torch.from_numpy(bitmap).cuda()
    features = ExpertHashQuery.apply(xy_d, tables_d, expert_d, stride, records, 32, bitmap_d)
    torch.cuda.synchronize()
    want = oracle.expert_query(xy, tables.astype(np.float16), expert, stride, records, 32, bitmap)
    assert np.array_equal(features.cpu().numpy().view(np.uint16), want.view(np.uint16))
    assert (want[:, 20:] == 0).any(), 'the case should hide some fine cells'
    upstream = (rng.standard_normal((n, 32)) * 0.01).astype(np.float16)
    up_d = torch.from_numpy(upstream).cuda()
    grad = torch.empty(tables.size, dtype=torch.float32, device='cuda')
    _lib.check(_lib.library().odie_expert_hash_backward(xy_d.data_ptr(), n, up_d.data_ptr(), 32, stride,
                                                        expert_d.data_ptr(), _hash_table(records), len(records),
                                                        bitmap_d.data_ptr(), grad.data_ptr(), tables.size, _stream()))
    torch.cuda.synchronize()
    backward = lambda up: oracle.expert_backward(xy, up, expert, stride, records, tables.size, bitmap)  # noqa
    close_bound(grad.cpu().numpy(), backward(upstream), scatter_bound(backward, upstream), 'allocated expert scatter')


def test_routed_step_with_allocation_matches_oracle(cuda):
    config, model, rgb, opt = setup(experts=4)
    opt.close()
    rng = np.random.default_rng(6)
    tiles = rng.random((4, 3)) < 0.5
    model.set_allocation(torch.from_numpy(tiles), 16, SHAPE)
    from odie_b200.data import ByteTarget
    from odie_b200.native_backend import NativeOptimizer
    opt = NativeOptimizer(model, ByteTarget(torch.from_numpy(rgb).cuda()), SHAPE, config, [model.grid], batch=1024)
    n = 1000
    ids = torch.from_numpy(np.sort(rng.integers(0, SHAPE[0] * SHAPE[1], n))).cuda()
    snap = [t.detach().cpu().numpy().copy() for t in (model.grid, model.router_grid, model.gate.params,
                                                      model.decoder.params)]
    opt.call('step_grads', ids.data_ptr(), n, 2)
    torch.cuda.synchronize()
    bitmap = model.allocation_bitmap.cpu().numpy()
    ref = oracle.reference_step_experts(rgb, ids.cpu().numpy(), SHAPE, snap[0], model.records, model.expert_total, 4,
                                        snap[1], model.router_records, snap[2], snap[3], bitmap=bitmap)
    W = opt.pointers['input_width']
    assert np.array_equal(opt.copied('expert_ids', (n,), torch.int32).cpu().numpy(), ref['expert'])
    raw = read_rows(opt, 'raw', n, W)
    assert np.array_equal(raw.view(np.uint16), ref['raw'].view(np.uint16)), 'allocated expert features differ'
    close(opt.copied('squares', (n,), torch.float32).cpu().numpy(), ref['squares'], 2e-3, 1e-3, 'squares')
    grad = opt.copied('grid_grad', (snap[0].size,), torch.float32).cpu().numpy()
    backward = lambda up: oracle.expert_backward(ref['xy'], up, ref['expert'], model.expert_total,  # noqa: E731
                                                 model.records, snap[0].size, bitmap)
    close_bound(grad, ref['grid_grad'], scatter_bound(backward, ref['values'], 2e-3, 1e-3, FP16_QUANTUM),
                'allocated expert grid gradient')
    hidden = np.nonzero(ref['grid_grad'] == 0)[0]
    assert np.all(grad[hidden] == 0), 'a hidden cell received a gradient'
    opt.close()
