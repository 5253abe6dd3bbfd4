"""GPU parity of live residual scoring (a17), exact greedy selection (a18) and tile top-k.

All bit-exact: against the reference's own CPU outputs (golden vectors), the
C oracle, and the reference's own CUDA selection/residual kernels compiled
from source (oracle/_ref).
"""
import ctypes as C
from pathlib import Path

import numpy as np
import pytest
import torch

from oracle import oracle
from odie_b200 import _lib
from odie_b200 import selection as host
from odie_b200.gpu_residual import ResidualAccumulator, select_device, select_live

pytestmark = pytest.mark.gpu
ROOT = Path(__file__).resolve().parents[1]


def greedy_cases(g):
    keys = sorted({k.rsplit('_scores', 1)[0] for k in g if k.endswith('_scores')})
    for key in keys:
        parts = key.split('_')
        yield key, int(parts[-2][1:]), int(parts[-1][1:])


def test_greedy_matches_reference_golden(cuda, golden):
    g = golden('greedy.npz')
    for key, r, cap in greedy_cases(g):
        scores = torch.from_numpy(np.abs(g[f'{key}_scores']) * 0 + g[f'{key}_scores']).cuda()
        for tag, normalized in (('B2', True), ('E', False)):
            support, record = select_device(scores, r * r, r, cap, normalized=normalized, chunk=7)
            assert np.array_equal(support, g[f'{key}_{tag}_selected'].astype(bool)), (key, tag)
            assert record['iterations'] == int(g[f'{key}_{tag}_iterations']), (key, tag)


@pytest.mark.parametrize('r,frac', [(128, .2), (300, .05)])
def test_greedy_large_vs_oracle(cuda, r, frac):
    rng = np.random.default_rng(r)
    scores = rng.random(r * r) ** 4
    scores[rng.random(r * r) < .2] = 0.
    scores[::17] = scores[::17].round(2)  # ties
    cap = int(host.align8(r * r) * frac) // 8 * 8
    chosen, nodes, iterations, used = oracle.select_benefit_cost(scores, r, cap, True)
    support, record = select_device(torch.from_numpy(scores).cuda(), r * r, r, cap)
    assert np.array_equal(support, chosen)
    assert record['iterations'] == iterations and record['closure_nodes'] == used


def test_greedy_trace_records_order(cuda):
    rng = np.random.default_rng(1)
    r, cap = 32, 256
    scores = rng.random(r * r)
    trace = torch.full((r * r,), -1, dtype=torch.int32, device='cuda')
    support, record = select_device(torch.from_numpy(scores).cuda(), r * r, r, cap, trace=trace)
    order = trace[:record['iterations']].cpu().numpy()
    assert len(set(order.tolist())) == record['iterations'] and support[order].all()


def reference_selection():
    path = ROOT / 'oracle' / '_ref' / 'libref_selection.so'
    if not path.exists():
        pytest.skip('reference GPU oracle (oracle/_ref) was not built')
    lib = C.CDLL(str(path))
    p, i = C.c_void_p, C.c_int
    lib.selection_init.argtypes = [p, i, i, p, p, p, p, p, p, p, i, C.c_uint64]
    lib.selection_chunk.argtypes = [p, i, i, i, i, C.c_bool, p, p, p, p, p, p, i, i, p, p, C.c_uint64]
    return lib


def test_greedy_matches_reference_kernel(cuda):
    """Same buffers, same calls: the reference's selection kernels and ours choose the same cells in the same order."""
    ref = reference_selection()
    rng = np.random.default_rng(9)
    r, cap = 96, 1600
    n, points = r * r, host.align8(r * r)
    scores = torch.from_numpy(rng.random(n) ** 3).cuda()
    sizes, offsets, tree_size = host.tree_shape(n)
    results = []
    for lib in (ref, _lib.library()):
        missing = torch.empty(n, dtype=torch.int32, device='cuda')
        chosen = torch.empty(n, dtype=torch.uint8, device='cuda')
        nodes = torch.empty(points, dtype=torch.uint8, device='cuda')
        tree = torch.empty(tree_size, dtype=torch.int32, device='cuda')
        stats = torch.zeros(4, dtype=torch.int64, device='cuda')
        trace = torch.full((n,), -1, dtype=torch.int32, device='cuda')
        do, ds = torch.from_numpy(offsets).cuda(), torch.from_numpy(sizes).cuda()
        stream = torch.cuda.current_stream().cuda_stream
        assert lib.selection_init(scores.data_ptr(), n, points, missing.data_ptr(), chosen.data_ptr(), nodes.data_ptr(),
                                  tree.data_ptr(), stats.data_ptr(), offsets.ctypes.data, sizes.ctypes.data,
                                  len(sizes), stream) == 0
        for _ in range(n // 512 + 2):
            assert lib.selection_chunk(scores.data_ptr(), n, points, r, cap, True, missing.data_ptr(), chosen.data_ptr(),
                                       nodes.data_ptr(), tree.data_ptr(), do.data_ptr(), ds.data_ptr(), len(sizes), 512,
                                       stats.data_ptr(), trace.data_ptr(), stream) == 0
            if stats[2].item():
                break
        results.append((chosen.cpu().numpy(), nodes.cpu().numpy(), stats.cpu().numpy(), trace.cpu().numpy()))
    (c0, n0, s0, t0), (c1, n1, s1, t1) = results
    assert s0[2] == 1 and s1[2] == 1 and s0[3] == 0 and s1[3] == 0
    assert np.array_equal(c0, c1) and np.array_equal(n0, n1) and np.array_equal(s0[:2], s1[:2])
    assert np.array_equal(t0[:s0[1]], t1[:s1[1]])


@pytest.mark.parametrize('key', ['37x53_8', '64x48_13', '101x77_100'])
def test_score_chunk_matches_reference_golden(cuda, golden, key):
    g = golden('residual.npz')
    pred, u8, total = g[f'res_pred_{key}'], g[f'res_u8_{key}'], g[f'res_total_{key}']
    h, w = map(int, key.split('_')[0].split('x'))
    r = int(key.split('_')[1])
    scores = ResidualAccumulator((h, w), r)
    pred_d, u8_d = torch.from_numpy(pred).cuda(), torch.from_numpy(u8).cuda()
    for begin in range(0, h * w, 997):
        end = min(begin + 997, h * w)
        scores.accumulate(pred_d[begin:end], u8_d[begin:end], begin)
    assert np.array_equal(scores.totals.cpu().numpy(), total)
    assert np.array_equal(scores.counts, g[f'res_counts_{key}'])


def test_score_chunk_fp32_target(cuda):
    rng = np.random.default_rng(3)
    h, w, r = 40, 60, 17
    pred = rng.random((h * w, 3), dtype=np.float32)
    target = rng.random((h * w, 3), dtype=np.float32)
    scores = ResidualAccumulator((h, w), r)
    scores.accumulate(torch.from_numpy(pred).cuda(), torch.from_numpy(target).cuda(), 0)
    expected = np.zeros(r * r)
    oracle.score_chunk(pred, target, 0, h * w, w, r, 0, r * r, scores.x_edges.cpu().numpy(),
                       scores.y_edges.cpu().numpy(), expected, False)
    assert np.array_equal(scores.totals.cpu().numpy(), expected)


def test_tile_topk_bit_exact(cuda):
    rng = np.random.default_rng(12)
    h, w, tile, k = 520, 700, 64, 30
    pred = rng.random((h * w, 3), dtype=np.float32)
    u8 = rng.integers(0, 256, (h * w, 3), dtype=np.uint8)
    tiles = ((w + tile - 1) // tile) * ((h + tile - 1) // tile)
    row_sums = torch.empty(tiles * tile, dtype=torch.float64, device='cuda')
    scores = torch.empty(tiles, dtype=torch.float64, device='cuda')
    chosen = torch.empty(k, dtype=torch.int64, device='cuda')
    selected = torch.empty(tiles, dtype=torch.uint8, device='cuda')
    pred_d, u8_d = torch.from_numpy(pred).cuda(), torch.from_numpy(u8).cuda()  # keep both alive during the call
    _lib.check(_lib.library().odie_tile_topk(pred_d.data_ptr(), u8_d.data_ptr(), h, w, tile, k,
                                             row_sums.data_ptr(), scores.data_ptr(), chosen.data_ptr(),
                                             selected.data_ptr(), torch.cuda.current_stream().cuda_stream))
    torch.cuda.synchronize()
    expected = oracle.tile_scores(pred, u8, h, w, tile)
    assert np.array_equal(scores.cpu().numpy(), expected)
    assert np.array_equal(chosen.cpu().numpy(), oracle.topk(expected, k))
    assert selected.sum().item() == k


def test_select_live_through_fused_decode(cuda):
    """The stage boundary on a packed-plane model with its training runtime attached: the whole image decodes
    through odie_decode in chunks, the residual totals equal the C oracle's over those very predictions bit for
    bit, and the chosen support is the oracle's exact B2 greedy on them; the module path (no runtime) chooses
    from its own predictions, within the fp16 tolerance of the fused ones."""
    from odie_b200.data import ByteTarget
    from odie_b200.model import PackedXYPlanes
    from odie_b200.native_backend import NativeOptimizer
    from tests.cases import close, plane_case, plane_config, random_image
    shape = (97, 131)
    resolutions, dims, supports, caps = plane_case(17, dense=10, packed=4, finest=64)
    config = plane_config(resolutions, dims, 10, seed=17)
    model = PackedXYPlanes(config, supports, dims, caps)
    rgb = random_image(*shape, 17)
    target = ByteTarget(torch.from_numpy(rgb).cuda())
    planes = [torch.nn.Parameter(model.grid[l['plane_offset']:l['plane_offset'] + l['plane_node_capacity'] *
                                            l['plane_dim']].detach()) for l in model.layout['levels']]
    opt = NativeOptimizer(model, target, shape, config, planes, batch=2048)
    ids = torch.randint(0, shape[0] * shape[1], (2048,), device='cuda', generator=torch.Generator('cuda').manual_seed(1))
    for _ in range(5):
        opt.train_batch(ids)
    opt.call('sync_weights')
    r, cap = resolutions[10], caps[10]  # the next level a stage boundary would open
    metrics, support, record, counts, timing, totals = select_live(model, target, shape, r, cap, 2, 1000,
                                                                   validate_scores=True)
    assert timing['decode_path'] == 'fused odie_decode'
    prediction = torch.empty((shape[0] * shape[1], 3), device='cuda')
    opt.decode(0, shape[0] * shape[1], rgb=prediction)
    torch.cuda.synchronize()
    boxes = ResidualAccumulator(shape, r)
    expected = np.zeros(r * r)
    oracle.score_chunk(prediction.cpu().numpy(), rgb, 0, shape[0] * shape[1], shape[1], r, 0, r * r,
                       boxes.x_edges.cpu().numpy(), boxes.y_edges.cpu().numpy(), expected, True)
    assert np.array_equal(totals, expected), 'live residual totals differ from the oracle on the fused predictions'
    chosen, nodes, iterations, used = oracle.select_benefit_cost(expected, r, cap)
    assert np.array_equal(support, chosen) and record['iterations'] == iterations and record['closure_nodes'] == used
    assert np.isfinite(metrics['mse']) and metrics['mse'] > 0
    # the module path (no runtime attached) on the same weights: its totals are the oracle's on its own predictions,
    # and those predictions are the fused ones within the fp16 decode tolerance
    model._odie_runtime = None
    metrics_m, support_m, _, _, timing_m, totals_m = select_live(model, target, shape, r, cap, 2, 1000,
                                                                 validate_scores=True)
    assert timing_m['decode_path'] == 'module forward'
    with torch.no_grad():
        from odie_b200.evaluation import coordinates
        module = model(coordinates(shape, torch.arange(shape[0] * shape[1], device='cuda'))).float()
    expected_m = np.zeros(r * r)
    oracle.score_chunk(module.cpu().numpy(), rgb, 0, shape[0] * shape[1], shape[1], r, 0, r * r,
                       boxes.x_edges.cpu().numpy(), boxes.y_edges.cpu().numpy(), expected_m, True)
    assert np.array_equal(totals_m, expected_m), 'module-path totals differ from the oracle on its own predictions'
    close(module.cpu().numpy(), prediction.cpu().numpy(), 2e-3, 1e-3, 'module vs fused predictions')
    opt.close()
