"""GPU parity of the gigapixel configuration itself (the benchmark's c4-experts layout), through the C-ABI.

The full model of the benchmark -- 64 routed experts (T = 2^14 per level, 24.4 M parameters, under the
50 MiB fp16 budget), 8 row bands of 8 experts over the 32768 x 32768 procedural image, the 64-logit router,
20 % of the 256 x 256 tiles allocated -- trains one step on a 2^14-coordinate sub-batch drawn as the benchmark
draws its batches, and is checked against the CPU oracle: coordinates, routing decisions, live logits and
encoded features bit-exact; the router probability within 1e-5; network quantities and gradients within 2e-3
per element plus 1e-3 of the tensor's RMS (fp16 network, tensor-core accumulation order); the Adam update of
the expert tables bit-exact given the step's gradient.  The same runs for one rank's share of the model
(bands 4-5 of 8).
"""
import numpy as np
import pytest
import torch

from oracle import oracle
from odie_b200.data import ByteTarget
from odie_b200.model import RoutedExperts
from odie_b200.native_backend import NativeOptimizer
from odie_b200 import workloads
from tests.cases import close, FP16_QUANTUM, close_bound, scatter_bound

pytestmark = pytest.mark.gpu
N = 1 << 14


@pytest.mark.parametrize('band', [(0, 1), (2, 4)])
def test_c4_layout_step_matches_oracle(cuda, band):
    config, rgb, shape = workloads.c4_experts(batch=N, band=band)
    model = RoutedExperts(config)
    assert model.experts == 64 and model.expert_total == 380688 and model.bands == 8
    assert workloads.fp16_payload_bytes(model) <= workloads.C4_BUDGET_BYTES
    full_ty = workloads.C4_SHAPE[0] // workloads.C4_TILE
    rng = np.random.default_rng(31)
    mask = np.zeros(full_ty * full_ty, dtype=np.uint8)
    mask[rng.choice(mask.size, int(round(0.2 * mask.size)), replace=False)] = 1
    tiles = torch.from_numpy(mask.reshape(full_ty, full_ty)).cuda()
    model.set_allocation(tiles, workloads.C4_TILE, workloads.C4_SHAPE)
    opt = NativeOptimizer(model, ByteTarget(rgb), shape, config, [model.grid], batch=N)
    first = config['row_offset'] // workloads.C4_TILE
    local_tiles = tiles[first:first + shape[0] // workloads.C4_TILE].bool()
    ids = workloads.allocated_stratified_ids(local_tiles, shape, N, torch.Generator(device='cuda').manual_seed(5),
                                             tile_px=workloads.C4_TILE)
    snapshot = [t.detach().cpu().numpy().copy() for t in (model.grid, model.router_grid, model.gate.params,
                                                          model.decoder.params)]
    opt.call('step_grads', ids.data_ptr(), N, 2)
    torch.cuda.synchronize()
    assert opt.copied('error_flag', (1,), torch.int32).item() == 0, 'a bounded device wait ran out'
    banding = dict(bands=8, first_band=model.first_band, per_band=8, rows=model.image_rows,
                   row_offset=config['row_offset'])
    ref = oracle.reference_step_experts(None, ids.cpu().numpy(), shape, snapshot[0], model.records,
                                        model.expert_total, model.experts_held, snapshot[1], model.router_records,
                                        snapshot[2], snapshot[3], bitmap=model.allocation_bitmap.cpu().numpy(),
                                        banding=banding, targets=rgb[ids].cpu().numpy())
    cap = opt.pointers['capacity']
    assert np.array_equal(opt.copied('xy', (cap, 2), torch.float32)[:N].cpu().numpy(), ref['xy'])
    expert = opt.copied('expert_ids', (N,), torch.int32).cpu().numpy()
    assert np.array_equal(expert, ref['expert']), 'routing decisions differ'
    assert len(np.unique(ref['band'])) == model.bands_held and len(np.unique(expert)) > model.bands_held
    logits = opt.copied('logits', (cap, opt.pointers['live']), torch.float16)[:N].cpu().numpy()
    assert np.array_equal(logits.view(np.uint16), ref['live_logits'].view(np.uint16)), 'live logits differ'
    close(opt.copied('prob', (N,), torch.float32).cpu().numpy(), ref['prob'], 1e-5, 0.0, 'router probability')
    rows = lambda name: opt.copied(name, (cap, 32), torch.float16)[:N].cpu().numpy()  # noqa: E731
    assert np.array_equal(rows('router_in').view(np.uint16), ref['router_features'].view(np.uint16))
    assert np.array_equal(rows('raw').view(np.uint16), ref['raw'].view(np.uint16)), 'expert features differ'
    fine = [2 * l for l, r in enumerate(model.records) if r.get('cells', -1) >= 0]
    hidden = (ref['raw'][:, fine] == 0).all(1)
    assert fine and hidden.any() and not hidden.all(), 'the batch should reach both allocated and hidden fine cells'
    close(opt.copied('squares', (N,), torch.float32).cpu().numpy(), ref['squares'], 2e-3, 1e-3, 'squares')
    close(rows('gvals').astype(np.float32), ref['values'], 2e-3, 1e-3, 'expert grid values', quantum=FP16_QUANTUM)
    close(rows('router_gvals').astype(np.float32), ref['router_values'], 2e-3, 1e-3, 'router grid values',
          quantum=FP16_QUANTUM)
    heads = opt.copied('head_grad', (opt.pointers['head_count'],), torch.float32).cpu().numpy()
    close(heads, ref['head_grad'], 2e-3, 1e-3, 'router and decoder weight gradients')
    grad = opt.copied('grid_grad', (snapshot[0].size,), torch.float32).cpu().numpy()
    bitmap = model.allocation_bitmap.cpu().numpy()
    experts_backward = lambda up: oracle.expert_backward(ref['xy'], up, ref['expert'], model.expert_total,  # noqa
                                                         model.records, snapshot[0].size, bitmap)
    close_bound(grad, ref['grid_grad'], scatter_bound(experts_backward, ref['values'], 2e-3, 1e-3, FP16_QUANTUM),
                'expert grid gradient')
    router_backward = lambda up: oracle.hash_backward(ref['xy'], up, model.router_records, snapshot[1].size)  # noqa
    close_bound(opt.copied('router_grad', (snapshot[1].size,), torch.float32).cpu().numpy(), ref['router_grid_grad'],
                scatter_bound(router_backward, ref['router_values'], 2e-3, 1e-3, FP16_QUANTUM), 'router grid gradient')
    # the update: bit-exact Adam (zero-gradient entries skipped) given the step's own gradient
    opt.call('grid_update')
    torch.cuda.synchronize()
    p, _, _, steps, _ = oracle.adam(snapshot[0], np.zeros_like(snapshot[0]), np.zeros_like(snapshot[0]),
                                    np.zeros(snapshot[0].size, np.uint32), grad, 128., config['grid_lr'],
                                    skip_zero=True)
    assert np.array_equal(model.grid.detach().cpu().numpy(), p), 'expert table update differs'
    opt.close()
