"""GPU parity of the benchmark's other configurations, built exactly as bench.py builds them (odie_b200/workloads.py):
c2-experts (16 routed experts, T = 2^16, the 2040 x 1356 image), c3-experts (8 experts, T = 2^17, the 4096 x 4096
image, 30 % of the 256 x 256 tiles allocated) and c2-planes (the reference's packed planes with the DIV2K plan and
its three on-demand levels), each training one step on a 2^14-coordinate sub-batch drawn as the benchmark draws its
batches, through the C-ABI, against the CPU oracle.

Criteria as in test_gpu_c4.py: coordinates, visibility, routing, live logits and encoded features bit-exact; network
quantities and gradients within 2e-3 per element plus 1e-3 of the tensor's RMS; grid gradients within the fp32
summation bound of their terms plus the values' own tolerance; the grid's Adam update bit-exact given the step's
gradient.
"""
import numpy as np
import pytest
import torch

from oracle import oracle
from odie_b200 import workloads
from odie_b200.data import ByteTarget, stratified_batches
from odie_b200.model import RoutedExperts
from odie_b200.native_backend import NativeOptimizer
from tests.cases import FP16_QUANTUM, close, close_bound, layout_numpy, scatter_bound

pytestmark = pytest.mark.gpu
N = 1 << 14


def check_adam(opt, model, grid0, grad, lr):
    opt.call('grid_update')
    torch.cuda.synchronize()
    p, *_ = oracle.adam(grid0, np.zeros_like(grid0), np.zeros_like(grid0), np.zeros(grid0.size, np.uint32), grad, 128.,
                        lr, skip_zero=True)
    assert np.array_equal(model.grid.detach().cpu().numpy(), p), 'grid update differs'


@pytest.mark.parametrize('name', ['c2-experts', 'c3-experts'])
def test_expert_config_step_matches_oracle(cuda, name):
    if name == 'c2-experts':
        config, rgb, shape = workloads.c2_experts(batch=N)
    else:
        config, rgb, shape = workloads.c3_experts(batch=N)
    model = RoutedExperts(config)
    bitmap = None
    generator = torch.Generator(device='cuda').manual_seed(9)
    if name == 'c3-experts':
        ty, tx = shape[0] // workloads.C3_TILE, shape[1] // workloads.C3_TILE
        rng = np.random.default_rng(13)
        mask = np.zeros(ty * tx, dtype=np.uint8)
        mask[rng.choice(mask.size, int(round(0.3 * mask.size)), replace=False)] = 1
        tiles = torch.from_numpy(mask.reshape(ty, tx)).cuda()
        model.set_allocation(tiles, workloads.C3_TILE, shape)
        bitmap = model.allocation_bitmap.cpu().numpy()
        ids = workloads.allocated_stratified_ids(tiles.bool(), shape, N, generator, tile_px=workloads.C3_TILE)
    else:
        ids = next(stratified_batches(shape, N, generator, steps=1))
    rgb = rgb.cuda()
    opt = NativeOptimizer(model, ByteTarget(rgb), shape, config, [model.grid], batch=N)
    snapshot = [t.detach().cpu().numpy().copy() for t in (model.grid, model.router_grid, model.gate.params,
                                                          model.decoder.params)]
    opt.call('step_grads', ids.data_ptr(), N, 2)
    torch.cuda.synchronize()
    assert opt.copied('error_flag', (1,), torch.int32).item() == 0, 'a bounded device wait ran out'
    ref = oracle.reference_step_experts(None, ids.cpu().numpy(), shape, snapshot[0], model.records,
                                        model.expert_total, model.experts_held, snapshot[1], model.router_records,
                                        snapshot[2], snapshot[3], bitmap=bitmap, targets=rgb[ids].cpu().numpy())
    cap = opt.pointers['capacity']
    assert np.array_equal(opt.copied('xy', (cap, 2), torch.float32)[:N].cpu().numpy(), ref['xy'])
    expert = opt.copied('expert_ids', (N,), torch.int32).cpu().numpy()
    assert np.array_equal(expert, ref['expert']), 'routing decisions differ'
    assert len(np.unique(expert)) > 1, 'the batch should reach several experts'
    logits = opt.copied('logits', (cap, opt.pointers['live']), torch.float16)[:N].cpu().numpy()
    assert np.array_equal(logits.view(np.uint16), ref['live_logits'].view(np.uint16)), 'live logits differ'
    close(opt.copied('prob', (N,), torch.float32).cpu().numpy(), ref['prob'], 1e-5, 0.0, 'router probability')
    rows = lambda key: opt.copied(key, (cap, 32), torch.float16)[:N].cpu().numpy()  # noqa: E731
    assert np.array_equal(rows('router_in').view(np.uint16), ref['router_features'].view(np.uint16))
    assert np.array_equal(rows('raw').view(np.uint16), ref['raw'].view(np.uint16)), 'expert features differ'
    close(opt.copied('squares', (N,), torch.float32).cpu().numpy(), ref['squares'], 2e-3, 1e-3, 'squares')
    close(rows('gvals').astype(np.float32), ref['values'], 2e-3, 1e-3, 'expert grid values', quantum=FP16_QUANTUM)
    close(rows('router_gvals').astype(np.float32), ref['router_values'], 2e-3, 1e-3, 'router grid values',
          quantum=FP16_QUANTUM)
    close(opt.copied('head_grad', (opt.pointers['head_count'],), torch.float32).cpu().numpy(), ref['head_grad'],
          2e-3, 1e-3, 'router and decoder weight gradients')
    grad = opt.copied('grid_grad', (snapshot[0].size,), torch.float32).cpu().numpy()
    backward = lambda up: oracle.expert_backward(ref['xy'], up, ref['expert'], model.expert_total,  # noqa: E731
                                                 model.records, snapshot[0].size, bitmap)
    close_bound(grad, ref['grid_grad'], scatter_bound(backward, ref['values'], 2e-3, 1e-3, FP16_QUANTUM),
                'expert grid gradient')
    router_backward = lambda up: oracle.hash_backward(ref['xy'], up, model.router_records, snapshot[1].size)  # noqa
    close_bound(opt.copied('router_grad', (snapshot[1].size,), torch.float32).cpu().numpy(), ref['router_grid_grad'],
                scatter_bound(router_backward, ref['router_values'], 2e-3, 1e-3, FP16_QUANTUM), 'router grid gradient')
    check_adam(opt, model, snapshot[0], grad, config['grid_lr'])
    opt.close()


def test_c2_planes_step_matches_oracle(cuda):
    config, supports, dims, caps, rgb, shape = workloads.c2_planes(batch=N)
    model, target, planes = workloads.build_plane_model(config, supports, dims, caps, rgb)
    opt = NativeOptimizer(model, target, shape, config, planes, batch=N)
    grid = model.grid.detach().cpu().numpy().copy()
    gate = model.gate.params.detach().cpu().numpy().copy()
    dec = model.decoder.params.detach().cpu().numpy().copy()
    ids = next(stratified_batches(shape, N, torch.Generator(device='cuda').manual_seed(10), steps=1))
    opt.call('step_grads', ids.data_ptr(), N, 2)
    torch.cuda.synchronize()
    assert opt.copied('error_flag', (1,), torch.int32).item() == 0, 'a bounded device wait ran out'
    lay = layout_numpy({k: getattr(model, k).cpu() for k in ('descriptors', 'node_bitmap', 'node_prefix', 'bitmap')})
    ref = oracle.reference_step(rgb.numpy(), ids.cpu().numpy(), shape, grid, lay, gate, dec, model.n_levels,
                                model.input_width, active=model.active_prefix)
    cap = opt.pointers['capacity']
    width = opt.pointers['input_width']
    assert np.array_equal(opt.copied('xy', (cap, 2), torch.float32)[:N].cpu().numpy(), ref['xy'])
    words = opt.copied('vis', (model.n_levels, cap // 32), torch.int32).cpu().numpy().view(np.uint32)
    vis = np.unpackbits(words.view(np.uint8), axis=1, bitorder='little')[:, :N].T
    assert np.array_equal(vis, ref['vis']), 'visibility differs'
    pairs = opt.copied('raw', (width // 2, cap, 2), torch.float16)[:, :N, :]
    raw = pairs.permute(1, 0, 2).reshape(N, width).cpu().numpy()
    assert np.array_equal(raw.view(np.uint16), ref['raw'].view(np.uint16)), 'encoded features differ'
    close(opt.copied('squares', (N,), torch.float32).cpu().numpy(), ref['squares'], 2e-3, 1e-3, 'squares')
    values = opt.copied('gvals', (cap, width), torch.float16)[:N].cpu().numpy()
    close(values.astype(np.float32), ref['values'], 2e-3, 1e-3, 'grid-gradient values', quantum=FP16_QUANTUM)
    close(opt.copied('head_grad', (opt.pointers['head_count'],), torch.float32).cpu().numpy(), ref['head_grad'],
          2e-3, 1e-3, 'head gradients')
    grad = opt.copied('grid_grad', (grid.size,), torch.float32).cpu().numpy()
    backward = lambda up: oracle.query_backward(ref['xy'], up, lay['descriptors'], lay['node_bitmap'],  # noqa: E731
                                                lay['node_prefix'], lay['bitmap'], grid.size)
    close_bound(grad, ref['grid_grad'], scatter_bound(backward, ref['values'], 2e-3, 1e-3, FP16_QUANTUM),
                'grid gradient')
    check_adam(opt, model, grid, grad, config['grid_lr'])
    opt.close()


@pytest.mark.parametrize('batch', ['coherent', 'uniform'])
def test_router_scatter_strategy_matches_oracle(cuda, batch):
    """The router-grid scatter chooses its strategy from the batch on the device: a raster-ordered 128 x 128 block
    of pixels (consecutive coordinates share cells) takes global reductions (strategy 1), uniform pixel ids the
    per-block shared-memory tables (strategy 0).  Either way the router grid gradient matches the oracle within the
    fp32 summation bound."""
    config, rgb, shape = workloads.c2_experts(batch=N)
    model = RoutedExperts(config)
    height, width = shape
    if batch == 'coherent':
        ys, xs = torch.meshgrid(torch.arange(128) + 300, torch.arange(128) + 700, indexing='ij')
        ids = (ys * width + xs).reshape(-1).cuda()
    else:
        ids = torch.randint(0, height * width, (N,), generator=torch.Generator().manual_seed(5)).cuda()
    rgb = rgb.cuda()
    opt = NativeOptimizer(model, ByteTarget(rgb), shape, config, [model.grid], batch=N)
    snapshot = [t.detach().cpu().numpy().copy() for t in (model.grid, model.router_grid, model.gate.params,
                                                          model.decoder.params)]
    opt.call('step_grads', ids.data_ptr(), N, 2)
    torch.cuda.synchronize()
    assert opt.copied('error_flag', (1,), torch.int32).item() == 0, 'a bounded device wait ran out'
    strategy = int(opt.copied('scatter_strategy', (2,), torch.int32)[0])
    assert strategy == (1 if batch == 'coherent' else 0), f'router scatter strategy {strategy}'
    ref = oracle.reference_step_experts(None, ids.cpu().numpy(), shape, snapshot[0], model.records,
                                        model.expert_total, model.experts_held, snapshot[1], model.router_records,
                                        snapshot[2], snapshot[3], targets=rgb[ids].cpu().numpy())
    cap = opt.pointers['capacity']
    rows = opt.copied('router_gvals', (cap, 32), torch.float16)[:N].cpu().numpy()
    close(rows.astype(np.float32), ref['router_values'], 2e-3, 1e-3, 'router grid values', quantum=FP16_QUANTUM)
    router_backward = lambda up: oracle.hash_backward(ref['xy'], up, model.router_records, snapshot[1].size)  # noqa
    close_bound(opt.copied('router_grad', (snapshot[1].size,), torch.float32).cpu().numpy(), ref['router_grid_grad'],
                scatter_bound(router_backward, ref['router_values'], 2e-3, 1e-3, FP16_QUANTUM), 'router grid gradient')
    opt.close()
