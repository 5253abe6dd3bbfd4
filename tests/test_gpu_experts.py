"""GPU parity of the routed multi-expert path through the C-ABI.

Routing decisions, hash indices and encoded features are bit-exact against the
CPU oracle; the router probability within 1e-5 (fp32: CUDA's expf may differ
from the host's by an ulp); fp16 network quantities within 2e-3 relative per
element plus 1e-3 of the tensor's RMS (the tensor cores accumulate in another order
than the oracle's fp64 products); fp32 scatters within 1e-5 given the same fp16 values.
"""
import numpy as np
import pytest
import torch

from oracle import oracle
from odie_b200 import _lib
from odie_b200.data import ByteTarget
from odie_b200.evaluation import coordinates
from odie_b200.layout import hash_levels
from odie_b200.model import ExpertHashQuery, RoutedExperts, route
from odie_b200.native_backend import NativeOptimizer
from tests.cases import close, random_image, FP16_QUANTUM, close_bound, scatter_bound

pytestmark = pytest.mark.gpu
SHAPE = (61, 47)


def experts_config(experts=4, seed=3, batch=1024):
    return dict(representation='routed_experts', experts=experts, seed=seed, grid_init=0.05, router_init=0.5,
                hash_encoding=dict(otype='HashGrid', n_levels=16, n_features_per_level=2, log2_hashmap_size=10,
                                   base_resolution=4, per_level_scale=1.5),
                router_encoding=dict(otype='HashGrid', n_levels=16, n_features_per_level=2, log2_hashmap_size=8,
                                     base_resolution=2, per_level_scale=1.2),
                grid_lr=1e-2, gate_lr=1e-3, decoder_lr=1e-3, batch_size=batch)


def setup(experts=4, seed=3, batch=1024):
    config = experts_config(experts, seed, batch)
    model = RoutedExperts(config)
    rgb = random_image(*SHAPE, seed)
    target = ByteTarget(torch.from_numpy(rgb).cuda())
    opt = NativeOptimizer(model, target, SHAPE, config, [model.grid], batch=batch)
    return config, model, rgb, opt


def read_rows(opt, name, n, width):
    """A row-major [capacity][width] fp16 buffer (the heads' gradient values)."""
    return opt.copied(name, (opt.pointers['capacity'], width), torch.float16)[:n].cpu().numpy()


def read_pair_major(opt, name, n, width):
    cap = opt.pointers['capacity']
    pairs = opt.copied(name, (width // 2, cap, 2), torch.float16)[:, :n, :]
    return pairs.permute(1, 0, 2).reshape(n, width).cpu().numpy()


def test_router_bit_exact(cuda):
    rng = np.random.default_rng(5)
    n, width = 4099, 32
    features = (rng.standard_normal((n, width)) * 0.7).astype(np.float16)
    features[100:110] = features[90:100]                       # repeated rows
    weights = (rng.standard_normal(32 * width + 32 * 32 + 16 * 32) * 0.25).astype(np.float16)
    weights[32 * width + 32 * 32 + 3 * 32:32 * width + 32 * 32 + 4 * 32] = \
        weights[32 * width + 32 * 32 + 7 * 32:32 * width + 32 * 32 + 8 * 32]  # logits 3 and 7 tie exactly
    for experts in (16, 11, 1):
        expert, prob, logits = route(torch.from_numpy(features).cuda(), torch.from_numpy(weights).cuda(), experts)
        torch.cuda.synchronize()
        w1, w2, w3 = np.split(weights, [32 * width, 32 * width + 32 * 32])
        e_ref, p_ref, z_ref = oracle.router(features, w1, w2, w3, 32, experts)
        z = logits.cpu().numpy().view(np.uint16)
        assert z.shape[1] == (8 if experts <= 8 else 16)
        assert np.array_equal(z[:, :experts], z_ref.view(np.uint16)[:, :experts]), 'router logits differ'
        assert (z[:, experts:] == 0).all(), 'logit padding must be zero'
        assert np.array_equal(expert.cpu().numpy(), e_ref), 'routing decisions differ'
        close(prob.cpu().numpy(), p_ref, 1e-5, 0.0, 'router probability')
        if experts == 1:
            assert (expert.cpu().numpy() == 0).all() and (prob.cpu().numpy() == 1).all()


def test_expert_hash_query_bit_exact_and_scatter(cuda):
    rng = np.random.default_rng(8)
    encoding = experts_config()['hash_encoding']
    records, stride = hash_levels(encoding)
    experts, n = 5, 3000
    tables = (rng.standard_normal(experts * stride) * 0.1).astype(np.float32)
    xy = rng.random((n, 2), dtype=np.float32)
    xy[:4] = [[0, 0], [1, 1], [0, 1], [1, 0]]
    expert = rng.integers(0, experts, n).astype(np.int32)
    xy_d, tables_d, expert_d = (torch.from_numpy(a).cuda() for a in (xy, tables, expert))
    features = ExpertHashQuery.apply(xy_d, tables_d, expert_d, stride, records, 32)
    torch.cuda.synchronize()
    expected = oracle.expert_query(xy, tables.astype(np.float16), expert, stride, records, 32)
    assert np.array_equal(features.cpu().numpy().view(np.uint16), expected.view(np.uint16))
    upstream = (rng.standard_normal((n, 32)) * 0.01).astype(np.float16)
    grad = torch.empty(tables.size, dtype=torch.float32, device='cuda')
    up_d = torch.from_numpy(upstream).cuda()
    from odie_b200.model import _hash_table, _stream
    _lib.check(_lib.library().odie_expert_hash_backward(xy_d.data_ptr(), n, up_d.data_ptr(), 32, stride,
                                                        expert_d.data_ptr(), _hash_table(records), len(records),
                                                        None, grad.data_ptr(), tables.size, _stream()))
    torch.cuda.synchronize()
    backward = lambda up: oracle.expert_backward(xy, up, expert, stride, records, tables.size)  # noqa: E731
    close_bound(grad.cpu().numpy(), backward(upstream), scatter_bound(backward, upstream), 'expert scatter')


@pytest.mark.parametrize('experts,order', [(4, 'random'), (16, 'random'), (4, 'sorted')])
def test_experts_step_matches_oracle(cuda, experts, order):
    """order 'sorted': raster-ordered ids, so neighbouring lanes share cells (long runs in the scatter)."""
    config, model, rgb, opt = setup(experts=experts)
    n = 1000
    ids_np = np.random.default_rng(1).integers(0, SHAPE[0] * SHAPE[1], n)
    ids = torch.from_numpy(np.sort(ids_np) if order == 'sorted' else ids_np).cuda()
    tables = model.grid.detach().cpu().numpy().copy()
    router_table = model.router_grid.detach().cpu().numpy().copy()
    router_params = model.gate.params.detach().cpu().numpy().copy()
    decoder_params = model.decoder.params.detach().cpu().numpy().copy()
    opt.call('step_grads', ids.data_ptr(), n, 2)
    torch.cuda.synchronize()
    assert opt.copied('error_flag', (1,), torch.int32).item() == 0, 'a bounded device wait ran out'
    ref = oracle.reference_step_experts(rgb, ids.cpu().numpy(), SHAPE, tables, model.records, model.expert_total,
                                        experts, router_table, model.router_records, router_params, decoder_params)
    W = opt.pointers['input_width']
    xy = opt.copied('xy', (opt.pointers['capacity'], 2), torch.float32)[:n].cpu().numpy()
    assert np.array_equal(xy, ref['xy'])
    rin = read_rows(opt, 'router_in', n, W)
    assert np.array_equal(rin.view(np.uint16), ref['router_features'].view(np.uint16)), 'router-grid features differ'
    expert = opt.copied('expert_ids', (n,), torch.int32).cpu().numpy()
    assert np.array_equal(expert, ref['expert']), 'routing decisions differ'
    assert len(np.unique(expert)) > 1, 'the test case should route to several experts'
    close(opt.copied('prob', (n,), torch.float32).cpu().numpy(), ref['prob'], 1e-5, 0.0, 'router probability')
    raw = read_rows(opt, 'raw', n, W)
    assert np.array_equal(raw.view(np.uint16), ref['raw'].view(np.uint16)), 'expert features differ'
    close(opt.copied('squares', (n,), torch.float32).cpu().numpy(), ref['squares'], 2e-3, 1e-3, 'squares')
    values = read_rows(opt, 'gvals', n, W)
    close(values.astype(np.float32), ref['values'], 2e-3, 1e-3, 'expert grid values', quantum=FP16_QUANTUM)
    router_values = read_rows(opt, 'router_gvals', n, W)
    close(router_values.astype(np.float32), ref['router_values'], 2e-3, 1e-3, 'router grid values',
          quantum=FP16_QUANTUM)
    heads = opt.copied('head_grad', (opt.pointers['head_count'],), torch.float32).cpu().numpy()
    split = opt.pointers['gate_count']
    close(heads[:split], ref['head_grad'][:split], 2e-3, 1e-3, 'router weight gradients')
    close(heads[split:], ref['head_grad'][split:], 2e-3, 1e-3, 'decoder weight gradients')
    grad = opt.copied('grid_grad', (tables.size,), torch.float32).cpu().numpy()
    experts_backward = lambda up: oracle.expert_backward(ref['xy'], up, ref['expert'], model.expert_total,  # noqa
                                                         model.records, tables.size)
    values16 = values.astype(np.float16)
    close_bound(grad, experts_backward(values16), scatter_bound(experts_backward, values16),
                'expert scatter given the kernel values')
    close_bound(grad, ref['grid_grad'], scatter_bound(experts_backward, ref['values'], 2e-3, 1e-3, FP16_QUANTUM),
                'expert grid gradient end to end')
    rgrad = opt.copied('router_grad', (router_table.size,), torch.float32).cpu().numpy()
    router_backward = lambda up: oracle.hash_backward(ref['xy'], up, model.router_records, router_table.size)  # noqa
    router16 = router_values.astype(np.float16)
    close_bound(rgrad, router_backward(router16), scatter_bound(router_backward, router16),
                'router scatter given the kernel values')
    close_bound(rgrad, ref['router_grid_grad'],
                scatter_bound(router_backward, ref['router_values'], 2e-3, 1e-3, FP16_QUANTUM),
                'router grid gradient end to end')
    opt.close()


def test_experts_training_and_decode(cuda):
    config, model, rgb, opt = setup(experts=8, seed=9, batch=1024)
    opt.prepare_epoch()
    generator = torch.Generator(device='cuda').manual_seed(3)
    losses = []
    for _ in range(40):
        ids = torch.randint(0, SHAPE[0] * SHAPE[1], (1024,), device='cuda', generator=generator)
        losses.append(float(opt.train_batch(ids)))
    torch.cuda.synchronize()
    assert all(np.isfinite(losses))
    assert np.mean(losses[-5:]) < np.mean(losses[:5])
    assert opt.copied('error_flag', (1,), torch.int32).item() == 0
    steps = opt.copied('head_steps', (opt.pointers['head_count'],), torch.int32).cpu().numpy()
    assert (steps == 40).all()
    assert opt.copied('router_steps', (model.router_grid.numel(),), torch.int32).cpu().numpy().max() == 40
    opt.call('sync_weights')
    pixels = SHAPE[0] * SHAPE[1]
    rgb32 = torch.empty((pixels, 3), device='cuda')
    rgb8 = torch.empty((pixels, 3), dtype=torch.uint8, device='cuda')
    opt.decode(0, pixels, rgb=rgb32, rgb8=rgb8)
    with torch.no_grad():
        xy = coordinates(SHAPE, torch.arange(pixels, device='cuda'))
        module = model(xy).float()
    close(rgb32.cpu().numpy(), module.cpu().numpy(), 2e-3, 1e-3, 'decode vs module path')
    assert torch.equal(rgb8, torch.round(rgb32.clamp(0, 1) * 255).to(torch.uint8))
    opt.close()


BANDED = dict(bands=4, per_band=8)  # 32 experts: the 64-row router and 8 live logits per coordinate


def banded_setup(first_band=0, bands_held=4, seed=13, batch=1024, full=(120, 47)):
    """Spatial expert ownership on a small image: the full image has `full` rows x columns cut into 4 bands of 8
    experts; this runtime holds bands [first_band, first_band + bands_held) and their rows."""
    height, width = full
    band_rows = height // BANDED['bands']
    row0, rows = first_band * band_rows, bands_held * band_rows
    config = experts_config(BANDED['bands'] * BANDED['per_band'], seed, batch)
    config.update(bands=BANDED['bands'], experts_per_band=BANDED['per_band'], first_band=first_band,
                  bands_held=bands_held, image_rows=height, row_offset=row0)
    model = RoutedExperts(config)
    rgb = random_image(rows, width, seed)
    opt = NativeOptimizer(model, ByteTarget(torch.from_numpy(rgb).cuda()), (rows, width), config, [model.grid],
                          batch=batch)
    banding = dict(bands=BANDED['bands'], first_band=first_band, per_band=BANDED['per_band'], rows=height,
                   row_offset=row0)
    return config, model, rgb, (rows, width), opt, banding


def test_router_banded_bit_exact(cuda):
    """64 logit rows, 8 bands of 8: every coordinate chooses among its band's experts, in local numbering when
    the runtime holds bands 2..5 only; exact ties, band edges and the first/last rows included."""
    rng = np.random.default_rng(21)
    n, width, rows = 5003, 32, 1000
    features = (rng.standard_normal((n, width)) * 0.7).astype(np.float16)
    weights = (rng.standard_normal(32 * width + 32 * 32 + 64 * 32) * 0.25).astype(np.float16)
    w3 = 32 * width + 32 * 32
    weights[w3 + 17 * 32:w3 + 18 * 32] = weights[w3 + 20 * 32:w3 + 21 * 32]  # logits 17 and 20 (band 2) tie
    for first, held in ((0, 8), (2, 4)):
        band_rows = rows // 8
        local = rng.integers(first * band_rows, (first + held) * band_rows, n)
        local[:6] = [first * band_rows, (first + held) * band_rows - 1, (first + 1) * band_rows - 1,
                     (first + 1) * band_rows, 0 if first == 0 else first * band_rows, rows - 1 if first + held == 8
                     else (first + held) * band_rows - 1]
        y = (local.astype(np.float32) * np.float32(1.0 / (rows - 1))).astype(np.float32)
        xy = np.stack((rng.random(n, dtype=np.float32), y), 1).astype(np.float32)
        banding = dict(bands=8, first_band=first, per_band=8, rows=rows)
        expert, prob, logits = route(torch.from_numpy(features).cuda(), torch.from_numpy(weights).cuda(), held * 8,
                                     torch.from_numpy(xy).cuda(), banding)
        torch.cuda.synchronize()
        band = oracle.band_rows_of(local, 1, dict(banding, experts=held * 8))
        w1, w2, w3w = np.split(weights, [32 * width, w3])
        choice, p_ref, z_ref = oracle.router(features, w1, w2, w3w, 32, 8, first=band * 8)
        assert np.array_equal(expert.cpu().numpy(), (band - first) * 8 + choice), 'banded routing differs'
        live = np.take_along_axis(z_ref.view(np.uint16), band[:, None] * 8 + np.arange(8)[None, :], 1)
        assert np.array_equal(logits.cpu().numpy().view(np.uint16), live), 'live logits differ'
        close(prob.cpu().numpy(), p_ref, 1e-5, 0.0, 'router probability')
        assert len(np.unique(band)) == held


@pytest.mark.parametrize('first_band,bands_held', [(0, 4), (2, 2)])
def test_banded_experts_step_matches_oracle(cuda, first_band, bands_held):
    """The wide routed-expert heads (64 logit rows, 8 live per coordinate, dWr1/dWr2 sharing one accumulator)
    against the oracle, for a runtime holding all bands and for one holding bands 2-3 of the full image."""
    config, model, rgb, shape, opt, banding = banded_setup(first_band, bands_held)
    n = 1000
    ids = torch.from_numpy(np.random.default_rng(4).integers(0, shape[0] * shape[1], n)).cuda()
    snapshot = [t.detach().cpu().numpy().copy() for t in (model.grid, model.router_grid, model.gate.params,
                                                          model.decoder.params)]
    opt.call('step_grads', ids.data_ptr(), n, 2)
    torch.cuda.synchronize()
    assert opt.copied('error_flag', (1,), torch.int32).item() == 0, 'a bounded device wait ran out'
    ref = oracle.reference_step_experts(rgb, ids.cpu().numpy(), shape, snapshot[0], model.records, model.expert_total,
                                        model.experts_held, snapshot[1], model.router_records, snapshot[2],
                                        snapshot[3], banding=banding)
    W = opt.pointers['input_width']
    xy = opt.copied('xy', (opt.pointers['capacity'], 2), torch.float32)[:n].cpu().numpy()
    assert np.array_equal(xy, ref['xy']), 'full-image coordinates differ'
    expert = opt.copied('expert_ids', (n,), torch.int32).cpu().numpy()
    assert np.array_equal(expert, ref['expert']), 'banded routing decisions differ'
    assert len(np.unique(ref['band'])) == bands_held
    live = opt.pointers['live']
    logits = opt.copied('logits', (opt.pointers['capacity'], live), torch.float16)[:n].cpu().numpy()
    assert np.array_equal(logits[:, :8].view(np.uint16), ref['live_logits'].view(np.uint16)), 'live logits differ'
    close(opt.copied('prob', (n,), torch.float32).cpu().numpy(), ref['prob'], 1e-5, 0.0, 'router probability')
    raw = read_rows(opt, 'raw', n, W)
    assert np.array_equal(raw.view(np.uint16), ref['raw'].view(np.uint16)), 'expert features differ'
    close(opt.copied('squares', (n,), torch.float32).cpu().numpy(), ref['squares'], 2e-3, 1e-3, 'squares')
    close(read_rows(opt, 'gvals', n, W).astype(np.float32), ref['values'], 2e-3, 1e-3, 'expert grid values',
          quantum=FP16_QUANTUM)
    close(read_rows(opt, 'router_gvals', n, W).astype(np.float32), ref['router_values'], 2e-3, 1e-3,
          'router grid values', quantum=FP16_QUANTUM)
    heads = opt.copied('head_grad', (opt.pointers['head_count'],), torch.float32).cpu().numpy()
    split = opt.pointers['gate_count']
    assert split == 32 * 32 + 32 * 32 + 64 * 32
    close(heads[:32 * 32], ref['head_grad'][:32 * 32], 2e-3, 1e-3, 'router W1 gradient')
    close(heads[32 * 32:2 * 32 * 32], ref['head_grad'][32 * 32:2 * 32 * 32], 2e-3, 1e-3, 'router W2 gradient')
    close(heads[2 * 32 * 32:split], ref['head_grad'][2 * 32 * 32:split], 2e-3, 1e-3, 'router W3 gradient')
    close(heads[split:], ref['head_grad'][split:], 2e-3, 1e-3, 'decoder weight gradients')
    grad = opt.copied('grid_grad', (snapshot[0].size,), torch.float32).cpu().numpy()
    experts_backward = lambda up: oracle.expert_backward(ref['xy'], up, ref['expert'], model.expert_total,  # noqa
                                                         model.records, snapshot[0].size)
    close_bound(grad, ref['grid_grad'], scatter_bound(experts_backward, ref['values'], 2e-3, 1e-3, FP16_QUANTUM),
                'expert grid gradient end to end')
    rgrad = opt.copied('router_grad', (snapshot[1].size,), torch.float32).cpu().numpy()
    router_backward = lambda up: oracle.hash_backward(ref['xy'], up, model.router_records, snapshot[1].size)  # noqa
    close_bound(rgrad, ref['router_grid_grad'],
                scatter_bound(router_backward, ref['router_values'], 2e-3, 1e-3, FP16_QUANTUM),
                'router grid gradient end to end')
    opt.close()


def test_banded_model_is_the_same_at_every_split(cuda):
    """The same global expert's table and the same shared weights whichever rank holds its band."""
    whole = banded_setup(0, 4)
    half = banded_setup(2, 2)
    stride = whole[1].expert_total
    assert torch.equal(whole[1].grid[2 * 8 * stride:].cpu(), half[1].grid.cpu())
    for a, b in ((whole[1].router_grid, half[1].router_grid), (whole[1].gate.params, half[1].gate.params),
                 (whole[1].decoder.params, half[1].decoder.params)):
        assert torch.equal(a.cpu(), b.cpu())
    whole[4].close()
    half[4].close()
