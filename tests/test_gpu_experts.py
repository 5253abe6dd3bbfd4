"""GPU parity of the routed multi-expert path through the C-ABI.

Routing decisions, hash indices and encoded features are bit-exact against the
CPU oracle; the router probability within 1e-5 (fp32: CUDA's expf may differ
from the host's by an ulp); fp16 network quantities within 2e-3 relative to the
tensor's scale (the tensor cores accumulate in another order than the oracle's
fp64 products); fp32 scatters within 1e-5 given the same fp16 values.
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
from tests.cases import close, random_image

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
        assert np.array_equal(logits.cpu().numpy().view(np.uint16), z_ref.view(np.uint16)), 'router logits differ'
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
    close(grad.cpu().numpy(), oracle.expert_backward(xy, upstream, expert, stride, records, tables.size), 1e-5, 1e-6,
          'expert scatter')


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
    close(opt.copied('squares', (n,), torch.float32).cpu().numpy(), ref['squares'], 2e-3, 2e-3, 'squares')
    values = read_rows(opt, 'gvals', n, W)
    close(values.astype(np.float32), ref['values'], 2e-3, 2e-3, 'expert grid values')
    router_values = read_rows(opt, 'router_gvals', n, W)
    close(router_values.astype(np.float32), ref['router_values'], 2e-3, 2e-3, 'router grid values')
    heads = opt.copied('head_grad', (opt.pointers['head_count'],), torch.float32).cpu().numpy()
    split = opt.pointers['gate_count']
    close(heads[:split], ref['head_grad'][:split], 2e-3, 2e-3, 'router weight gradients')
    close(heads[split:], ref['head_grad'][split:], 2e-3, 2e-3, 'decoder weight gradients')
    grad = opt.copied('grid_grad', (tables.size,), torch.float32).cpu().numpy()
    scatter = oracle.expert_backward(ref['xy'], values.astype(np.float16), ref['expert'], model.expert_total,
                                     model.records, tables.size)
    close(grad, scatter, 1e-5, 1e-6, 'expert scatter given the kernel values')
    close(grad, ref['grid_grad'], 2e-3, 2e-3, 'expert grid gradient end to end')
    rgrad = opt.copied('router_grad', (router_table.size,), torch.float32).cpu().numpy()
    close(rgrad, oracle.hash_backward(ref['xy'], router_values.astype(np.float16), model.router_records,
                                      router_table.size), 1e-5, 1e-6, 'router scatter given the kernel values')
    close(rgrad, ref['router_grid_grad'], 2e-3, 2e-3, 'router grid gradient end to end')
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
    close(rgb32.cpu().numpy(), module.cpu().numpy(), 2e-3, 2e-3, 'decode vs module path')
    assert torch.equal(rgb8, torch.round(rgb32.clamp(0, 1) * 255).to(torch.uint8))
    opt.close()
