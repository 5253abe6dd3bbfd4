"""GPU parity of the native training step (a1, a6-a14, a20) through the odie_* C-ABI.

The oracle restates the reference step (odie/native/runtime.cu:253-312) on the
CPU.  Integer/byte parts (coordinates, visibility, encoded features) are
bit-exact; fp16 network quantities (grid-gradient values, squares, head
gradients) agree within 2e-3 relative (the fp16 tolerance) because the fused
tensor-core heads accumulate in a different order than the oracle's fp64
products; the fp32 scatter agrees within 1e-5 given the same fp16 inputs; Adam
is bit-exact given the same gradients.
"""
import json

import numpy as np
import pytest
import torch

from oracle import oracle
from odie_b200 import _lib
from odie_b200.data import ByteTarget
from odie_b200.evaluation import coordinates
from odie_b200.model import PackedXYPlanes
from odie_b200.native_backend import NativeOptimizer
from tests.cases import close, layout_numpy, plane_case, plane_config, random_image, FP16_QUANTUM, close_bound, scatter_bound

pytestmark = pytest.mark.gpu
SHAPE = (61, 47)


def setup(seed=7, router=True, k=0, activation='sigmoid', batch=1024, dims=None):
    resolutions, dims, supports, caps = plane_case(seed, dims=dims)
    config = plane_config(resolutions, dims, 10, seed=seed, router=router, k=k, activation=activation)
    config['batch_size'] = batch
    model = PackedXYPlanes(config, supports, dims, caps)
    rgb = random_image(*SHAPE, seed)
    target = ByteTarget(torch.from_numpy(rgb).cuda())
    planes = [torch.nn.Parameter(model.grid[l['plane_offset']:l['plane_offset'] + l['plane_node_capacity'] *
                                            l['plane_dim']].detach()) for l in model.layout['levels']]
    opt = NativeOptimizer(model, target, SHAPE, config, planes, batch=batch)
    return config, model, rgb, opt


def snapshot(model):
    gate = model.gate.params.detach().cpu().numpy().copy() if model.gate is not None else np.zeros(0, np.float32)
    return (model.grid.detach().cpu().numpy().copy(), gate, model.decoder.params.detach().cpu().numpy().copy())


def read_rows(opt, name, n, width):
    """A row-major [capacity][width] fp16 buffer (the heads' gradient values)."""
    return opt.copied(name, (opt.pointers['capacity'], width), torch.float16)[:n].cpu().numpy()


def read_pair_major(opt, name, n, width):
    cap = opt.pointers['capacity']
    pairs = opt.copied(name, (width // 2, cap, 2), torch.float16)[:, :n, :]
    return pairs.permute(1, 0, 2).reshape(n, width).cpu().numpy()


def reference(model, rgb, ids, grid, gate, dec, router=True, k=0, softplus=False):
    lay = layout_numpy({k2: getattr(model, k2).cpu() for k2 in ('descriptors', 'node_bitmap', 'node_prefix', 'bitmap')})
    return oracle.reference_step(rgb, ids, SHAPE, grid, lay, gate, dec, model.n_levels, model.input_width,
                                 router=router, k_fixed=k, softplus=softplus)


@pytest.mark.parametrize('router,k,activation,order', [(True, 0, 'sigmoid', 'random'), (True, 3, 'softplus', 'random'),
                                                      (False, 0, 'sigmoid', 'random'), (True, 0, 'sigmoid', 'sorted')])
def test_step_gradients_match_oracle(cuda, router, k, activation, order):
    """order 'sorted': raster-ordered ids, so neighbouring lanes share cells (long runs in the scatter)."""
    config, model, rgb, opt = setup(router=router, k=k, activation=activation)
    grid, gate, dec = snapshot(model)
    n = 1000  # not a multiple of the 16-row tiles
    ids_np = np.random.default_rng(1).integers(0, SHAPE[0] * SHAPE[1], n)
    ids = torch.from_numpy(np.sort(ids_np) if order == 'sorted' else ids_np).cuda()
    lib = _lib.library()
    opt.call('step_grads', ids.data_ptr(), n, 2)
    torch.cuda.synchronize()
    assert opt.copied('error_flag', (1,), torch.int32).item() == 0, 'a bounded device wait ran out'
    W = opt.pointers['input_width']
    ref = reference(model, rgb, ids.cpu().numpy(), grid, gate, dec, router, k, activation == 'softplus')
    # bit-exact integer/byte stages
    xy = opt.copied('xy', (opt.pointers['capacity'], 2), torch.float32)[:n].cpu().numpy()
    assert np.array_equal(xy, ref['xy'])
    words = opt.copied('vis', (16, opt.pointers['capacity'] // 32), torch.int32).cpu().numpy().view(np.uint32)
    vis = np.unpackbits(words.view(np.uint8), axis=1, bitorder='little')[:, :n].T  # bit-packed [levels][capacity/32]
    assert np.array_equal(vis, ref['vis'])
    raw = read_pair_major(opt, 'raw', n, W)
    diff = np.argwhere(raw.view(np.uint16) != ref['raw'].view(np.uint16))
    assert not diff.size, (f'{len(diff)} encoded features differ, first (row, col) {diff[:5].tolist()}: '
                           f'{raw[tuple(diff[0])]} vs {ref["raw"][tuple(diff[0])]}')
    # fp16 network quantities
    squares = opt.copied('squares', (n,), torch.float32).cpu().numpy()
    close(squares, ref['squares'], 2e-3, 1e-3, 'squares')
    values = read_rows(opt, 'gvals', n, W)
    close(values.astype(np.float32), ref['values'], 2e-3, 1e-3, 'grid-gradient values', quantum=FP16_QUANTUM)
    heads = opt.copied('head_grad', (opt.pointers['head_count'],), torch.float32).cpu().numpy()
    close(heads, ref['head_grad'], 2e-3, 1e-3, 'head gradients')
    # the fp32 scatter, given the kernel's own fp16 values: fp32 tolerance
    grad = opt.copied('grid_grad', (model.grid.numel(),), torch.float32).cpu().numpy()
    lay = layout_numpy({k2: getattr(model, k2).cpu() for k2 in ('descriptors', 'node_bitmap', 'node_prefix', 'bitmap')})
    backward = lambda up: oracle.query_backward(ref['xy'], up, lay['descriptors'], lay['node_bitmap'],  # noqa: E731
                                                lay['node_prefix'], lay['bitmap'], grid.size)
    values16 = values.astype(np.float16)
    close_bound(grad, backward(values16), scatter_bound(backward, values16), 'grid scatter')
    # end to end: the values' own tolerance carried through the bilinear weights
    close_bound(grad, ref['grid_grad'], scatter_bound(backward, ref['values'], 2e-3, 1e-3, FP16_QUANTUM),
                'grid gradient end to end')
    opt.close()


def test_adam_bit_exact_given_gradients(cuda):
    config, model, rgb, opt = setup(seed=21)
    grid, gate, dec = snapshot(model)
    n = 1024
    ids = torch.from_numpy(np.random.default_rng(2).integers(0, SHAPE[0] * SHAPE[1], n)).cuda()
    lib = _lib.library()
    opt.call('step_grads', ids.data_ptr(), n, 2)
    G = opt.copied('grid_grad', (grid.size,), torch.float32).cpu().numpy()
    H = opt.copied('head_grad', (opt.pointers['head_count'],), torch.float32).cpu().numpy()
    opt.call('grid_update')
    opt.call('step_heads')
    torch.cuda.synchronize()
    p, _, _, steps, half = oracle.adam(grid, np.zeros_like(grid), np.zeros_like(grid), np.zeros(grid.size, np.uint32),
                                       G, 128., config['grid_lr'], skip_zero=True)
    assert np.array_equal(model.grid.detach().cpu().numpy(), p)
    assert np.array_equal(opt.copied('grid_steps', (grid.size,), torch.int32).cpu().numpy(), steps.astype(np.int32))
    mirror = opt.copied('grid_half', (grid.size,), torch.float16).cpu().numpy()
    assert np.array_equal(mirror.view(np.uint16), half.view(np.uint16))
    assert (G == 0).any() and (steps == 0).any(), 'zero-gradient entries must be skipped'
    g_count = gate.size
    gp, *_ = oracle.adam(gate, np.zeros_like(gate), np.zeros_like(gate), np.zeros(g_count, np.uint32), H[:g_count],
                         16384., config['gate_lr'], skip_zero=False)
    dp, *_ = oracle.adam(dec, np.zeros_like(dec), np.zeros_like(dec), np.zeros(dec.size, np.uint32), H[g_count:],
                         16384., config['decoder_lr'], skip_zero=False)
    assert np.array_equal(model.gate.params.detach().cpu().numpy(), gp)
    assert np.array_equal(model.decoder.params.detach().cpu().numpy(), dp)
    opt.close()


def test_graph_replay_trains_and_counts_steps(cuda):
    config, model, rgb, opt = setup(seed=5, batch=1024)
    model.set_active_prefix(16)
    opt.prepare_epoch()
    generator = torch.Generator(device='cuda').manual_seed(3)
    losses = []
    for _ in range(30):
        ids = torch.randint(0, SHAPE[0] * SHAPE[1], (1024,), device='cuda', generator=generator)
        losses.append(float(opt.train_batch(ids)))
    torch.cuda.synchronize()
    assert all(np.isfinite(losses))
    assert np.mean(losses[-5:]) < np.mean(losses[:5])
    steps = opt.copied('head_steps', (opt.pointers['head_count'],), torch.int32).cpu().numpy()
    assert (steps == 30).all()
    assert opt.recaptures == 1
    state = opt.state_summary()
    assert 'hash_fnv1a64' in state and state['bytes'] > 0
    assert opt.state.get(opt.param_groups[0]['params'][0]) == {'native_adam_state': True}
    assert opt.state.get(opt.param_groups[0]['params'][15]) == {}, 'an empty future plane stays pristine'
    opt.close()


def test_decode_matches_module_path(cuda):
    config, model, rgb, opt = setup(seed=8)
    generator = torch.Generator(device='cuda').manual_seed(4)
    for _ in range(5):
        opt.train_batch(torch.randint(0, SHAPE[0] * SHAPE[1], (1024,), device='cuda', generator=generator))
    torch.cuda.synchronize()
    opt.call('sync_weights')
    pixels = SHAPE[0] * SHAPE[1]
    rgb32 = torch.empty((pixels, 3), device='cuda')
    rgb8 = torch.empty((pixels, 3), dtype=torch.uint8, device='cuda')
    opt.decode(0, pixels, rgb=rgb32, rgb8=rgb8)
    with torch.no_grad():
        module = model(coordinates(SHAPE, torch.arange(pixels, device='cuda'))).float()
    close(rgb32.cpu().numpy(), module.cpu().numpy(), 2e-3, 1e-3, 'decode vs module path')
    expected8 = torch.round(rgb32.clamp(0, 1) * 255).to(torch.uint8)
    assert torch.equal(rgb8, expected8)
    opt.close()


def test_create_rejects_invalid_settings(cuda):
    lib = _lib.library()
    bad = json.dumps(dict(stream=0, total=0, width=4, height=4, grid=0, rgb=0, decoder=0, gate=0, active=2,
                          grid_lr=1e-2, gate_lr=1e-3, decoder_lr=1e-3))
    assert lib.odie_create(bad.encode()) is None
    assert 'total' in _lib.error()


def test_mode_bits(cuda):
    """The reference's mode bits are accepted (their paths are always taken or superseded); other bits are refused
    with a message."""
    import json as _json
    config, model, rgb, opt = setup(seed=5)
    assert opt.pointers['mode'] == 20 and opt.pointers['grid_gradient_precision'] == 'fp32'
    assert opt.pointers['half_grad'] == 0 and opt.pointers['output'] == 0
    opt.close()
    lib = _lib.library()
    settings = dict(stream=torch.cuda.current_stream().cuda_stream, total=model.grid.numel(), width=SHAPE[1],
                    height=SHAPE[0], mode=32, rgb=0, grid=model.grid.data_ptr(), decoder=model.decoder.params.data_ptr(),
                    gate=model.gate.params.data_ptr(), levels=16, active=16, descriptors=model.descriptors.data_ptr(),
                    node_bitmap=model.node_bitmap.data_ptr(), node_prefix=model.node_prefix.data_ptr(),
                    bitmap=model.bitmap.data_ptr(), grid_lr=1e-2, gate_lr=1e-3, decoder_lr=1e-3)
    assert not lib.odie_create(_json.dumps(settings).encode())
    assert 'mode' in _lib.error()
