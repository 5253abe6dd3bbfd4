"""GPU parity of the on-device packed-plane index (odie_plane_index) with the reference's layout.

The fixtures in tests/golden/layout.npz were produced by the reference's own
plane_closure / make_layout (odie/model.py:36-118); the device builder must
reproduce them bit for bit, and match the host builder on random supports,
including empty, full and edge-cell supports and resolutions whose R^2 is not a
multiple of 8 or 64.
"""
import time

import numpy as np
import pytest
import torch

from odie_b200 import layout

pytestmark = pytest.mark.gpu


def host_tables(support, r):
    nodes = layout.plane_closure(support, r)
    bits, prefix = layout.make_node_index(nodes, layout.align8(r * r))
    return nodes.numpy(), bits.numpy(), prefix.numpy(), layout.cell_bitmap(support, r).numpy()


def device_tables(support, r):
    bits, prefix, bitmap, count, nodes = layout.plane_index_device(torch.from_numpy(support).cuda(), r)
    torch.cuda.synchronize()
    n = int(count)
    return nodes[:n].cpu().numpy(), bits.cpu().numpy(), prefix.cpu().numpy(), bitmap.cpu().numpy()


def test_device_closure_matches_reference_fixtures(cuda, golden):
    g = golden('layout.npz')
    for key in (k for k in g if k.startswith('clo_support_')):
        r = int(key.split('_')[-1])
        nodes, _, _, _ = device_tables(g[key].astype(bool), r)
        assert np.array_equal(nodes, g[f'clo_plane_{r}']), key


def test_device_layout_matches_reference_make_layout(cuda, golden):
    g = golden('layout.npz')
    resolutions = [int(r) for r in g['lay_resolutions']]
    config = dict(resolutions=resolutions, n_levels=len(resolutions), representation='xy_planes', coarse_levels=0,
                  gate_topology='shared', gate_position='feature', initial_active_prefix=3)
    supports = [torch.from_numpy(g[f'lay_support_{l}']).cuda() for l in range(len(resolutions))]
    out = layout.make_layout_device(config, supports, [int(d) for d in g['lay_dims']], [int(c) for c in g['lay_caps']])
    assert np.array_equal(out['descriptors'].cpu().numpy(), g['lay_descriptors'])
    assert np.array_equal(out['node_bitmap'].cpu().numpy().view(np.int64), g['lay_node_bitmap'])
    assert np.array_equal(out['node_prefix'].cpu().numpy(), g['lay_node_prefix'])
    assert np.array_equal(out['bitmap'].cpu().numpy(), g['lay_bitmap'])
    assert out['params'] == int(g['lay_params']) and out['input_width'] == int(g['lay_input_width'])


@pytest.mark.parametrize('r', [1, 2, 3, 5, 7, 8, 9, 31, 64, 65, 127, 300, 1023, 2049])
def test_device_index_matches_host_on_random_supports(cuda, r):
    rng = np.random.default_rng(r)
    cases = [np.zeros(r * r, bool), np.ones(r * r, bool), rng.random(r * r) < 0.2, rng.random(r * r) < 0.9]
    edge = np.zeros(r * r, bool)
    edge[-1] = True               # the last cell: its corners wrap past R^2
    edge[r - 1] = True            # right edge of the first row
    cases.append(edge)
    for support in cases:
        got, want = device_tables(support, r), host_tables(support, r)
        for name, a, b in zip(('nodes', 'node bitmap', 'prefix', 'cell bitmap'), got, want):
            assert np.array_equal(a, b), f'R={r}: {name} differs'


def test_device_index_at_gigapixel_resolution(cuda):
    """R = 8192 (67 M cells), the reference's gigapixel on-demand planes: equal tables, and the time of both."""
    r = 8192
    g = torch.Generator(device='cuda').manual_seed(3)
    coarse = torch.rand((64, 64), device='cuda', generator=g) < 0.2   # 20 % of 128 x 128-cell tiles
    support = coarse.repeat_interleave(128, 0).repeat_interleave(128, 1).reshape(-1).contiguous()
    layout.plane_index_device(support, r)  # warm-up
    torch.cuda.synchronize()
    started = time.perf_counter()
    bits, prefix, bitmap, count, nodes = layout.plane_index_device(support, r)
    torch.cuda.synchronize()
    device_s = time.perf_counter() - started
    host = support.cpu().numpy()
    started = time.perf_counter()
    h_nodes, h_bits, h_prefix, h_bitmap = host_tables(host, r)
    host_s = time.perf_counter() - started
    n = int(count)
    assert n == h_nodes.size
    assert np.array_equal(nodes[:n].cpu().numpy(), h_nodes)
    assert np.array_equal(bits.cpu().numpy(), h_bits) and np.array_equal(prefix.cpu().numpy(), h_prefix)
    assert np.array_equal(bitmap.cpu().numpy(), h_bitmap)
    print(f'R=8192 plane index: device {device_s * 1e3:.2f} ms, host {host_s * 1e3:.0f} ms')


def test_activate_support_builds_the_host_layout_on_device(cuda):
    """Opening a plane (stage boundary) gives the same tables as the host builder and the reference's init."""
    from odie_b200.model import PackedXYPlanes
    from tests.cases import plane_case, plane_config
    resolutions, dims, supports, caps = plane_case(9, dense=10, packed=4, finest=96)
    level = 14
    r = resolutions[level]
    support = torch.from_numpy(np.random.default_rng(4).random(r * r) < 0.05)
    caps[level] = layout.align8(layout.plane_closure(support.numpy(), r).numel()) + 8  # fixed at construction
    config = plane_config(resolutions, dims, 10, seed=9)
    model = PackedXYPlanes(config, supports, dims, caps)
    model.set_active_prefix(level)
    with pytest.raises(ValueError, match='closes over'):
        model.activate_support(level, torch.ones(r * r, dtype=torch.bool))
    report = model.activate_support(level, support)
    new_supports = list(supports)
    new_supports[level] = support
    host = layout.make_layout(config, new_supports, dims, caps)
    for name in ('descriptors', 'node_bitmap', 'node_prefix', 'bitmap'):
        assert torch.equal(getattr(model, name).cpu(), host[name]), name
    item = host['levels'][level]
    nodes = item['nodes']
    assert report['selected_nodes'] == nodes.numel()
    seed = ((config['seed'] + 1000003 * (level + 1)) % 2**31 + 104729 * 3) % 2**31
    dense = torch.empty((item['native_plane_points'], max(2, dims[level])), device='cuda')
    dense.normal_(0., config['feature_init_std'], generator=torch.Generator(device='cuda').manual_seed(seed))
    expected = dense.index_select(0, nodes.cuda())[:, :dims[level]].reshape(-1)
    got = model.grid[item['plane_offset']:item['plane_offset'] + expected.numel()]
    assert torch.equal(got, expected)
