"""Drop-in model / autograd API of the reference (odie/model.py, odie/hash_grid.py).

`PackedQuery` and `HashQuery` run the sm_100a encode kernels through the C-ABI
(libodie_b200.so); the module glue around them (feature masks, gates,
index_select) follows odie/model.py:266-279.  The heads are the reference's
fully fused MLP shapes (odie/model.py:186-195): no biases, ReLU hidden layers,
linear output, fp16 activations, fp32 masters, padded input columns fed with
1.0.  Their parameters are laid out row-major [out][in] per layer (gate: W1, W2;
decoder: W1, W2, W3), the layout the fused training kernel reads.
"""
from copy import deepcopy
import math

import torch
from torch import nn

from . import _lib
from .layout import (ADDRESSING_VERSION, COORDINATE_VERSION, LAYOUT_VERSION, align8, check_gate_k, hash_levels,
                     make_layout, make_layout_device, make_node_index, plane_closure, plane_index_device)

__all__ = ['router_weights', 'align8', 'plane_closure', 'make_node_index', 'make_layout', 'PackedQuery',
           'HashQuery', 'ExpertHashQuery', 'route', 'Head', 'PackedXYPlanes', 'HashGrid', 'RoutedExperts',
           'build_model']


def router_weights(logits, activation):
    """Per-level gate of the router logits (odie/model.py:17-22)."""
    if activation == 'sigmoid':
        return torch.sigmoid(logits)
    if activation == 'softplus':
        return torch.nn.functional.softplus(logits, beta=1., threshold=20.)
    raise ValueError('Unknown router activation: ' + activation)


def _stream():
    return torch.cuda.current_stream().cuda_stream


class PackedQuery(torch.autograd.Function):
    """Packed-plane query: fp16 features [N, width] and visibility [N, L] (odie/model.py:137-151)."""

    @staticmethod
    def forward(ctx, coordinates, grid, descriptors, node_bitmap, node_prefix, bitmap, width):
        for t in (coordinates, grid, descriptors, node_bitmap, node_prefix, bitmap):
            if not t.is_cuda or not t.is_contiguous():
                raise ValueError('PackedQuery inputs must be contiguous CUDA tensors')
        if coordinates.dtype != torch.float32 or coordinates.ndim != 2 or coordinates.shape[1] != 2:
            raise ValueError('coordinates must be CUDA contiguous FP32 Nx2')
        if grid.dtype != torch.float32 or grid.ndim != 1:
            raise ValueError('grid must be flat CUDA FP32')
        levels = descriptors.shape[0]
        n = coordinates.shape[0]
        features = torch.empty((n, width), dtype=torch.float16, device=coordinates.device)
        visible = torch.empty((n, levels), dtype=torch.bool, device=coordinates.device)
        lib = _lib.library()
        _lib.check(lib.odie_query_forward(coordinates.data_ptr(), n, grid.data_ptr(), descriptors.data_ptr(), levels,
                                          node_bitmap.data_ptr(), node_prefix.data_ptr(), bitmap.data_ptr(), width,
                                          features.data_ptr(), visible.data_ptr(), _stream()), 'odie_query_forward')
        ctx.save_for_backward(coordinates, descriptors, node_bitmap, node_prefix, bitmap)
        ctx.param_count = grid.numel()
        ctx.mark_non_differentiable(visible)
        return features, visible

    @staticmethod
    def backward(ctx, feature_gradient, visibility_gradient):
        coordinates, descriptors, node_bitmap, node_prefix, bitmap = ctx.saved_tensors
        upstream = feature_gradient.to(torch.float16).contiguous()
        gradient = torch.empty(ctx.param_count, dtype=torch.float32, device=coordinates.device)
        _lib.check(_lib.library().odie_query_backward(
            coordinates.data_ptr(), coordinates.shape[0], upstream.data_ptr(), upstream.shape[1],
            descriptors.data_ptr(), descriptors.shape[0], node_bitmap.data_ptr(), node_prefix.data_ptr(),
            bitmap.data_ptr(), gradient.data_ptr(), ctx.param_count, _stream()), 'odie_query_backward')
        return None, gradient, None, None, None, None, None


def _hash_table(records):
    table = (_lib.HashLevel * len(records))()
    for i, r in enumerate(records):
        table[i] = _lib.HashLevel(r['scale'], r['resolution'], r['capacity'], r['offset'], r['features'],
                                  r['column'], r['hashed'], int(r.get('cells', -1)))
    return table


class HashQuery(torch.autograd.Function):
    """Hashed multiresolution encoding (the TCNN HashGrid of odie/hash_grid.py:27)."""

    @staticmethod
    def forward(ctx, coordinates, table, records, width):
        n = coordinates.shape[0]
        features = torch.empty((n, width), dtype=torch.float16, device=coordinates.device)
        levels = _hash_table(records)
        _lib.check(_lib.library().odie_hash_forward(coordinates.data_ptr(), n, table.data_ptr(), levels, len(records),
                                                    width, features.data_ptr(), _stream()), 'odie_hash_forward')
        ctx.save_for_backward(coordinates)
        ctx.records, ctx.count = records, table.numel()
        return features

    @staticmethod
    def backward(ctx, feature_gradient):
        (coordinates,) = ctx.saved_tensors
        upstream = feature_gradient.to(torch.float16).contiguous()
        gradient = torch.empty(ctx.count, dtype=torch.float32, device=coordinates.device)
        _lib.check(_lib.library().odie_hash_backward(coordinates.data_ptr(), coordinates.shape[0], upstream.data_ptr(),
                                                     upstream.shape[1], _hash_table(ctx.records), len(ctx.records),
                                                     gradient.data_ptr(), ctx.count, _stream()), 'odie_hash_backward')
        return None, gradient, None, None


class ExpertHashQuery(torch.autograd.Function):
    """Hashed encoding with one table per expert: row i reads expert[i]'s table (routed experts)."""

    @staticmethod
    def forward(ctx, coordinates, tables, expert, expert_stride, records, width, bitmap=None):
        """bitmap: optional CUDA uint8 cell-visibility bytes addressed by each record's 'cells' offset."""
        n = coordinates.shape[0]
        features = torch.empty((n, width), dtype=torch.float16, device=coordinates.device)
        _lib.check(_lib.library().odie_expert_hash_forward(
            coordinates.data_ptr(), n, tables.data_ptr(), expert_stride, expert.data_ptr(), _hash_table(records),
            len(records), width, _lib.ptr(bitmap), features.data_ptr(), _stream()), 'odie_expert_hash_forward')
        ctx.save_for_backward(coordinates, expert)
        ctx.records, ctx.count, ctx.stride, ctx.bitmap = records, tables.numel(), expert_stride, bitmap
        ctx.mark_non_differentiable(expert)
        return features

    @staticmethod
    def backward(ctx, feature_gradient):
        coordinates, expert = ctx.saved_tensors
        upstream = feature_gradient.to(torch.float16).contiguous()
        gradient = torch.empty(ctx.count, dtype=torch.float32, device=coordinates.device)
        _lib.check(_lib.library().odie_expert_hash_backward(
            coordinates.data_ptr(), coordinates.shape[0], upstream.data_ptr(), upstream.shape[1], ctx.stride,
            expert.data_ptr(), _hash_table(ctx.records), len(ctx.records), _lib.ptr(ctx.bitmap), gradient.data_ptr(),
            ctx.count, _stream()), 'odie_expert_hash_backward')
        return None, gradient, None, None, None, None, None


def route(features, router_weights16, experts):
    """Top-1 routing: (expert int32 [N], probability fp32 [N], fp16 logits [N, 16]), bit-exact (router.cu)."""
    features = features.to(torch.float16).contiguous()
    n, width = features.shape
    expert = torch.empty(n, dtype=torch.int32, device=features.device)
    prob = torch.empty(n, dtype=torch.float32, device=features.device)
    logits = torch.empty((n, 16), dtype=torch.float16, device=features.device)
    weights = router_weights16.to(torch.float16).contiguous()
    _lib.check(_lib.library().odie_router_forward(features.data_ptr(), n, width, weights.data_ptr(), int(experts),
                                                  expert.data_ptr(), prob.data_ptr(), logits.data_ptr(), _stream()),
               'odie_router_forward')
    return expert, prob, logits


class Head(nn.Module):
    """Bias-free ReLU MLP with fp16 activations and an fp32 master `params` vector."""

    def __init__(self, n_input, n_output, width, depth, seed, device='cuda'):
        super().__init__()
        self.n_input, self.n_output = n_input, n_output
        self.padded_input = (n_input + 15) // 16 * 16
        self.padded_output = (n_output + 15) // 16 * 16
        self.shapes = [(width, self.padded_input)] + [(width, width)] * (depth - 1) + [(self.padded_output, width)]
        generator = torch.Generator().manual_seed(int(seed))
        chunks = []
        for out_dim, in_dim in self.shapes:
            bound = math.sqrt(6.0 / (in_dim + out_dim))
            chunks.append((torch.rand((out_dim, in_dim), generator=generator) * 2 - 1).mul_(bound).flatten())
        self.params = nn.Parameter(torch.cat(chunks).to(device))

    def matrices(self, values=None):
        values = self.params if values is None else values
        out, offset = [], 0
        for out_dim, in_dim in self.shapes:
            out.append(values[offset:offset + out_dim * in_dim].view(out_dim, in_dim))
            offset += out_dim * in_dim
        return out

    def forward(self, x):
        """fp16 in -> fp16 out [N, padded_output]; fp32 accumulation, fp16 rounding per layer."""
        n = x.shape[0]
        if x.shape[1] < self.padded_input:
            x = torch.cat([x, torch.ones((n, self.padded_input - x.shape[1]), dtype=x.dtype, device=x.device)], 1)
        h = x.to(torch.float16)
        mats = self.matrices()
        for i, w in enumerate(mats):
            z = h.float() @ w.to(torch.float16).float().t()
            if i + 1 < len(mats):
                z = torch.relu(z)
            h = z.to(torch.float16)
        return h


class PackedXYPlanes(nn.Module):
    """Packed multiresolution planes with a shared per-level gate and decoder (odie/model.py:154-314)."""

    def __init__(self, config, supports, plane_dims, plane_node_caps, axis_mode='none', kernel_a=0.,
                 kernel_omega=1.5 * math.pi):
        super().__init__()
        if axis_mode != 'none' or kernel_a != 0.:
            raise ValueError('No axis branches or non-linear interpolation kernel in this ablation')
        self.config = deepcopy(config)
        self.router_enabled = config.get('router_enabled', True)
        self.gate_coarse_levels_K = check_gate_k(config)
        self.layout = make_layout(config, supports, plane_dims, plane_node_caps)
        self.supports = self.layout['supports']
        self.plane_dims, self.plane_node_caps = list(plane_dims), list(plane_node_caps)
        self.input_width = self.layout['input_width']
        self.n_levels = int(config['n_levels'])
        device = torch.device('cuda')
        seed = int(config['seed'])
        self.grid = nn.Parameter(torch.zeros(self.layout['params'], dtype=torch.float32, device=device))
        self.initialized_planes = [False] * self.n_levels
        with torch.no_grad():
            for level, item in enumerate(self.layout['levels']):
                if item['nodes'].numel():
                    self._initialize_plane(level)
        for name in ('descriptors', 'node_bitmap', 'node_prefix', 'bitmap'):
            self.register_buffer(name, self.layout[name].to(device), persistent=False)
        for name in ('node_bitmap', 'node_prefix', 'bitmap'):
            self.layout.pop(name)
        feature_levels = [level for level, dim in enumerate(plane_dims) for _ in range(dim)]
        self.register_buffer('feature_levels', torch.tensor(feature_levels, dtype=torch.int64, device=device),
                             persistent=False)
        self.register_buffer('level_active', torch.ones(self.n_levels, dtype=torch.bool, device=device), persistent=False)
        self.register_buffer('feature_active', torch.ones(self.input_width, dtype=torch.float16, device=device),
                             persistent=False)
        self.active_prefix = self.n_levels
        self.gate = (Head(self.input_width, self.n_levels, 32, 1, (seed + 2000003) % 2**31)
                     if self.router_enabled else None)
        self.decoder = Head(self.input_width, 3, 64, 2, (seed + 4000037) % 2**31)
        gate_count = self.gate.params.numel() if self.gate is not None else 0
        if gate_count != config['gate_parameters'] or self.decoder.params.numel() != config['decoder_parameters']:
            raise RuntimeError('Unexpected head allocation for the configured input width')

    def query_features(self, coordinates):
        if coordinates.dtype != torch.float32 or coordinates.ndim != 2 or coordinates.shape[1] != 2 or \
                coordinates.requires_grad:
            raise ValueError('Coordinates must be FP32 Nx2, without coordinate gradients')
        return PackedQuery.apply(coordinates.contiguous(), self.grid, self.descriptors, self.node_bitmap,
                                 self.node_prefix, self.bitmap, self.input_width)

    @torch.no_grad()
    def _initialize_plane(self, level):
        """Seeded N(0, std) draw over the dense plane, gathered at the retained nodes (odie/model.py:208-224)."""
        if self.initialized_planes[level]:
            raise RuntimeError('Each plane must be initialized exactly once')
        item = self.layout['levels'][level]
        level_seed = (self.config['seed'] + 1000003 * (level + 1)) % (2**31)
        branch_seed = (level_seed + 104729 * 3) % (2**31)
        generator = torch.Generator(device=self.grid.device).manual_seed(branch_seed)
        dense = torch.empty((item['native_plane_points'], max(2, item['plane_dim'])), dtype=torch.float32,
                            device=self.grid.device)
        dense.normal_(0., self.config['feature_init_std'], generator=generator)
        values = dense.index_select(0, item['nodes'].to(self.grid.device))[:, :item['plane_dim']].reshape(-1)
        self.grid[item['plane_offset']:item['plane_offset'] + values.numel()].copy_(values)
        self.initialized_planes[level] = True

    @torch.no_grad()
    def activate_support(self, level, support):
        """Open the next plane on a selected support without moving storage (odie/model.py:226-257)."""
        if level != self.active_prefix or not 2 <= level < self.n_levels:
            raise ValueError('Select the next unopened plane before advancing the prefix')
        if self.initialized_planes[level] or bool(self.supports[level].any()):
            raise RuntimeError('An opened support cannot be replaced or initialized again')
        resolution = self.config['resolutions'][level]
        if support.device.type != 'cpu' or support.dtype != torch.bool or tuple(support.shape) != (resolution**2,):
            raise ValueError('New support must be a flat CPU bool R^2 tensor')
        device = self.grid.device
        count = int(plane_index_device(support.to(device), resolution, with_nodes=False)[3])
        if not 0 < count <= self.plane_node_caps[level]:
            raise ValueError('New support requires a nonempty complete closure within its cap')
        storage = self.grid.data_ptr()
        supports = list(self.supports)
        supports[level] = support.clone()
        # every level's closure, node index and cell bitmap rebuilt on the GPU (odie_plane_index)
        layout = make_layout_device(self.config, [s.to(device) for s in supports], self.plane_dims,
                                    self.plane_node_caps)
        nodes = layout['levels'][level]['nodes']
        for name in ('descriptors', 'node_bitmap', 'node_prefix', 'bitmap'):
            setattr(self, name, layout.pop(name))
        layout['supports'] = [s.cpu() for s in layout['supports']]
        self.layout, self.supports = layout, layout['supports']
        self._initialize_plane(level)
        if self.grid.data_ptr() != storage:
            raise AssertionError('Packed storage changed during plane activation')
        points = layout['levels'][level]['native_plane_points']
        return {'level': level, 'initialized_once': True, 'grid_storage_unchanged': True,
                'original_dense_f2_seed': (self.config['seed'] + 1000003 * (level + 1) + 104729 * 3) % (2**31),
                'native_dense_draw_shape': [points, max(2, self.plane_dims[level])], 'selected_nodes': nodes.numel()}

    def set_active_prefix(self, prefix):
        if not isinstance(prefix, int) or not 2 <= prefix <= self.n_levels:
            raise ValueError('Active prefix must be an integer between 2 and declared level count')
        self.active_prefix = prefix
        self.level_active.copy_(torch.arange(self.n_levels, device=self.grid.device) < prefix)
        self.feature_active.copy_((self.feature_levels < prefix).to(torch.float16))

    def forward(self, coordinates):
        raw, visible = self.query_features(coordinates)
        raw = raw * self.feature_active
        if self.gate is None:
            return self.decoder(raw).float()[:, :3]
        if self.active_prefix > self.gate_coarse_levels_K:
            own = router_weights(self.gate(raw)[:, :self.n_levels].float(),
                                 self.config.get('router_output_activation', 'sigmoid'))
            k = self.gate_coarse_levels_K
            gates = torch.cat([torch.ones_like(own[:, :k]), own[:, k:]], dim=1)
        else:
            gates = torch.ones_like(visible, dtype=torch.float32)
        effective = gates * (visible & self.level_active).float()
        weights = effective.to(raw.dtype).index_select(1, self.feature_levels)
        return self.decoder(raw * weights).float()[:, :3]

    def storage_stats(self):
        grid = self.grid.numel()
        gate = self.gate.params.numel() if self.gate is not None else 0
        heads = gate + self.decoder.params.numel()
        node_bitmaps = self.node_bitmap.numel() * self.node_bitmap.element_size()
        prefixes = self.node_prefix.numel() * self.node_prefix.element_size()
        bitmaps = self.bitmap.numel() * self.bitmap.element_size()
        descriptors = self.descriptors.numel() * self.descriptors.element_size()
        gate_index = self.feature_levels.numel() * self.feature_levels.element_size()
        flags = (self.level_active.numel() * self.level_active.element_size() +
                 self.feature_active.numel() * self.feature_active.element_size())
        return {'actual_params': grid + heads, 'grid_params': grid, 'head_params': heads, 'gate_params': gate,
                'decoder_params': self.decoder.params.numel(), 'router_enabled': self.router_enabled,
                'axis_params': 0, 'plane_params': grid, 'plane_caps': self.plane_node_caps,
                'fp16_parameter_payload_bytes': 2 * (grid + heads), 'fp32_master_bytes': 4 * (grid + heads),
                'adam_moment_bytes': 8 * (grid + heads), 'full_gradient_bytes': 4 * (grid + heads),
                'index_bytes': node_bitmaps + prefixes, 'node_bitmap_bytes': node_bitmaps,
                'node_prefix_bytes': prefixes, 'bitmap_bytes': bitmaps, 'descriptor_bytes': descriptors,
                'runtime_index_bytes': node_bitmaps + prefixes + bitmaps + descriptors + gate_index + flags,
                'active_flag_bytes': flags, 'input_width': self.input_width,
                'native_input_padding': (self.input_width + 15) // 16 * 16, 'axis_mode': 'none',
                'active_layers_from_update1': int(self.config.get('initial_active_prefix', 2)),
                'active_prefix': self.active_prefix, 'gate_coarse_levels_K': int(self.config['coarse_levels']),
                'full_cover_coarse_layers': self.config.get('full_cover_coarse_layers', [0, 1]),
                'plane_dims': self.plane_dims, 'coordinate_version': COORDINATE_VERSION,
                'layout_version': LAYOUT_VERSION, 'addressing_version': ADDRESSING_VERSION,
                'query_cuda_launches': 1, 'backward_cuda_launches': 1,
                'forward_precision': 'P01 FP32 geometry and FP16 interpolation chain',
                'gradient_precision': 'FP16 feature gradient, FP32 interpolation weights and reductions',
                'levels': [{k: v for k, v in level.items() if k != 'nodes'} for level in self.layout['levels']]}


class HashGrid(nn.Module):
    """Hashed multiresolution grid with optional per-level gate (odie/hash_grid.py:8-80)."""

    def __init__(self, config, supports, plane_dims, plane_node_caps):
        super().__init__()
        if supports or config['initial_active_prefix'] != config['n_levels']:
            raise ValueError('HashGrid requires no supports and all levels active')
        self.config = deepcopy(config)
        self.router_enabled = config['router_enabled']
        self.n_levels = self.active_prefix = config['n_levels']
        self.gate_coarse_levels_K = config['gate_coarse_levels_K']
        self.input_width = sum(plane_dims)
        self.plane_dims, self.plane_node_caps = list(plane_dims), list(plane_node_caps)
        self.supports = []
        self.records, total = hash_levels(config['hash_encoding'])
        generator = torch.Generator().manual_seed(int(config['seed']))
        self.grid = nn.Parameter(((torch.rand(total, generator=generator) * 2 - 1) * 1e-4).cuda())
        self.register_buffer('feature_levels', torch.tensor(
            [level for level, dim in enumerate(plane_dims) for _ in range(dim)], dtype=torch.int64, device='cuda'),
            persistent=False)
        seed = int(config['seed'])
        self.gate = (Head(self.input_width, self.n_levels, 32, 1, (seed + 2000003) % 2**31)
                     if self.router_enabled else None)
        self.decoder = Head(self.input_width, 3, 64, 2, (seed + 4000037) % 2**31)
        levels, offset = [], 0
        for dim, cap in zip(plane_dims, plane_node_caps):
            levels.append(dict(plane_offset=offset, plane_node_capacity=cap, plane_dim=dim))
            offset += dim * cap
        self.layout = dict(levels=levels)
        gate = self.gate.params.numel() if self.gate is not None else 0
        if self.grid.numel() != offset or self.decoder.params.numel() != config['decoder_parameters'] or \
                gate != config['gate_parameters']:
            raise RuntimeError('Actual allocation differs from the reference HashGrid budget')

    def set_active_prefix(self, prefix):
        if prefix != self.n_levels:
            raise ValueError('The no-on-demand model always trains every level')

    def forward(self, coordinates):
        raw = HashQuery.apply(coordinates.contiguous(), self.grid, self.records, self.input_width)
        if self.gate is not None:
            weights = router_weights(self.gate(raw)[:, :self.n_levels].float(), self.config['router_output_activation'])
            k = self.gate_coarse_levels_K
            if k:
                weights = torch.cat((torch.ones_like(weights[:, :k]), weights[:, k:]), dim=1)
            raw = raw * weights.to(raw.dtype).index_select(1, self.feature_levels)
        return self.decoder(raw).float()[:, :3]

    def storage_stats(self):
        grid, decoder = self.grid.numel(), self.decoder.params.numel()
        gate = self.gate.params.numel() if self.gate is not None else 0
        heads = gate + decoder
        return dict(actual_params=grid + heads, grid_params=grid, head_params=heads, gate_params=gate,
                    decoder_params=decoder, router_enabled=self.router_enabled, plane_caps=self.plane_node_caps,
                    fp16_parameter_payload_bytes=2 * (grid + heads), input_width=self.input_width,
                    layout_version='hash-grid-v1', addressing_version='instant-ngp-spatial-hash')


class RoutedExperts(nn.Module):
    """Routed multi-expert hash-grid encoding with a shared decoder (16 routed experts in the benchmark; no reference counterpart).

    A coarse shared hash grid (``router_encoding``) feeds the router MLP
    (W -> 32 -> 32 -> 16 logits, top-1 over ``experts``); coordinate i is then
    encoded by its expert's own hash grid (``hash_encoding``; the tables of all
    experts are one flat fp32 parameter, expert-major) and the features, scaled
    by the router probability rounded to fp16, go through the shared decoder
    (W -> 64 -> 64 -> 3).  Training runs in the native runtime; this module's
    forward is the evaluation/decode path.
    """

    def __init__(self, config):
        super().__init__()
        self.config = deepcopy(config)
        self.experts = int(config['experts'])
        if not 1 <= self.experts <= 16:
            raise ValueError('experts must be within 1..16')
        encoding, router_encoding = config['hash_encoding'], config['router_encoding']
        self.records, self.expert_total = hash_levels(encoding)
        self.router_records, router_total = hash_levels(router_encoding)
        self.n_levels = self.active_prefix = int(encoding['n_levels'])
        self.gate_coarse_levels_K = 0
        self.input_width = (self.n_levels * int(encoding['n_features_per_level']) + 15) // 16 * 16
        router_width = (int(router_encoding['n_levels']) * int(router_encoding['n_features_per_level']) + 15) // 16 * 16
        if router_width != self.input_width:
            raise ValueError('router and expert encodings must have the same width')
        seed = int(config['seed'])
        generator = torch.Generator().manual_seed(seed)
        self.grid = nn.Parameter(((torch.rand(self.experts * self.expert_total, generator=generator) * 2 - 1)
                                  * float(config.get('grid_init', 1e-4))).cuda())
        self.router_grid = nn.Parameter(((torch.rand(router_total, generator=generator) * 2 - 1)
                                         * float(config.get('router_init', 1e-1))).cuda())
        self.gate = Head(self.input_width, 16, 32, 2, (seed + 2000003) % 2**31)  # the router MLP
        self.decoder = Head(self.input_width, 3, 64, 2, (seed + 4000037) % 2**31)
        self.supports = []

    def set_active_prefix(self, prefix):
        if prefix != self.n_levels:
            raise ValueError('routed experts always train every level')

    @torch.no_grad()
    def set_allocation(self, tiles, tile_px, shape, dense_resolution=None):
        """On-demand allocation (the allocation benchmark): restrict the expert levels finer than dense_resolution to the
        cells whose centre pixel lies in an allocated tile.  tiles: CUDA uint8/bool [tiles_y, tiles_x] (e.g. the top-k
        of odie_tile_topk); shape: (height, width) of the image.  Default dense_resolution: cells no smaller than
        half a tile stay dense.  Hidden cells give zero features and receive no gradient."""
        tiles = tiles.to(device=self.grid.device, dtype=torch.uint8).contiguous()
        tiles_y, tiles_x = tiles.shape
        height, width = shape
        if dense_resolution is None:
            dense_resolution = 2 * max(tiles_x, tiles_y) + 1
        cells, offset = [], 0
        for r in self.records:
            if r['resolution'] <= dense_resolution:
                cells.append(-1)
            else:
                cells.append(offset)
                offset += (r['resolution'] ** 2 + 7) // 8
        bitmap = torch.zeros(max(offset, 1), dtype=torch.uint8, device=self.grid.device)
        lib = _lib.library()
        for r, c in zip(self.records, cells):
            if c >= 0:
                _lib.check(lib.odie_allocation_bitmap(tiles.data_ptr(), tiles_x, tiles_y, int(tile_px), int(height),
                                                      int(width), r['resolution'], bitmap[c:].data_ptr(), _stream()),
                           'odie_allocation_bitmap')
        for r, c in zip(self.records, cells):
            r['cells'] = c
        self.allocation_bitmap, self.allocation_cells = bitmap, cells
        return bitmap, cells

    def allocation_settings(self):
        """The runtime's 'allocation' settings, or None before set_allocation."""
        if getattr(self, 'allocation_bitmap', None) is None:
            return None
        return {'bitmap': self.allocation_bitmap.data_ptr(), 'cells': list(self.allocation_cells)}

    def route(self, coordinates):
        with torch.no_grad():
            features = HashQuery.apply(coordinates.contiguous(), self.router_grid, self.router_records, self.input_width)
            return route(features, self.gate.params, self.experts)

    def forward(self, coordinates):
        expert, prob, _ = self.route(coordinates)
        features = ExpertHashQuery.apply(coordinates.contiguous(), self.grid, expert, self.expert_total, self.records,
                                         self.input_width, getattr(self, 'allocation_bitmap', None))
        gated = features * prob.to(torch.float16)[:, None]
        return self.decoder(gated).float()[:, :3]

    def storage_stats(self):
        grid, router_grid = self.grid.numel(), self.router_grid.numel()
        heads = self.gate.params.numel() + self.decoder.params.numel()
        return dict(actual_params=grid + router_grid + heads, grid_params=grid, router_grid_params=router_grid,
                    head_params=heads, experts=self.experts, fp16_parameter_payload_bytes=2 * (grid + router_grid + heads),
                    input_width=self.input_width, addressing_version='instant-ngp-spatial-hash')


def build_model(config, supports, plane_dims, plane_node_caps, **kwargs):
    if config['representation'] == 'routed_experts':
        return RoutedExperts(config)
    if config['representation'] == 'hash_grid':
        return HashGrid(config, supports, plane_dims, plane_node_caps)
    return PackedXYPlanes(config, supports, plane_dims, plane_node_caps, **kwargs)
