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

import numpy as np
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


def router_out(model_experts):
    """Logit rows of the router MLP: 16 for up to 16 experts, 64 for up to 64."""
    if not 1 <= model_experts <= 64:
        raise ValueError('the router takes 1..64 experts')
    return 16 if model_experts <= 16 else 64


def route(features, router_weights16, experts, xy=None, banding=None):
    """Top-1 routing, bit-exact (router.cu): (expert int32 [N], probability fp32 [N], fp16 live logits [N, live]).

    Without banding every coordinate chooses among `experts`.  banding (dict: bands, first_band, per_band,
    rows): spatial expert ownership -- the coordinate (xy, CUDA fp32 [N, 2]) of global row y chooses among the
    experts of band floor(y * bands / rows); `experts` is then the number held (local numbering)."""
    features = features.to(torch.float16).contiguous()
    n, width = features.shape
    b = banding or dict(bands=1, first_band=0, per_band=int(experts), rows=2)
    live = 8 if b['per_band'] <= 8 else 16
    expert = torch.empty(n, dtype=torch.int32, device=features.device)
    prob = torch.empty(n, dtype=torch.float32, device=features.device)
    logits = torch.empty((n, live), dtype=torch.float16, device=features.device)
    weights = router_weights16.to(torch.float16).contiguous()
    xy = None if xy is None else xy.to(torch.float32).contiguous()
    if b['bands'] > 1 and xy is None:
        raise ValueError('banded routing needs the coordinates')
    _lib.check(_lib.library().odie_router_forward_banded(
        features.data_ptr(), _lib.ptr(xy), n, width, weights.data_ptr(), int(experts), int(b['bands']),
        int(b['first_band']), int(b['per_band']), int(b['rows']), expert.data_ptr(), prob.data_ptr(),
        logits.data_ptr(), live, _stream()), 'odie_router_forward_banded')
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


def plane_seed(seed, level):
    """Seed of level `level`'s first-opening draw: the reference's per-level seed for its F = 2 branch
    ((seed + 1000003 (level + 1)) + 104729 * 3 mod 2^31, odie/model.py:208-224); a seeding contract, so that
    a plane opened here starts from the same values."""
    return ((seed + 1000003 * (level + 1)) % 2**31 + 104729 * 3) % 2**31


class PackedXYPlanes(nn.Module):
    """Packed multiresolution planes behind a shared per-level gate and decoder: the module the reference's
    training loop drives (odie/model.py:154-314).

    Storage: one flat fp32 `grid`, level after level, each level holding the rows of its closure nodes
    (all nodes of a full level).  Index buffers (descriptors, node bitmap words, prefixes, cell bitmap) live on
    the device and are rebuilt there when a level opens (make_layout_device).  The heads are the fully fused
    MLP shapes (Head).  forward(coordinates) is the evaluation path; training runs in the native runtime."""

    BUFFERS = ('descriptors', 'node_bitmap', 'node_prefix', 'bitmap')

    def __init__(self, config, supports, plane_dims, plane_node_caps, axis_mode='none', kernel_a=0.,
                 kernel_omega=1.5 * math.pi):
        super().__init__()
        if axis_mode != 'none' or kernel_a != 0.:
            raise ValueError('only the plain planes (no axis branches, bilinear kernel) are built here')
        self.config = deepcopy(config)
        self.n_levels = int(config['n_levels'])
        self.router_enabled = config.get('router_enabled', True)
        self.gate_coarse_levels_K = check_gate_k(config)
        self.plane_dims, self.plane_node_caps = list(plane_dims), list(plane_node_caps)
        layout = make_layout(config, supports, plane_dims, plane_node_caps)
        self.input_width = layout['input_width']
        device = torch.device('cuda')
        self.grid = nn.Parameter(torch.zeros(layout['params'], dtype=torch.float32, device=device))
        self.initialized_planes = [False] * self.n_levels
        self._install(layout, device)
        with torch.no_grad():
            for level, entry in enumerate(self.layout['levels']):
                if entry['nodes'].numel():
                    self._initialize_plane(level)
        column_level = torch.tensor([l for l, dim in enumerate(plane_dims) for _ in range(dim)], dtype=torch.int64)
        self.register_buffer('feature_levels', column_level.to(device), persistent=False)
        self.register_buffer('level_active', torch.ones(self.n_levels, dtype=torch.bool, device=device),
                             persistent=False)
        self.register_buffer('feature_active', torch.ones(self.input_width, dtype=torch.float16, device=device),
                             persistent=False)
        self.active_prefix = self.n_levels
        seed = int(config['seed'])
        self.gate = Head(self.input_width, self.n_levels, 32, 1, (seed + 2000003) % 2**31) if self.router_enabled else None
        self.decoder = Head(self.input_width, 3, 64, 2, (seed + 4000037) % 2**31)
        counts = (self.gate.params.numel() if self.gate is not None else 0, self.decoder.params.numel())
        if counts != (config['gate_parameters'], config['decoder_parameters']):
            raise RuntimeError(f'head parameters {counts} differ from the configured '
                               f'{(config["gate_parameters"], config["decoder_parameters"])}')

    def _install(self, layout, device):
        """Adopt a layout: its index tensors become device buffers, the rest stays in self.layout."""
        for name in self.BUFFERS:
            tensor = layout.pop(name).to(device)
            if name in self._buffers:
                setattr(self, name, tensor)
            else:
                self.register_buffer(name, tensor, persistent=False)
        layout['supports'] = [support.cpu() for support in layout['supports']]
        self.layout, self.supports = layout, layout['supports']

    def query_features(self, coordinates):
        """fp16 features [N, input_width] and visibility [N, L] of fp32 coordinates [N, 2] (PackedQuery)."""
        if coordinates.dtype != torch.float32 or coordinates.ndim != 2 or coordinates.shape[1] != 2:
            raise ValueError(f'coordinates must be fp32 [N, 2], got {coordinates.dtype} {tuple(coordinates.shape)}')
        if coordinates.requires_grad:
            raise ValueError('the planes take no gradient with respect to the coordinates')
        return PackedQuery.apply(coordinates.contiguous(), self.grid, self.descriptors, self.node_bitmap,
                                 self.node_prefix, self.bitmap, self.input_width)

    @torch.no_grad()
    def _initialize_plane(self, level):
        """First opening of a level: N(0, feature_init_std) over the whole native plane ([points, max(2, F)], drawn
        with torch's CUDA generator at plane_seed), kept at the closure nodes only."""
        if self.initialized_planes[level]:
            raise RuntimeError(f'level {level} was already initialised')
        entry = self.layout['levels'][level]
        device = self.grid.device
        draw = torch.empty((entry['native_plane_points'], max(2, entry['plane_dim'])), dtype=torch.float32,
                           device=device)
        draw.normal_(0., self.config['feature_init_std'],
                     generator=torch.Generator(device=device).manual_seed(plane_seed(self.config['seed'], level)))
        kept = draw.index_select(0, entry['nodes'].to(device))[:, :entry['plane_dim']].reshape(-1)
        self.grid[entry['plane_offset']:entry['plane_offset'] + kept.numel()].copy_(kept)
        self.initialized_planes[level] = True

    def _check_new_support(self, level, support):
        resolution = self.config['resolutions'][level]
        if level != self.active_prefix or not 2 <= level < self.n_levels:
            raise ValueError(f'level {level} is not the next level to open (active prefix {self.active_prefix})')
        if self.initialized_planes[level] or bool(self.supports[level].any()):
            raise RuntimeError(f'level {level} is open already')
        if support.device.type != 'cpu' or support.dtype != torch.bool or tuple(support.shape) != (resolution**2,):
            raise ValueError(f'a support is a flat CPU bool tensor of R^2 = {resolution**2} cells')
        nodes = int(plane_index_device(support.to(self.grid.device), resolution, with_nodes=False)[3])
        if not 0 < nodes <= self.plane_node_caps[level]:
            raise ValueError(f'the support closes over {nodes} nodes; level {level} takes 1..{self.plane_node_caps[level]}')

    @torch.no_grad()
    def activate_support(self, level, support):
        """Open `level` on the chosen cells: every level's index rebuilt on the GPU, the grid storage kept in place,
        the new level's rows drawn once.  Returns the activation report."""
        self._check_new_support(level, support)
        device, storage = self.grid.device, self.grid.data_ptr()
        supports = [s.to(device) for s in self.supports]
        supports[level] = support.to(device)
        self._install(make_layout_device(self.config, supports, self.plane_dims, self.plane_node_caps), device)
        self._initialize_plane(level)
        if self.grid.data_ptr() != storage:
            raise AssertionError('opening a level moved the grid storage')
        entry = self.layout['levels'][level]
        return {'level': level, 'initialized_once': True, 'grid_storage_unchanged': True,
                'original_dense_f2_seed': plane_seed(self.config['seed'], level),
                'native_dense_draw_shape': [entry['native_plane_points'], max(2, self.plane_dims[level])],
                'selected_nodes': entry['nodes'].numel()}

    def set_active_prefix(self, prefix):
        if not isinstance(prefix, int) or not 2 <= prefix <= self.n_levels:
            raise ValueError(f'the active prefix is an integer in 2..{self.n_levels}')
        self.active_prefix = prefix
        self.level_active.copy_(torch.arange(self.n_levels, device=self.grid.device) < prefix)
        self.feature_active.copy_((self.feature_levels < prefix).to(torch.float16))

    def gates(self, raw, visible):
        """Per-level weights of the decoder input: the router's sigmoid/softplus gate (1 for the first K levels,
        and for every level while only those are open), zero for hidden or inactive levels."""
        k = self.gate_coarse_levels_K
        if self.gate is None:
            return None
        if self.active_prefix > k:
            learned = router_weights(self.gate(raw)[:, :self.n_levels].float(),
                                     self.config.get('router_output_activation', 'sigmoid'))
            learned[:, :k] = 1.0
        else:
            learned = torch.ones(visible.shape, dtype=torch.float32, device=raw.device)
        return learned * (visible & self.level_active).float()

    def forward(self, coordinates):
        raw, visible = self.query_features(coordinates)
        raw = raw * self.feature_active
        weights = self.gates(raw, visible)
        if weights is not None:
            raw = raw * weights.to(raw.dtype).index_select(1, self.feature_levels)
        return self.decoder(raw).float()[:, :3]

    def storage_stats(self):
        """Parameter and index storage (the key set of odie/model.py:281-314)."""
        nbytes = lambda t: t.numel() * t.element_size()  # noqa: E731
        grid = self.grid.numel()
        gate = self.gate.params.numel() if self.gate is not None else 0
        heads = gate + self.decoder.params.numel()
        words, prefixes = nbytes(self.node_bitmap), nbytes(self.node_prefix)
        cells, descriptors = nbytes(self.bitmap), nbytes(self.descriptors)
        flags = nbytes(self.level_active) + nbytes(self.feature_active)
        stats = dict(actual_params=grid + heads, grid_params=grid, head_params=heads, gate_params=gate,
                     decoder_params=self.decoder.params.numel(), router_enabled=self.router_enabled, axis_params=0,
                     plane_params=grid, plane_caps=self.plane_node_caps)
        for key, per_param in (('fp16_parameter_payload_bytes', 2), ('fp32_master_bytes', 4),
                               ('adam_moment_bytes', 8), ('full_gradient_bytes', 4)):
            stats[key] = per_param * (grid + heads)
        stats.update(index_bytes=words + prefixes, node_bitmap_bytes=words, node_prefix_bytes=prefixes,
                     bitmap_bytes=cells, descriptor_bytes=descriptors,
                     runtime_index_bytes=words + prefixes + cells + descriptors + nbytes(self.feature_levels) + flags,
                     active_flag_bytes=flags, input_width=self.input_width,
                     native_input_padding=(self.input_width + 15) // 16 * 16, axis_mode='none',
                     active_layers_from_update1=int(self.config.get('initial_active_prefix', 2)),
                     active_prefix=self.active_prefix, gate_coarse_levels_K=int(self.config['coarse_levels']),
                     full_cover_coarse_layers=self.config.get('full_cover_coarse_layers', [0, 1]),
                     plane_dims=self.plane_dims, coordinate_version=COORDINATE_VERSION, layout_version=LAYOUT_VERSION,
                     addressing_version=ADDRESSING_VERSION, query_cuda_launches=1, backward_cuda_launches=1,
                     forward_precision='P01 FP32 geometry and FP16 interpolation chain',
                     gradient_precision='FP16 feature gradient, FP32 interpolation weights and reductions',
                     levels=[{k: v for k, v in entry.items() if k != 'nodes'} for entry in self.layout['levels']])
        return stats


class HashGrid(nn.Module):
    """Hashed multiresolution grid (the TCNN HashGrid of odie/hash_grid.py:8-80, with the published Instant-NGP
    spatial hash) behind the same optional per-level gate and decoder as the planes; every level is open."""

    def __init__(self, config, supports, plane_dims, plane_node_caps):
        super().__init__()
        if supports or config['initial_active_prefix'] != config['n_levels']:
            raise ValueError('a hash grid has no supports and trains every level from the start')
        self.config = deepcopy(config)
        self.router_enabled = config['router_enabled']
        self.n_levels = self.active_prefix = config['n_levels']
        self.gate_coarse_levels_K = config['gate_coarse_levels_K']
        self.input_width = sum(plane_dims)
        self.plane_dims, self.plane_node_caps = list(plane_dims), list(plane_node_caps)
        self.supports = []
        self.records, total = hash_levels(config['hash_encoding'])
        seed = int(config['seed'])
        table = (torch.rand(total, generator=torch.Generator().manual_seed(seed)) * 2 - 1) * 1e-4
        self.grid = nn.Parameter(table.cuda())
        columns = [l for l, dim in enumerate(plane_dims) for _ in range(dim)]
        self.register_buffer('feature_levels', torch.tensor(columns, dtype=torch.int64, device='cuda'),
                             persistent=False)
        self.gate = Head(self.input_width, self.n_levels, 32, 1, (seed + 2000003) % 2**31) if self.router_enabled else None
        self.decoder = Head(self.input_width, 3, 64, 2, (seed + 4000037) % 2**31)
        offsets = np.cumsum([0] + [dim * cap for dim, cap in zip(plane_dims, plane_node_caps)])
        self.layout = dict(levels=[dict(plane_offset=int(o), plane_node_capacity=cap, plane_dim=dim)
                                   for o, dim, cap in zip(offsets[:-1], plane_dims, plane_node_caps)])
        gate = self.gate.params.numel() if self.gate is not None else 0
        expected = (int(offsets[-1]), config['decoder_parameters'], config['gate_parameters'])
        if (self.grid.numel(), self.decoder.params.numel(), gate) != expected:
            raise RuntimeError('the hash grid or its heads differ from the configured budget')

    def set_active_prefix(self, prefix):
        if prefix != self.n_levels:
            raise ValueError('a hash grid always trains every level')

    def forward(self, coordinates):
        raw = HashQuery.apply(coordinates.contiguous(), self.grid, self.records, self.input_width)
        if self.gate is not None:
            weights = router_weights(self.gate(raw)[:, :self.n_levels].float(), self.config['router_output_activation'])
            weights[:, :self.gate_coarse_levels_K] = 1.0
            raw = raw * weights.to(raw.dtype).index_select(1, self.feature_levels)
        return self.decoder(raw).float()[:, :3]

    def storage_stats(self):
        grid, decoder = self.grid.numel(), self.decoder.params.numel()
        gate = self.gate.params.numel() if self.gate is not None else 0
        return dict(actual_params=grid + gate + decoder, grid_params=grid, head_params=gate + decoder,
                    gate_params=gate, decoder_params=decoder, router_enabled=self.router_enabled,
                    plane_caps=self.plane_node_caps, fp16_parameter_payload_bytes=2 * (grid + gate + decoder),
                    input_width=self.input_width, layout_version='hash-grid-v1',
                    addressing_version='instant-ngp-spatial-hash')


class RoutedExperts(nn.Module):
    """Routed multi-expert hash-grid encoding with a shared decoder (no reference counterpart).

    A coarse shared hash grid (``router_encoding``) feeds the router MLP
    (W -> 32 -> 32 -> 16 or 64 logits, top-1); coordinate i is then encoded by
    its expert's own hash grid (``hash_encoding``; the tables of the experts held
    here are one flat fp32 parameter, expert-major) and the features, scaled by
    the router probability rounded to fp16, go through the shared decoder
    (W -> 64 -> 64 -> 3).

    Spatial expert ownership (``bands`` > 1): the full image of ``image_rows``
    rows is cut into equal row bands, band b owns experts [b * per, (b + 1) *
    per) with per = ``experts_per_band``, and a coordinate chooses among its
    band's experts only.  A data-parallel rank holds bands [first_band,
    first_band + bands_held) and only their expert tables; every expert's table
    is seeded by its global number, so the model is the same however the bands
    are split.  Training runs in the native runtime; this module's forward is the
    evaluation/decode path.
    """

    def __init__(self, config):
        super().__init__()
        self.config = deepcopy(config)
        self.experts = int(config['experts'])  # of the whole model
        self.bands = int(config.get('bands', 1))
        self.per_band = int(config.get('experts_per_band', self.experts))
        self.first_band = int(config.get('first_band', 0))
        self.bands_held = int(config.get('bands_held', self.bands))
        if self.per_band * self.bands != self.experts or not 1 <= self.experts <= 64:
            raise ValueError('experts must be bands x experts_per_band, within 1..64')
        if self.bands > 1 and self.per_band not in (8, 16):
            raise ValueError('banded routing takes 8 or 16 experts per band')
        if not (0 <= self.first_band and self.first_band + self.bands_held <= self.bands and self.bands_held >= 1):
            raise ValueError('the bands held must lie within the bands')
        self.image_rows = int(config.get('image_rows', 2))
        self.experts_held = self.bands_held * self.per_band
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
        scale = float(config.get('grid_init', 1e-4))
        first_expert = self.first_band * self.per_band
        tables = [(torch.rand(self.expert_total, generator=torch.Generator().manual_seed(seed + 7919 * (e + 1))) * 2 - 1)
                  * scale for e in range(first_expert, first_expert + self.experts_held)]
        self.grid = nn.Parameter(torch.cat(tables).cuda())
        self.router_grid = nn.Parameter(((torch.rand(router_total, generator=torch.Generator().manual_seed(seed)) * 2 - 1)
                                         * float(config.get('router_init', 1e-1))).cuda())
        self.gate = Head(self.input_width, router_out(self.experts), 32, 2, (seed + 2000003) % 2**31)  # the router MLP
        self.decoder = Head(self.input_width, 3, 64, 2, (seed + 4000037) % 2**31)
        self.supports = []

    @property
    def banding(self):
        """The router's banding (router.cuh Banding) for the bands held here."""
        return dict(bands=self.bands, first_band=self.first_band, per_band=self.per_band, rows=self.image_rows)

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
        """(local expert, probability, live logits) of full-image coordinates."""
        with torch.no_grad():
            features = HashQuery.apply(coordinates.contiguous(), self.router_grid, self.router_records, self.input_width)
            return route(features, self.gate.params, self.experts_held, coordinates, self.banding)

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
                    head_params=heads, experts=self.experts, experts_held=self.experts_held, bands=self.bands,
                    fp16_parameter_payload_bytes=2 * (grid + router_grid + heads),
                    input_width=self.input_width, addressing_version='instant-ngp-spatial-hash')


def build_model(config, supports, plane_dims, plane_node_caps, **kwargs):
    if config['representation'] == 'routed_experts':
        return RoutedExperts(config)
    if config['representation'] == 'hash_grid':
        return HashGrid(config, supports, plane_dims, plane_node_caps)
    return PackedXYPlanes(config, supports, plane_dims, plane_node_caps, **kwargs)
