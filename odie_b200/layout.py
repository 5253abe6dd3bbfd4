"""Packed-plane layout: supports -> descriptors, node index and cell bitmaps.

Host-side (CPU) construction of the addressing tables that the encode kernels
read.  Same contract as the reference (odie/model.py:33-118):
  descriptor row [R, points, plane offset, node word offset, cell bitmap
  offset, F, feature offset, direct] (int32), points = align8(R^2);
  node index 'node-bitmap64-exclusive-prefix32': one uint64 presence word per
  64 nodes plus the exclusive popcount prefix of the words (int32);
  cell bitmap: one bit per cell, LSB-first, R^2 padded to align8.
"""
import numpy as np
import torch

COORDINATE_VERSION = 'unit-endpoints-native-fmaf-half-cell-align8-modulo-v1'
LAYOUT_VERSION = 'packed-xy-only-native-closure-v1'
ADDRESSING_VERSION = 'node-bitmap64-exclusive-prefix32-v1'
INT32_MAX = 2**31 - 1


def align8(value):
    return -(-int(value) // 8) * 8


def plane_closure(support, resolution):
    """Sorted unique corner nodes of the selected cells, modulo align8(R^2) (odie/model.py:37-40)."""
    points = align8(resolution * resolution)
    cells = np.flatnonzero(np.asarray(support, dtype=bool))
    present = np.zeros(points, dtype=bool)
    for delta in (0, 1, resolution, resolution + 1):
        present[(cells + delta) % points] = True
    return torch.from_numpy(np.flatnonzero(present).astype(np.int64))


def make_node_index(nodes, points):
    """Presence words and exclusive word ranks of sorted unique nodes (odie/model.py:43-61)."""
    if not isinstance(points, int) or not 0 < points <= INT32_MAX:
        raise ValueError('Native node universe must fit positive int32 addressing')
    if nodes.device.type != 'cpu' or nodes.dtype != torch.int64 or nodes.ndim != 1:
        raise ValueError('Nodes must be a flat CPU int64 tensor')
    ids = nodes.numpy()
    if ids.size and (ids[0] < 0 or ids[-1] >= points or np.any(np.diff(ids) <= 0)):
        raise ValueError('Nodes must be sorted, unique and inside the native universe')
    words = -(-points // 64)
    present = np.zeros(words * 64, dtype=bool)
    present[ids] = True
    packed = np.packbits(present.reshape(words, 64), axis=1, bitorder='little')
    bitmap = np.ascontiguousarray(packed).view('<u8').reshape(words)
    counts = present.reshape(words, 64).sum(axis=1)
    prefix = (np.cumsum(counts) - counts).astype(np.int32)
    return torch.from_numpy(bitmap.astype(np.uint64)), torch.from_numpy(prefix)


def cell_bitmap(support, resolution):
    padded = np.zeros(align8(resolution * resolution), dtype=bool)
    padded[:resolution * resolution] = np.asarray(support, dtype=bool)
    return torch.from_numpy(np.packbits(padded, bitorder='little'))


def check_gate_k(config):
    """The number of leading levels the gate leaves at weight 1 (must equal coarse_levels)."""
    k = int(config.get('gate_coarse_levels_K', config['coarse_levels']))
    if int(config['coarse_levels']) != k or not 0 <= k <= int(config['n_levels']):
        raise ValueError(f'gate K = {k} must equal coarse_levels and lie within 0..n_levels')
    return k


def _check_plan(config, supports, plane_dims, plane_node_caps):
    """The planes configuration this layout can express: one support, feature count and node cap per level."""
    levels = int(config['n_levels'])
    lengths = {len(config['resolutions']), len(supports), len(plane_dims), len(plane_node_caps)}
    if lengths != {levels}:
        raise ValueError(f'resolutions, supports, feature counts and node caps must each list {levels} levels')
    if any(int(f) not in (1, 2, 4) for f in plane_dims):
        raise ValueError('every level holds 1, 2 or 4 features per node')
    if config['representation'] != 'xy_planes':
        raise ValueError('a packed-plane layout needs the xy_planes representation')
    if config['gate_topology'] != 'shared' or config['gate_position'] != 'feature':
        raise ValueError('the gate is one shared MLP applied to the features')
    check_gate_k(config)


class _Packer:
    """Running offsets of the packed layout: parameters, feature columns, node-index words, cell-bitmap bytes."""

    def __init__(self):
        self.params = self.column = self.words = self.cell_bytes = 0
        self.rows, self.node_words, self.prefixes, self.cell_maps, self.levels, self.supports = [], [], [], [], [], []

    def add(self, level, resolution, dim, cap, support, must_be_full):
        """A level whose support is a CPU bool tensor: closure, node index and cell bitmap built on the host."""
        if support.device.type != 'cpu' or support.dtype != torch.bool or tuple(support.shape) != (resolution ** 2,):
            raise ValueError(f'level {level}: a support is a flat CPU bool tensor of R^2 = {resolution ** 2} cells')
        if must_be_full and not bool(support.all()):
            raise ValueError(f'level {level} is one of the initial levels and must cover every cell')
        support = support.clone()
        points = align8(resolution * resolution)
        nodes = plane_closure(support.numpy(), resolution)
        index = make_node_index(nodes, points) if nodes.numel() != points else None
        self.place(level, resolution, dim, cap, support, nodes, nodes.numel(), int(support.sum()), index,
                   cell_bitmap(support.numpy(), resolution))

    def place(self, level, resolution, dim, cap, support, nodes, count, allowed, index, cells):
        """Append one level: its descriptor row, node index (None for a full plane) and cell bitmap."""
        points = align8(resolution * resolution)
        if cap % 8 or not count <= cap <= points:
            raise ValueError(f'level {level}: node cap {cap} must be a multiple of 8 between the closure '
                             f'({count} nodes) and the plane ({points})')
        if points > INT32_MAX or self.params + cap * dim > INT32_MAX:
            raise ValueError(f'level {level}: the layout outgrows int32 offsets')
        direct = count == points  # a full plane needs no node index
        word_start, words = -1, 0
        if not direct:
            bits, prefix = index
            word_start, words = self.words, bits.numel()
            self.node_words.append(bits)
            self.prefixes.append(prefix)
            self.words += words
        self.rows.append([resolution, points, self.params, word_start, self.cell_bytes, dim, self.column, int(direct)])
        self.levels.append({'level': level, 'resolution': resolution, 'plane_dim': dim, 'allowed_cells': allowed,
                            'plane_retained_nodes': count, 'plane_node_capacity': cap,
                            'plane_unused_slots': cap - count, 'native_plane_points': points,
                            'plane_offset': self.params, 'feature_offset': self.column, 'nodes': nodes,
                            'node_index_words': words, 'direct_node_access': direct})
        self.cell_maps.append(cells)
        self.supports.append(support)
        self.params += cap * dim
        self.column += dim
        self.cell_bytes += cells.numel()

    def tables(self):
        def joined(parts, dtype):
            return torch.cat(parts) if parts else torch.empty(0, dtype=dtype)
        device = self.cell_maps[0].device if self.cell_maps else 'cpu'
        return {'descriptors': torch.tensor(self.rows, dtype=torch.int32, device=device),
                'node_bitmap': joined(self.node_words, torch.uint64), 'node_prefix': joined(self.prefixes, torch.int32),
                'bitmap': torch.cat(self.cell_maps), 'levels': self.levels, 'supports': self.supports,
                'params': self.params, 'input_width': self.column}


def make_layout(config, supports, plane_dims, plane_node_caps):
    """Descriptor rows and index tables of every plane, built on the host (the contract of odie/model.py:64-118):
    levels packed in order, each holding cap x F parameters, its features at the next columns, its node index
    words and cell-bitmap bytes appended after the previous level's."""
    _check_plan(config, supports, plane_dims, plane_node_caps)
    initial = int(config['initial_active_prefix'])
    packer = _Packer()
    for level, (resolution, dim, cap, support) in enumerate(zip(config['resolutions'], plane_dims, plane_node_caps,
                                                                 supports)):
        packer.add(level, int(resolution), int(dim), int(cap), support, level < initial)
    return packer.tables()


def float32(value):
    return float(np.float32(value))


def hash_grid_layout(encoding):
    """fp32 grid scales, resolutions and aligned capacities of a HashGrid encoding (odie/config.py:83-94)."""
    levels = int(encoding['n_levels'])
    base = int(encoding['base_resolution'])
    log2t = int(encoding['log2_hashmap_size'])
    growth = float32(encoding['per_level_scale'])
    if not 2 <= levels <= 20 or base < 2 or not 3 <= log2t <= 30 or not growth > 1:
        raise ValueError('Invalid HashGrid encoding')
    log_growth = float32(np.log2(growth))
    scales, resolutions, capacities = [], [], []
    for i in range(levels):
        scale = float32(float32(float32(2.0 ** float32(i * log_growth)) * base) - 1)
        resolution = int(np.ceil(scale)) + 1
        scales.append(scale)
        resolutions.append(resolution)
        capacities.append(min(align8(resolution * resolution), 1 << log2t))
    return scales, resolutions, capacities


def hash_levels(encoding):
    """Per-level records for the hashed encode kernels (odie_hash_level of include/odie_b200.h)."""
    scales, resolutions, capacities = hash_grid_layout(encoding)
    features = int(encoding['n_features_per_level'])
    out, offset = [], 0
    for level, (s, r, cap) in enumerate(zip(scales, resolutions, capacities)):
        out.append(dict(scale=s, resolution=r, capacity=cap, offset=offset, features=features,
                        column=level * features, hashed=int(r * r > cap)))
        offset += cap * features
    return out, offset


def plane_index_device(support, resolution, with_nodes=True, stream=None):
    """Node presence words, exclusive word prefix, cell bitmap, node count and (optionally) the sorted closure of
    one level, built on the GPU (odie_plane_index).  support: CUDA bool [R^2].  Returns device tensors and the node
    count as a device int64 scalar; nothing is synchronised."""
    from . import _lib
    if not support.is_cuda or support.dtype != torch.bool or tuple(support.shape) != (resolution * resolution,):
        raise ValueError('support must be a flat CUDA bool R^2 tensor')
    device = support.device
    points = align8(resolution * resolution)
    words = -(-points // 64)
    node_bitmap = torch.empty(words, dtype=torch.uint64, device=device)
    prefix = torch.empty(words, dtype=torch.int32, device=device)
    bitmap = torch.empty(points // 8, dtype=torch.uint8, device=device)
    count = torch.empty((), dtype=torch.int64, device=device)
    nodes = torch.empty(points, dtype=torch.int64, device=device) if with_nodes else None
    lib = _lib.library()
    scratch = torch.empty(int(lib.odie_plane_index_scratch(resolution)), dtype=torch.int32, device=device)
    support = support.contiguous()
    _lib.check(lib.odie_plane_index(support.data_ptr(), resolution, node_bitmap.data_ptr(), prefix.data_ptr(),
                                    bitmap.data_ptr(), count.data_ptr(), _lib.ptr(nodes), scratch.data_ptr(),
                                    _lib.stream_handle(stream)), 'odie_plane_index')
    return node_bitmap, prefix, bitmap, count, nodes


def make_layout_device(config, supports, plane_dims, plane_node_caps):
    """make_layout with every level's closure, node index and cell bitmap built on the GPU (odie_plane_index).

    supports: CUDA bool [R^2] tensors.  Same checks and the same tables as make_layout, as device tensors (the
    'nodes' entries are device int64 tensors); one host synchronisation reads every level's node count."""
    _check_plan(config, supports, plane_dims, plane_node_caps)
    resolutions = [int(r) for r in config['resolutions']]
    built = []
    for level, (r, support) in enumerate(zip(resolutions, supports)):
        if not support.is_cuda or support.dtype != torch.bool or tuple(support.shape) != (r * r,):
            raise ValueError(f'level {level}: a support is a flat CUDA bool tensor of R^2 = {r * r} cells')
        built.append(plane_index_device(support, r))
    summary = torch.stack([torch.stack((b[3], s.sum(), s.all().long())) for b, s in zip(built, supports)]).cpu().tolist()
    initial = int(config['initial_active_prefix'])
    packer = _Packer()
    for level, (r, dim, cap, support, (bits, prefix, cells, _, nodes), (count, allowed, full)) in enumerate(
            zip(resolutions, plane_dims, plane_node_caps, supports, built, summary)):
        if level < initial and not full:
            raise ValueError(f'level {level} is one of the initial levels and must cover every cell')
        packer.place(level, r, int(dim), int(cap), support.clone(), nodes[:count], int(count), int(allowed),
                     (bits, prefix), cells)
    return packer.tables()
