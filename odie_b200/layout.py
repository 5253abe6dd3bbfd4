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
    k = int(config.get('gate_coarse_levels_K', config['coarse_levels']))
    if not 0 <= k <= int(config['n_levels']) or int(config['coarse_levels']) != k:
        raise ValueError('Gate K must agree with coarse_levels and remain within declared level count')
    return k


def make_layout(config, supports, plane_dims, plane_node_caps):
    """Descriptors and index tables of all planes (odie/model.py:64-118)."""
    resolutions = [int(r) for r in config['resolutions']]
    levels = int(config['n_levels'])
    if not (len(resolutions) == len(supports) == len(plane_dims) == len(plane_node_caps) == levels):
        raise ValueError('Require aligned level descriptors and F1/F2/F4 features')
    if any(f not in (1, 2, 4) for f in plane_dims):
        raise ValueError('Require aligned level descriptors and F1/F2/F4 features')
    if config['representation'] != 'xy_planes':
        raise ValueError('XY-only representation is required')
    check_gate_k(config)
    if config['gate_topology'] != 'shared' or config['gate_position'] != 'feature':
        raise ValueError('Preserve the shared feature gate')
    initial = int(config['initial_active_prefix'])
    descriptors, bitmaps, node_words, prefixes, info, clean = [], [], [], [], [], []
    params = column = word_offset = byte_offset = 0
    for level in range(levels):
        r, dim, cap, support = resolutions[level], int(plane_dims[level]), int(plane_node_caps[level]), supports[level]
        if support.device.type != 'cpu' or support.dtype != torch.bool or tuple(support.shape) != (r * r,):
            raise ValueError('Support must be a flat CPU bool R^2 tensor')
        if level < initial and not bool(support.all()):
            raise ValueError('Declared initial full-cover supports must remain full')
        support = support.clone()
        points = align8(r * r)
        nodes = plane_closure(support.numpy(), r)
        if cap % 8 or not nodes.numel() <= cap <= points:
            raise ValueError('Aligned node capacity must contain the complete interpolation closure')
        if points > INT32_MAX or params + cap * dim > INT32_MAX:
            raise ValueError('Native points and packed offsets must fit int32 addressing')
        direct = nodes.numel() == points
        if direct:
            word_start = -1
            words = 0
        else:
            bits, prefix = make_node_index(nodes, points)
            word_start, words = word_offset, bits.numel()
            node_words.append(bits)
            prefixes.append(prefix)
            word_offset += words
        bitmap = cell_bitmap(support.numpy(), r)
        descriptors.append([r, points, params, word_start, byte_offset, dim, column, int(direct)])
        info.append({'level': level, 'resolution': r, 'plane_dim': dim, 'allowed_cells': int(support.sum()),
                     'plane_retained_nodes': nodes.numel(), 'plane_node_capacity': cap,
                     'plane_unused_slots': cap - nodes.numel(), 'native_plane_points': points,
                     'plane_offset': params, 'feature_offset': column, 'nodes': nodes,
                     'node_index_words': words, 'direct_node_access': direct})
        bitmaps.append(bitmap)
        clean.append(support)
        params += cap * dim
        column += dim
        byte_offset += bitmap.numel()
    return {'descriptors': torch.tensor(descriptors, dtype=torch.int32),
            'node_bitmap': torch.cat(node_words) if node_words else torch.empty(0, dtype=torch.uint64),
            'node_prefix': torch.cat(prefixes) if prefixes else torch.empty(0, dtype=torch.int32),
            'bitmap': torch.cat(bitmaps), 'levels': info, 'supports': clean,
            'params': params, 'input_width': column}


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
    """make_layout with the per-level closure, node index and cell bitmap built on the GPU.

    supports: CUDA bool [R^2] tensors.  Same validation and the same tables as make_layout (device tensors; the
    'nodes' entries are device int64 tensors); one host synchronisation reads all levels' node counts."""
    resolutions = [int(r) for r in config['resolutions']]
    levels = int(config['n_levels'])
    if not (len(resolutions) == len(supports) == len(plane_dims) == len(plane_node_caps) == levels):
        raise ValueError('Require aligned level descriptors and F1/F2/F4 features')
    if any(f not in (1, 2, 4) for f in plane_dims):
        raise ValueError('Require aligned level descriptors and F1/F2/F4 features')
    if config['representation'] != 'xy_planes':
        raise ValueError('XY-only representation is required')
    check_gate_k(config)
    if config['gate_topology'] != 'shared' or config['gate_position'] != 'feature':
        raise ValueError('Preserve the shared feature gate')
    initial = int(config['initial_active_prefix'])
    built = []
    for level in range(levels):
        r, support = resolutions[level], supports[level]
        if not support.is_cuda or support.dtype != torch.bool or tuple(support.shape) != (r * r,):
            raise ValueError('Support must be a flat CUDA bool R^2 tensor')
        built.append(plane_index_device(support, r))
    counts = torch.stack([b[3] for b in built]).cpu().tolist()
    full = torch.stack([s.all() for s in supports]).cpu().tolist()
    allowed = torch.stack([s.sum() for s in supports]).cpu().tolist()
    descriptors, bitmaps, node_words, prefixes, info, clean = [], [], [], [], [], []
    params = column = word_offset = byte_offset = 0
    for level in range(levels):
        r, dim, cap = resolutions[level], int(plane_dims[level]), int(plane_node_caps[level])
        if level < initial and not full[level]:
            raise ValueError('Declared initial full-cover supports must remain full')
        points = align8(r * r)
        count = int(counts[level])
        if cap % 8 or not count <= cap <= points:
            raise ValueError('Aligned node capacity must contain the complete interpolation closure')
        if points > INT32_MAX or params + cap * dim > INT32_MAX:
            raise ValueError('Native points and packed offsets must fit int32 addressing')
        bits, prefix, bitmap, _, nodes = built[level]
        direct = count == points
        if direct:
            word_start, words = -1, 0
        else:
            word_start, words = word_offset, bits.numel()
            node_words.append(bits)
            prefixes.append(prefix)
            word_offset += words
        descriptors.append([r, points, params, word_start, byte_offset, dim, column, int(direct)])
        info.append({'level': level, 'resolution': r, 'plane_dim': dim, 'allowed_cells': int(allowed[level]),
                     'plane_retained_nodes': count, 'plane_node_capacity': cap, 'plane_unused_slots': cap - count,
                     'native_plane_points': points, 'plane_offset': params, 'feature_offset': column,
                     'nodes': nodes[:count], 'node_index_words': words, 'direct_node_access': direct})
        bitmaps.append(bitmap)
        clean.append(supports[level].clone())
        params += cap * dim
        column += dim
        byte_offset += bitmap.numel()
    device = supports[0].device
    return {'descriptors': torch.tensor(descriptors, dtype=torch.int32, device=device),
            'node_bitmap': torch.cat(node_words) if node_words else torch.empty(0, dtype=torch.uint64, device=device),
            'node_prefix': torch.cat(prefixes) if prefixes else torch.empty(0, dtype=torch.int32, device=device),
            'bitmap': torch.cat(bitmaps), 'levels': info, 'supports': clean,
            'params': params, 'input_width': column}
