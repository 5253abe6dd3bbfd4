"""Benchmark workloads: seeded synthetic images plus the model layouts they train.

c2-planes: the reference's own method (packed multiresolution planes with a
per-level sigmoid router, odie/model.py) at the routed-expert benchmark's image shape
(2040 x 1356 u8, blobs + gratings + 1/f^2 noise) and batch (2^20 coords).  The
layout is the reference's DIV2K plan (odie/config.py:resolve at this image
class; resolutions 8..1020, 13 full-cover levels, 3 on-demand levels with
caps 181112/181112/181120, results/div2k_50/0028/odie/metrics.json), with the
on-demand supports chosen as the top cells of a seeded smooth residual field,
trimmed to their node caps.

c2-experts: the routed-expert benchmark itself -- 16 routed experts, each with its own
hash grid (L=16, F=2, T=2^16, base resolution 16, per-level scale 1.5, tables
U(-1e-4, 1e-4)), a top-1 router (W -> 32 -> 32 -> 16) over a coarse shared grid
(L=16, F=2, T=2^12, base 4, scale 1.2: resolutions 4..62, all dense, tables
U(-0.1, 0.1) so that the initial routing already splits the image), and the
shared 64-wide decoder, on the same 2040 x 1356 image with 2^20 coords.

c4-experts: the gigapixel benchmark -- a 32768 x 32768 procedural image (fractal
1/f^2 noise, sharp-edged Voronoi regions, a 64 x 64-cell texture atlas), 64 routed
experts under a 50 MiB fp16 budget (T = 2^14 per expert level: 24.4 M parameters,
46.5 MiB with the router grid and heads), owned spatially by 8 row bands of 8
experts each (a coordinate chooses among its band's experts), 20 % of the 256 x
256 tiles allocated, 2^22 coordinates per step and GPU.  Rank r of N holds bands
[8r/N, 8(r+1)/N) and their experts; the model is the same at every N.

c3-experts: the on-demand allocation benchmark -- a 4096 x 4096
image (1/f^2 noise + 200 sharp polygons), 8 routed experts with T = 2^17, the
residual of every 256 x 256 tile of the current model's decode, the top 30 %
tiles allocated (the fine expert levels restricted to their cells), and 2^21
coordinates per step, 70 % of them drawn from the allocated tiles.

Multi-GPU (c2, c3): rank r of N trains the model of row band r of the image (its
own tables: spatial ownership); the heads are shared.  c4 splits one fixed model.
"""
import math

import numpy as np

import torch

from . import layout as host_layout
from .data import ByteTarget, pink_noise, procedural_image, synthetic_image
from .model import PackedXYPlanes, RoutedExperts
from .parallel import band_rows

DIV2K_RESOLUTIONS = [8, 11, 15, 21, 29, 40, 56, 77, 106, 147, 203, 280, 387, 534, 738, 1020]
DIV2K_SPARSE_CAPS = {13: 181112, 14: 181112, 15: 181120}


def plane_model_config(resolutions, dims, initial, seed=1729, batch=1 << 20):
    width = (sum(dims) + 15) // 16 * 16
    return dict(resolutions=list(resolutions), n_levels=len(resolutions), representation='xy_planes', coarse_levels=0,
                gate_coarse_levels_K=0, gate_topology='shared', gate_position='feature', initial_active_prefix=initial,
                router_enabled=True, router_output_activation='sigmoid', seed=seed, feature_init_std=1e-3,
                gate_parameters=width * 32 + 32 * 16, decoder_parameters=width * 64 + 64 * 64 + 64 * 16,
                grid_lr=1e-2, gate_lr=1e-3, decoder_lr=1e-3, batch_size=batch)


def capped_support(resolution, cap, seed):
    """Cells above a threshold of a smooth seeded field, the threshold raised until the closure fits the cap."""
    field = pink_noise(resolution, resolution, seed)[..., 0].reshape(-1).numpy()
    lo, hi = float(field.min()), float(field.max())
    best = np.zeros(resolution * resolution, dtype=bool)
    for _ in range(40):
        mid = (lo + hi) / 2
        support = field > mid
        if host_layout.plane_closure(support, resolution).numel() <= cap:
            best, hi = support, mid
        else:
            lo = mid
    return best


def c2_planes(seed=1729, batch=1 << 20, band=(0, 1)):
    """(config, supports, dims, caps, rgb u8 [H*W, 3] on CPU, shape) of rank band[0] of band[1] (row bands)."""
    rgb, shape = synthetic_image('c2', seed=seed)
    rgb, (height, width) = band_of(rgb, shape, band)
    rank, ranks = band
    dims = [2] * 16
    supports, caps = [], []
    for level, r in enumerate(DIV2K_RESOLUTIONS):
        points = host_layout.align8(r * r)
        if level in DIV2K_SPARSE_CAPS:
            cap = DIV2K_SPARSE_CAPS[level]
            supports.append(torch.from_numpy(capped_support(r, cap, seed + 31 * level + rank)))
            caps.append(cap)
        else:
            supports.append(torch.ones(r * r, dtype=torch.bool))
            caps.append(points)
    config = plane_model_config(DIV2K_RESOLUTIONS, dims, 13, seed=seed + rank, batch=batch)
    return config, supports, dims, caps, rgb, (height, width)


def build_plane_model(config, supports, dims, caps, rgb, device='cuda'):
    model = PackedXYPlanes(config, supports, dims, caps)
    target = ByteTarget(rgb.to(device))
    planes = [torch.nn.Parameter(model.grid[l['plane_offset']:l['plane_offset'] + l['plane_node_capacity'] *
                                            l['plane_dim']].detach()) for l in model.layout['levels']]
    return model, target, planes


EXPERT_ENCODING = dict(otype='HashGrid', n_levels=16, n_features_per_level=2, log2_hashmap_size=16,
                       base_resolution=16, per_level_scale=1.5)
ROUTER_ENCODING = dict(otype='HashGrid', n_levels=16, n_features_per_level=2, log2_hashmap_size=12,
                       base_resolution=4, per_level_scale=1.2)


def experts_config(experts=16, seed=1729, batch=1 << 20, encoding=None, router_encoding=None):
    return dict(representation='routed_experts', experts=experts, seed=seed, grid_init=1e-4, router_init=0.1,
                hash_encoding=dict(encoding or EXPERT_ENCODING), router_encoding=dict(router_encoding or ROUTER_ENCODING),
                grid_lr=1e-2, gate_lr=1e-3, decoder_lr=1e-3, batch_size=batch)


def band_of(rgb, shape, band):
    """The u8 pixels and shape of row band band[0] of band[1] (odie_b200.parallel.band_rows)."""
    rank, ranks = band
    height, width = shape
    if ranks == 1:
        return rgb, shape
    first, last = band_rows(height, rank, ranks)
    return rgb.reshape(height, width, 3)[first:last].reshape(-1, 3).contiguous(), (last - first, width)


def c2_experts(seed=1729, batch=1 << 20, band=(0, 1)):
    """(config, rgb u8 [H*W, 3] on CPU, shape) of rank band[0] of band[1] (row bands)."""
    rgb, shape = synthetic_image('c2', seed=seed)
    rgb, shape = band_of(rgb, shape, band)
    return experts_config(seed=seed + band[0], batch=batch), rgb, shape


def build_expert_model(config, rgb, device='cuda'):
    model = RoutedExperts(config)
    return model, ByteTarget(rgb.to(device)), [model.grid]


C3_TILE = 256


def c3_experts(seed=1729, batch=1 << 21, band=(0, 1), device='cuda'):
    """(config, rgb u8 [H*W, 3] on CPU, shape) of the allocation benchmark for rank band[0] of band[1]."""
    rgb, shape = synthetic_image('c3', seed=seed, device=device)
    rgb, shape = band_of(rgb.cpu(), shape, band)
    encoding = dict(EXPERT_ENCODING, log2_hashmap_size=17)
    return experts_config(experts=8, seed=seed + band[0], batch=batch, encoding=encoding), rgb, shape


C4_SHAPE = (32768, 32768)
C4_BANDS, C4_PER_BAND = 8, 8
C4_TILE, C4_ALLOCATED = 256, 0.2
C4_ENCODING = dict(EXPERT_ENCODING, log2_hashmap_size=14)
C4_BUDGET_BYTES = 50 << 20


def c4_experts(seed=1729, batch=1 << 22, band=(0, 1), shape=C4_SHAPE, bands=C4_BANDS, per_band=C4_PER_BAND,
               encoding=None, device='cuda'):
    """(config, rgb u8 [rows * W, 3] on the GPU, (rows, W)) of rank band[0] of band[1]: the rank holds image bands
    [first, first + bands / ranks) -- their rows of the procedural image and their experts."""
    rank, ranks = band
    height, width = shape
    if bands % ranks or height % bands:
        raise ValueError('the ranks must split the bands, and the bands the rows, evenly')
    held = bands // ranks
    first = rank * held
    band_rows = height // bands
    row0, rows = first * band_rows, held * band_rows
    rgb = procedural_image(shape, seed, row0, rows, device=device)
    config = experts_config(experts=bands * per_band, seed=seed, batch=batch, encoding=encoding or C4_ENCODING)
    config.update(bands=bands, experts_per_band=per_band, first_band=first, bands_held=held, image_rows=height,
                  row_offset=row0)
    return config, rgb, (rows, width)


def fp16_payload_bytes(model):
    """fp16 bytes of every parameter of the whole model (all experts, whichever rank holds them)."""
    return 2 * (model.experts * model.expert_total + model.router_grid.numel() + model.gate.params.numel() +
                model.decoder.params.numel())


def allocated_ids(tiles, shape, count, generator, fraction=0.7, tile_px=C3_TILE):
    """count pixel ids: `fraction` of them uniform inside the allocated tiles (tiles: CUDA bool [ty, tx]), the rest
    uniform over the image, in random order."""
    height, width = shape
    device = tiles.device
    chosen = torch.nonzero(tiles.reshape(-1)).reshape(-1)
    inside = int(round(count * fraction)) if chosen.numel() else 0
    pick = chosen[torch.randint(0, chosen.numel(), (inside,), device=device, generator=generator)] if inside else \
        torch.zeros(0, dtype=torch.long, device=device)
    ty, tx = pick // tiles.shape[1], pick % tiles.shape[1]
    y = ty * tile_px + torch.randint(0, tile_px, (inside,), device=device, generator=generator)
    x = tx * tile_px + torch.randint(0, tile_px, (inside,), device=device, generator=generator)
    y, x = y.clamp_(max=height - 1), x.clamp_(max=width - 1)
    rest = torch.randint(0, height * width, (count - inside,), device=device, generator=generator)
    ids = torch.cat((y * width + x, rest))
    return ids[torch.randperm(count, device=device, generator=generator)]


def allocated_stratified_ids(tiles, shape, count, generator, fraction=0.7, tile_px=C3_TILE):
    """count pixel ids with the distribution of allocated_ids, stratified: `fraction` of them spread evenly over the
    allocated tiles (tile t in row-major tile order takes base + (t < extra) samples), each tile's share on a
    jittered columns x rows grid (columns = ceil(sqrt(share)), rows = ceil(share / columns)), then the rest on a
    jittered grid over the whole image; emitted tile by tile, row-major inside each grid, like the reference's
    stratified sampler (odie/data.py:63-80)."""
    height, width = shape
    device = tiles.device
    chosen = torch.nonzero(tiles.reshape(-1)).reshape(-1)
    inside = int(round(count * fraction)) if chosen.numel() else 0
    parts = []
    if inside:
        n_tiles = chosen.numel()
        share = torch.full((n_tiles,), inside // n_tiles, dtype=torch.long, device=device)
        share[:inside % n_tiles] += 1
        first = torch.cumsum(share, 0) - share
        tile = torch.repeat_interleave(torch.arange(n_tiles, device=device), share, output_size=inside)
        j = torch.arange(inside, device=device) - first[tile]
        cols = torch.ceil(torch.sqrt(share.double())).long().clamp_(min=1)[tile]
        rows = ((share[tile] + cols - 1) // cols).clamp_(min=1)
        t = chosen[tile]
        x0, y0 = (t % tiles.shape[1]) * tile_px, (t // tiles.shape[1]) * tile_px
        u = ((j % cols).double() + torch.rand(inside, device=device, generator=generator, dtype=torch.float64)) / cols
        v = ((j // cols).double() + torch.rand(inside, device=device, generator=generator, dtype=torch.float64)) / rows
        x = (x0 + (u * tile_px).long()).clamp_(max=width - 1)
        y = (y0 + (v * tile_px).long()).clamp_(max=height - 1)
        parts.append(y * width + x)
    rest = count - inside
    if rest:
        cols = max(1, math.ceil(math.sqrt(rest)))
        rows = -(-rest // cols)
        j = torch.arange(rest, device=device)
        u = ((j % cols).double() + torch.rand(rest, device=device, generator=generator, dtype=torch.float64)) / cols
        v = ((j // cols).double() + torch.rand(rest, device=device, generator=generator, dtype=torch.float64)) / rows
        x = (u * width).long().clamp_(max=width - 1)
        y = (v * height).long().clamp_(max=height - 1)
        parts.append(y * width + x)
    return torch.cat(parts) if parts else torch.zeros(0, dtype=torch.long, device=device)
