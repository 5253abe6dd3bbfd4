"""Generate golden vectors by running the reference ODIE code in this container.

Run once, where the reference tree is present:

    python tests/golden/make_golden.py [/path/to/reference]   (default: $ODIE_REFERENCE, else ../reference)

The reference's CPU code for the hot path's integer/byte and fp64 parts is
pure Python/NumPy/torch-CPU and runs here:
  odie/selection.py  native_thresholds, pixel_cells, residual_scores,
                     closure_nodes, select_benefit_cost (B2/E), select_mean_rank (B1)
  odie/model.py      plane_closure, make_node_index, make_layout
  odie/config.py     hash_grid_layout, resolve
  odie/support_codec.py  encode_support (bitmap / DEFLATE mask storage of the fp16 checkpoint)
The outputs are stored as small .npz fixtures beside this script so the tests
(and the GPU box, which has no reference tree) can pin the oracle and the
CUDA library against the reference itself.  Inputs are seeded synthetic data.
"""
import json
import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent


def reference_modules(root):
    sys.path.insert(0, str(root))
    import odie.selection as selection
    import odie.model as model
    import odie.config as config
    return selection, model, config


def thresholds(sel):
    out = {}
    for r in (2, 3, 7, 8, 13, 100, 128, 2048, 8192):
        out[f'thr_{r}'] = np.asarray(sel.native_thresholds(r), dtype=np.float32)
    return out


def pixel_cells(sel):
    out = {}
    # pixel_cells(shape, r) == ybucket[:, None] * r + xbucket[None, :]; the small
    # shapes store the full map, the large ones the two per-axis bucket vectors.
    for (h, w, r) in ((2, 2, 2), (37, 53, 8), (64, 80, 100)):
        out[f'cells_{h}x{w}_{r}'] = sel.pixel_cells((h, w), r).astype(np.int32)
    for (h, w, r) in ((1356, 2040, 813), (97, 3001, 2048), (4096, 4096, 3251)):
        cells = sel.pixel_cells((h, w), r).reshape(h, w)
        out[f'xbucket_{h}x{w}_{r}'] = (cells[0] % r).astype(np.int32)
        out[f'ybucket_{h}x{w}_{r}'] = (cells[:, 0] // r).astype(np.int32)
    return out


def residuals(sel):
    rng = np.random.default_rng(1729)
    out = {}
    for (h, w, r) in ((37, 53, 8), (64, 48, 13), (101, 77, 100)):
        pred = rng.random((h * w, 3), dtype=np.float32) * np.float32(1.2) - np.float32(0.1)
        u8 = rng.integers(0, 256, size=(h * w, 3), dtype=np.uint8)
        target = torch.from_numpy(u8).float().div_(255.).numpy()  # ByteTarget.cpu(), odie/data.py:27-28
        mean, total, counts = sel.residual_scores(pred, target, (h, w), r)
        key = f'{h}x{w}_{r}'
        out[f'res_pred_{key}'] = pred
        out[f'res_u8_{key}'] = u8
        out[f'res_total_{key}'] = total
        out[f'res_mean_{key}'] = mean
        out[f'res_counts_{key}'] = counts.astype(np.int64)
    return out


def selections(sel):
    rng = np.random.default_rng(4242)
    out = {}
    cases = []
    for r, frac in ((4, .5), (8, .3), (13, .25), (32, .2), (64, .15), (100, .1)):
        points = (r * r + 7) // 8 * 8
        cap = max(8, int(points * frac) // 8 * 8)
        cases.append((r, cap, 'random', rng.random(r * r) ** 3))
    # ties, zeros and repeated values exercise the id tie-break and free cells
    r = 16
    tied = np.round(rng.random(r * r) * 4) / 4
    tied[::7] = 0.
    cases.append((16, 96, 'tied', tied))
    cases.append((16, 0, 'capzero', rng.random(r * r)))
    cases.append((9, (81 + 7) // 8 * 8, 'full', rng.random(81)))
    sparse = np.zeros(24 * 24)
    sparse[rng.choice(576, 40, replace=False)] = rng.random(40)
    cases.append((24, 160, 'sparse', sparse))
    cases.append((40, 400, 'negzero', np.where(rng.random(1600) < .3, -0., rng.random(1600))))
    for i, (r, cap, name, scores) in enumerate(cases):
        scores = np.asarray(scores, dtype=np.float64)
        key = f'sel{i}_{name}_r{r}_c{cap}'
        out[f'{key}_scores'] = scores
        for normalized in (True, False):
            chosen, record = sel.select_benefit_cost(scores, r, cap, 2, normalize_by_cost=normalized)
            nodes = np.zeros((r * r + 7) // 8 * 8, dtype=bool)
            nodes[sel.closure_nodes(np.flatnonzero(chosen), r)] = True
            tag = 'B2' if normalized else 'E'
            out[f'{key}_{tag}_selected'] = chosen.astype(np.uint8)
            out[f'{key}_{tag}_nodes'] = nodes.astype(np.uint8)
            out[f'{key}_{tag}_iterations'] = np.int64(record['iterations'])
        chosen, record = sel.select_mean_rank(np.abs(scores), r, cap)
        out[f'{key}_B1_selected'] = chosen.astype(np.uint8)
    return out


def closures(sel, model):
    rng = np.random.default_rng(7)
    out = {}
    for r in (2, 5, 8, 13, 64):
        support = rng.random(r * r) < .3
        out[f'clo_support_{r}'] = support
        out[f'clo_nodes_{r}'] = sel.closure_nodes(np.flatnonzero(support), r).astype(np.int64)
        out[f'clo_plane_{r}'] = model.plane_closure(torch.from_numpy(support), r).numpy().astype(np.int64)
    for points in (8, 64, 72, 200, 4104):
        nodes = np.unique(rng.integers(0, points, size=points // 3))
        bitmap, prefix = model.make_node_index(torch.from_numpy(nodes.astype(np.int64)), points)
        out[f'idx_nodes_{points}'] = nodes.astype(np.int64)
        out[f'idx_bitmap_{points}'] = bitmap.view(torch.int64).numpy()
        out[f'idx_prefix_{points}'] = prefix.numpy()
    return out


def layouts(model):
    """make_layout on a 6-level config: 3 dense levels, 2 packed, 1 empty."""
    rng = np.random.default_rng(99)
    out = {}
    resolutions = [4, 7, 12, 20, 33, 50]
    dims = [2, 2, 2, 2, 4, 1]
    config = dict(resolutions=resolutions, n_levels=6, representation='xy_planes',
                  coarse_levels=0, gate_topology='shared', gate_position='feature',
                  initial_active_prefix=3)
    supports, caps = [], []
    for level, r in enumerate(resolutions):
        points = (r * r + 7) // 8 * 8
        if level < 3:
            support = torch.ones(r * r, dtype=torch.bool)
            cap = points
        elif level < 5:
            support = torch.from_numpy(rng.random(r * r) < .25)
            cap = (model.plane_closure(support, r).numel() + 7) // 8 * 8 + 16
        else:
            support = torch.zeros(r * r, dtype=torch.bool)
            cap = 64
        supports.append(support)
        caps.append(cap)
    layout = model.make_layout(config, supports, dims, caps)
    out['lay_resolutions'] = np.asarray(resolutions, dtype=np.int64)
    out['lay_dims'] = np.asarray(dims, dtype=np.int64)
    out['lay_caps'] = np.asarray(caps, dtype=np.int64)
    for level, s in enumerate(supports):
        out[f'lay_support_{level}'] = s.numpy()
    out['lay_descriptors'] = layout['descriptors'].numpy()
    out['lay_node_bitmap'] = layout['node_bitmap'].view(torch.int64).numpy()
    out['lay_node_prefix'] = layout['node_prefix'].numpy()
    out['lay_bitmap'] = layout['bitmap'].numpy()
    out['lay_params'] = np.int64(layout['params'])
    out['lay_input_width'] = np.int64(layout['input_width'])
    return out


def configs(config):
    out = {}
    encodings = {
        'c1': dict(otype='HashGrid', n_levels=16, n_features_per_level=2, log2_hashmap_size=19,
                   base_resolution=16, per_level_scale=1.5),
        'c2': dict(otype='HashGrid', n_levels=16, n_features_per_level=2, log2_hashmap_size=16,
                   base_resolution=16, per_level_scale=1.5),
        'tokyo': dict(otype='HashGrid', n_levels=16, n_features_per_level=2, log2_hashmap_size=21,
                      base_resolution=3, per_level_scale=1.841),
    }
    for name, enc in encodings.items():
        res, caps = config.hash_grid_layout(enc)
        out[f'hash_{name}_res'] = np.asarray(res, dtype=np.int64)
        out[f'hash_{name}_caps'] = np.asarray(caps, dtype=np.int64)
    # The resolved plan for the reference's gigapixel config (odie_gigapixel_50mib.json).
    raw = {'model': {'layers': 16, 'base_resolution': 8, 'max_resolution': 8192, 'features': 2, 'finest_features': 2},
           'data': {'sampling': 'stratified', 'target_storage': 'uint8'},
           'training': {'epochs': 50, 'batch_size': 65536, 'seed': 1729, 'epochs_per_stage': 1},
           'regions': {'backend': 'cuda_device'},
           'budget': {'parameter_payload_bytes': 52428800}}
    merged = config.merge(config.DEFAULT, {k: v for k, v in raw.items() if k != 'budget'})
    merged['budget'] = raw['budget']
    plan = config.resolve(merged, (32768, 32768), 32768 * 32768 * 3)
    out['plan_gigapixel_json'] = np.frombuffer(json.dumps(plan, sort_keys=True).encode(), dtype=np.uint8)
    return out


def support_codec():
    """The reference's per-level mask encodings (odie/support_codec.py encode_support) of seeded masks: constant,
    random, sparse, blocky (DEFLATE wins) and sizes that are not whole bytes.  Its optional JBIG1 bridge needs
    libjbig; as the reference does when that bridge is unavailable, masks are then stored as bitmap / DEFLATE, so
    the bridge is switched off here to record exactly that behaviour."""
    import odie.support_codec as codec
    codec.jbig_tool = lambda: None
    rng = np.random.default_rng(1729)
    masks = {'r1_one': np.ones(1, bool), 'r8_all': np.ones(64, bool), 'r9_none': np.zeros(81, bool),
             'r37_random': rng.random(37 * 37) < .3, 'r64_sparse': rng.random(64 * 64) < .02,
             'r5_single': np.eye(1, 25, 12, dtype=bool)[0], 'r3_pad': np.array([1, 0, 1, 1, 0, 0, 1, 0, 1], bool)}
    blocky = np.zeros((100, 100), bool)
    blocky[20:60, 30:90] = True
    masks['r100_blocky'] = blocky.reshape(-1)
    out = {}
    for key, mask in masks.items():
        record = codec.encode_support(torch.from_numpy(mask))
        out[f'{key}_mask'] = mask.astype(np.uint8)
        out[f'{key}_encoding'] = np.frombuffer(record['encoding'].encode(), dtype=np.uint8)
        out[f'{key}_meta'] = np.array([record['num_cells'], record['resolution'], record['selected_count']], np.int64)
        out[f'{key}_data'] = record['data'].numpy() if 'data' in record else np.zeros(0, np.uint8)
    return out


def main():
    sys.path.insert(0, str(HERE.parents[1]))
    from oracle.build_ref import reference_root
    root = Path(sys.argv[1]) if len(sys.argv) > 1 else reference_root()
    sel, model, config = reference_modules(root)
    fixtures = {
        'selection.npz': {**thresholds(sel), **pixel_cells(sel)},
        'residual.npz': residuals(sel),
        'greedy.npz': selections(sel),
        'layout.npz': {**closures(sel, model), **layouts(model)},
        'config.npz': configs(config),
        'support_codec.npz': support_codec(),
    }
    for name, arrays in fixtures.items():
        np.savez_compressed(HERE / name, **arrays)
        print(name, len(arrays), 'arrays', (HERE / name).stat().st_size, 'bytes')


if __name__ == '__main__':
    main()
