"""CPU oracle of the ODIE hot path -- TEST INFRASTRUCTURE ONLY.

Only tests/, __graft_entry__.smoke() and bench.py (cpu_baseline leg and the
--impl reference arm) may import this module.  The product (odie_b200) never
does; it has no CPU fallback.

Two layers:
  * liboracle.so (oracle.c): the reference's arithmetic restated in strict C,
    one function per reference function, each citing the file:line it follows;
  * this module: ctypes wrappers, and `reference_step`, the reference's native
    training step (odie/native/runtime.cu:253-312) restated on the CPU from
    those functions plus fp64 matrix products for the fully fused MLP heads
    (whose fp16 rounding points follow the reference's fp16 network:
    activations stored in fp16, products accumulated at higher precision).

Pinning: the C oracle's selection/scoring/layout functions are checked bit-for-
bit against golden vectors produced by the reference's own CPU code
(tests/golden/make_golden.py); the packed query against the reference's own
CUDA kernels compiled from source (oracle/build_ref.py) on the GPU box.  The
TCNN heads and TCNN Adam of the reference are third-party code that is not
vendored (instant-ngp abe236ee -> tiny-cuda-nn 2e757bb): their arithmetic is
parity-unpinned; the heads follow the fully fused MLP's published structure
and Adam follows torch.optim.Adam, the reference backend's optimizer.
"""
import ctypes as C
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIB_PATH = HERE / 'liboracle.so'

_lib = None


def lib():
    global _lib
    if _lib is None:
        if not LIB_PATH.exists() or LIB_PATH.stat().st_mtime < (HERE / 'oracle.c').stat().st_mtime:
            subprocess.run(['make', '-s', '-C', str(HERE)], check=True)
        _lib = C.CDLL(str(LIB_PATH))
    return _lib


def _p(a):
    return a.ctypes.data_as(C.c_void_p)


class HashLevelC(C.Structure):
    _fields_ = [('scale', C.c_float), ('res', C.c_int), ('capacity', C.c_int), ('offset', C.c_int),
                ('F', C.c_int), ('feature_offset', C.c_int), ('hashed', C.c_int), ('cells', C.c_int)]


def _hash_levels(records):
    arr = (HashLevelC * len(records))()
    for i, r in enumerate(records):
        arr[i] = HashLevelC(r['scale'], r['resolution'], r['capacity'], r['offset'], r['features'], r['column'],
                            r['hashed'], int(r.get('cells', -1)))
    return arr


# ---------------------------------------------------------------- wrappers
def coords(ids, width, height, row0=0, rows=None):
    """Coordinates of local pixel ids; row0/rows place the image's rows in a taller full image."""
    ids = np.ascontiguousarray(ids, dtype=np.int64)
    xy = np.empty((ids.size, 2), dtype=np.float32)
    if row0 == 0 and rows in (None, height):
        lib().oracle_coords(_p(ids), C.c_int64(ids.size), width, height, _p(xy))
    else:
        lib().oracle_coords_frame(_p(ids), C.c_int64(ids.size), width, row0, rows, _p(xy))
    return xy


def rows(xy, descriptors, node_bitmap, prefix, bitmap):
    xy = np.ascontiguousarray(xy, dtype=np.float32)
    desc = np.ascontiguousarray(descriptors, dtype=np.int32)
    n, levels = xy.shape[0], desc.shape[0]
    vis = np.empty((n, levels), dtype=np.uint8)
    out = np.empty((n, levels, 4), dtype=np.int32)
    nb = np.ascontiguousarray(node_bitmap).view(np.uint64) if node_bitmap.size else np.zeros(1, np.uint64)
    pf = np.ascontiguousarray(prefix, dtype=np.int32) if prefix.size else np.zeros(1, np.int32)
    lib().oracle_rows(_p(xy), C.c_int64(n), _p(desc), levels, _p(nb), _p(pf), _p(np.ascontiguousarray(bitmap)),
                      _p(vis), _p(out))
    return vis, out


def query(xy, grid, descriptors, node_bitmap, prefix, bitmap, width, active=None, raw_width=None, pad_ones=False):
    xy = np.ascontiguousarray(xy, dtype=np.float32)
    grid = np.ascontiguousarray(grid, dtype=np.float32)
    desc = np.ascontiguousarray(descriptors, dtype=np.int32)
    n, levels = xy.shape[0], desc.shape[0]
    out = np.zeros((n, width), dtype=np.uint16)
    vis = np.empty((n, levels), dtype=np.uint8)
    nb = np.ascontiguousarray(node_bitmap).view(np.uint64) if node_bitmap.size else np.zeros(1, np.uint64)
    pf = np.ascontiguousarray(prefix, dtype=np.int32) if prefix.size else np.zeros(1, np.int32)
    lib().oracle_query(_p(xy), C.c_int64(n), _p(grid), _p(desc), levels, _p(nb), _p(pf),
                       _p(np.ascontiguousarray(bitmap)), width, levels if active is None else active,
                       width if raw_width is None else raw_width, int(pad_ones), _p(out), _p(vis))
    return out.view(np.float16), vis


def query_backward(xy, upstream, descriptors, node_bitmap, prefix, bitmap, params):
    xy = np.ascontiguousarray(xy, dtype=np.float32)
    up = np.ascontiguousarray(upstream, dtype=np.float16).view(np.uint16)
    desc = np.ascontiguousarray(descriptors, dtype=np.int32)
    grad = np.zeros(params, dtype=np.float64)
    nb = np.ascontiguousarray(node_bitmap).view(np.uint64) if node_bitmap.size else np.zeros(1, np.uint64)
    pf = np.ascontiguousarray(prefix, dtype=np.int32) if prefix.size else np.zeros(1, np.int32)
    lib().oracle_query_backward(_p(xy), C.c_int64(xy.shape[0]), _p(up), up.shape[1], _p(desc), desc.shape[0],
                                _p(nb), _p(pf), _p(np.ascontiguousarray(bitmap)), _p(grad))
    return grad


def hash_indices(xy, records):
    xy = np.ascontiguousarray(xy, dtype=np.float32)
    n, levels = xy.shape[0], len(records)
    idx = np.empty((n, levels, 4), dtype=np.int32)
    w = np.empty((n, levels, 4), dtype=np.float32)
    lib().oracle_hash_indices(_p(xy), C.c_int64(n), _hash_levels(records), levels, _p(idx), _p(w))
    return idx, w


def _bitmap(bitmap):
    return None if bitmap is None else np.ascontiguousarray(bitmap, dtype=np.uint8)


def hash_query(xy, table16, records, width, bitmap=None):
    """bitmap: cell-visibility bytes addressed by each record's 'cells' offset (-1 or absent: all visible)."""
    xy = np.ascontiguousarray(xy, dtype=np.float32)
    table = np.ascontiguousarray(table16, dtype=np.float16).view(np.uint16)
    out = np.zeros((xy.shape[0], width), dtype=np.uint16)
    bits = _bitmap(bitmap)
    lib().oracle_hash_query(_p(xy), C.c_int64(xy.shape[0]), _p(table), _hash_levels(records), len(records), width,
                            None if bits is None else _p(bits), _p(out))
    return out.view(np.float16)


def hash_backward(xy, upstream, records, params, bitmap=None):
    xy = np.ascontiguousarray(xy, dtype=np.float32)
    up = np.ascontiguousarray(upstream, dtype=np.float16).view(np.uint16)
    grad = np.zeros(params, dtype=np.float64)
    bits = _bitmap(bitmap)
    lib().oracle_hash_backward(_p(xy), C.c_int64(xy.shape[0]), _p(up), up.shape[1], _hash_levels(records),
                               len(records), None if bits is None else _p(bits), _p(grad))
    return grad


def allocation_bitmap(tiles, tile_px, height, width, res):
    """Cell visibility of one level from an allocated-tile mask (oracle_allocation_bitmap)."""
    t = np.ascontiguousarray(tiles, dtype=np.uint8)
    out = np.zeros((res * res + 7) // 8, dtype=np.uint8)
    lib().oracle_allocation_bitmap(_p(t), t.shape[1], t.shape[0], tile_px, height, width, res, _p(out))
    return out


def gate_forward(raw, logits, vis, feature_level, k_fixed=0, softplus=False):
    raw = np.ascontiguousarray(raw, dtype=np.float16).view(np.uint16)
    lg = np.ascontiguousarray(logits, dtype=np.float16).view(np.uint16)
    vis = np.ascontiguousarray(vis, dtype=np.uint8)
    fl = np.ascontiguousarray(feature_level, dtype=np.int32)
    n, width = raw.shape
    levels = vis.shape[1]
    weighted = np.empty_like(raw)
    sig = np.empty((n, levels), dtype=np.float32)
    lib().oracle_gate_forward(_p(raw), _p(lg), _p(vis), C.c_int64(n), levels, width, lg.shape[1], _p(fl), k_fixed,
                              int(softplus), _p(weighted), _p(sig))
    return weighted.view(np.float16), sig


def gate_backward(raw, sig, vis, dz, level_offset, level_dim, gate_width=16, k_fixed=0, softplus=False):
    raw = np.ascontiguousarray(raw, dtype=np.float16).view(np.uint16)
    dz = np.ascontiguousarray(dz, dtype=np.float16).view(np.uint16)
    sig = np.ascontiguousarray(sig, dtype=np.float32)
    vis = np.ascontiguousarray(vis, dtype=np.uint8)
    n, width = raw.shape
    levels = vis.shape[1]
    direct = np.empty_like(raw)
    da = np.empty((n, gate_width), dtype=np.uint16)
    lib().oracle_gate_backward(_p(raw), _p(sig), _p(vis), _p(dz), C.c_int64(n), levels, width, gate_width,
                               _p(np.ascontiguousarray(level_offset, dtype=np.int32)),
                               _p(np.ascontiguousarray(level_dim, dtype=np.int32)), k_fixed, int(softplus),
                               _p(direct), _p(da))
    return direct.view(np.float16), da.view(np.float16)


def grid_values(direct, dr, router=True):
    d = np.ascontiguousarray(direct, dtype=np.float16).view(np.uint16)
    r = np.ascontiguousarray(dr if dr is not None else direct, dtype=np.float16).view(np.uint16)
    out = np.empty(d.shape, dtype=np.float32)
    lib().oracle_grid_values(_p(d), _p(r), C.c_int64(d.size), int(router), _p(out))
    return out


def loss_grad(output16, target, real=None):
    out = np.ascontiguousarray(output16, dtype=np.float16).view(np.uint16)
    target = np.ascontiguousarray(target, dtype=np.float32)
    n = out.shape[0]
    dy = np.empty((n, 16), dtype=np.uint16)
    squares = np.empty(n, dtype=np.float32)
    lib().oracle_loss_grad(_p(out), _p(target), C.c_int64(n), C.c_int64(n if real is None else real), _p(dy),
                           _p(squares))
    return dy.view(np.float16), squares


def target_u8(rgb, ids):
    rgb = np.ascontiguousarray(rgb, dtype=np.uint8)
    ids = np.ascontiguousarray(ids, dtype=np.int64)
    out = np.empty((ids.size, 3), dtype=np.float32)
    lib().oracle_target_u8(_p(rgb), _p(ids), C.c_int64(ids.size), _p(out))
    return out


def adam(p, m, v, steps, grad, loss_scale, lr, skip_zero, beta1=0.9, beta2=0.999, eps=1e-15):
    """In place on copies; returns (p, m, v, steps, half_copy)."""
    p, m, v = (np.array(x, dtype=np.float32, copy=True) for x in (p, m, v))
    steps = np.array(steps, dtype=np.uint32, copy=True)
    grad = np.ascontiguousarray(grad, dtype=np.float32)
    half = np.empty(p.size, dtype=np.uint16)
    lib().oracle_adam(_p(p), _p(m), _p(v), _p(steps), _p(grad), C.c_int64(p.size), C.c_float(loss_scale),
                      C.c_double(lr), C.c_double(beta1), C.c_double(beta2), C.c_double(eps), int(skip_zero), _p(half))
    return p, m, v, steps, p.astype(np.float16)  # fp16 copy of every entry (updated or skipped)


def score_chunk(prediction, target, begin, end, width, resolution, first_y, active_cells, xb, yb, totals, rgb8):
    pred = np.ascontiguousarray(prediction, dtype=np.float32)
    tgt = np.ascontiguousarray(target)
    lib().oracle_score_chunk(_p(pred), _p(tgt), C.c_int64(begin), C.c_int64(end), width, resolution, first_y,
                             active_cells, _p(np.ascontiguousarray(xb, dtype=np.int32)),
                             _p(np.ascontiguousarray(yb, dtype=np.int32)), _p(totals), int(rgb8))
    return totals


def select_benefit_cost(scores, resolution, cap, normalize=True):
    scores = np.ascontiguousarray(scores, dtype=np.float64)
    cells = resolution * resolution
    selected = np.empty(cells, dtype=np.uint8)
    nodes = np.empty((cells + 7) // 8 * 8, dtype=np.uint8)
    used = C.c_int64(0)
    lib().oracle_select_benefit_cost.restype = C.c_int64
    iterations = lib().oracle_select_benefit_cost(_p(scores), resolution, C.c_int64(cap), int(normalize),
                                                  _p(selected), _p(nodes), C.byref(used))
    return selected.astype(bool), nodes.astype(bool), int(iterations), int(used.value)


def select_mean_rank(scores, resolution, cap):
    scores = np.ascontiguousarray(scores, dtype=np.float64)
    cells = resolution * resolution
    selected = np.empty(cells, dtype=np.uint8)
    nodes = np.empty((cells + 7) // 8 * 8, dtype=np.uint8)
    lib().oracle_select_mean_rank(_p(scores), resolution, C.c_int64(cap), _p(selected), _p(nodes))
    return selected.astype(bool), nodes.astype(bool)


def tile_scores(prediction, target_u8_img, height, width, tile):
    tiles = ((width + tile - 1) // tile) * ((height + tile - 1) // tile)
    out = np.empty(tiles, dtype=np.float64)
    lib().oracle_tile_scores(_p(np.ascontiguousarray(prediction, dtype=np.float32)),
                             _p(np.ascontiguousarray(target_u8_img, dtype=np.uint8)), height, width, tile, _p(out))
    return out


def topk(scores, k):
    scores = np.ascontiguousarray(scores, dtype=np.float64)
    chosen = np.empty(k, dtype=np.int64)
    lib().oracle_topk(_p(scores), C.c_int64(scores.size), C.c_int64(k), _p(chosen))
    return chosen


def router(x16, w1, w2, w3, hidden, experts, first=None):
    """Top-1 routing.  first (int32 [n], optional): each coordinate's first live logit row; it then chooses among
    `experts` rows from there and the returned choice is relative to it.  Returns (choice, prob, all logits)."""
    x = np.ascontiguousarray(x16, dtype=np.float16).view(np.uint16)
    n, in_width = x.shape
    out_width = np.asarray(w3).size // hidden
    expert = np.empty(n, dtype=np.int32)
    prob = np.empty(n, dtype=np.float32)
    logits = np.empty((n, out_width), dtype=np.uint16)
    ws = [np.ascontiguousarray(w, dtype=np.float16).view(np.uint16) for w in (w1, w2, w3)]
    rows = None if first is None else np.ascontiguousarray(first, dtype=np.int32)
    if rows is not None:
        assert rows.shape == (n,) and rows.min(initial=0) >= 0 and rows.max(initial=0) + experts <= out_width
    lib().oracle_router(_p(x), C.c_int64(n), in_width, _p(ws[0]), hidden, _p(ws[1]), _p(ws[2]), out_width,
                        None if rows is None else _p(rows), experts, _p(expert), _p(prob), _p(logits))
    return expert, prob, logits.view(np.float16)


def band_rows_of(ids, width, banding):
    """Band of each local pixel id under spatial expert ownership (router.cuh Banding): the global row
    row_offset + id // width, its band floor(row * bands / rows), clamped to the bands held."""
    rows_global = banding.get('row_offset', 0) + np.asarray(ids, dtype=np.int64) // width
    band = rows_global * banding['bands'] // banding['rows']
    held = banding['experts'] // banding['per_band']
    return np.clip(band, banding['first_band'], banding['first_band'] + held - 1)


# ---------------------------------------------------------------- heads and the full step
def head_matrices(params, shapes):
    out, offset = [], 0
    for o, i in shapes:
        out.append(np.asarray(params[offset:offset + o * i], dtype=np.float32).reshape(o, i))
        offset += o * i
    return out


def head_shapes(width, hidden, depth, out):
    return [(hidden, width)] + [(hidden, hidden)] * (depth - 1) + [(out, hidden)]


def _f16(x):
    return np.asarray(x, dtype=np.float64).astype(np.float16)


def _mm(a16, w16t):
    """fp16 x fp16 products accumulated in fp64 (the network's higher-precision accumulation)."""
    return a16.astype(np.float64) @ w16t.astype(np.float64)


def reference_step(rgb, ids, shape, grid, layout, gate_params, decoder_params, levels, raw_width, router=True,
                   k_fixed=0, softplus=False, active=None):
    """One native training step of the reference, forward and backward, on the CPU.

    rgb: u8 [H*W, 3]; ids: int64 [n]; grid: fp32 master; layout: dict with
    descriptors/node_bitmap/node_prefix/bitmap (numpy).  Returns a dict of every
    intermediate: xy, target, raw, vis, logits, sig, weighted, out, dy, squares,
    dz, direct, da, dr, values (grid-gradient values, fp16-valued fp32),
    grid_grad (fp64, scale 128), head_grad (fp64, scale 16384, gate | decoder).
    """
    height, width = shape
    n = ids.size
    W = (raw_width + 15) // 16 * 16
    active = levels if active is None else active
    xy = coords(ids, width, height)
    target = target_u8(rgb, ids)
    desc = layout['descriptors']
    raw, vis = query(xy, grid, desc, layout['node_bitmap'], layout['node_prefix'], layout['bitmap'], W,
                     active=active, raw_width=raw_width, pad_ones=True)
    feature_level = np.full(W, -1, dtype=np.int32)
    level_offset = desc[:, 6].astype(np.int32)
    level_dim = desc[:, 5].astype(np.int32)
    for l in range(levels):
        feature_level[level_offset[l]:level_offset[l] + level_dim[l]] = l
    gate = head_matrices(gate_params, head_shapes(W, 32, 1, 16)) if router else None
    dec = head_matrices(decoder_params, head_shapes(W, 64, 2, 16))
    result = dict(xy=xy, target=target, raw=raw, vis=vis)
    if router:
        g1, g2 = (_f16(w) for w in gate)
        gh = _f16(np.maximum(_mm(raw, g1.T), 0))
        logits = _f16(_mm(gh, g2.T))
        weighted, sig = gate_forward(raw, logits, vis, feature_level, k_fixed, softplus)
        result.update(gh=gh, logits=logits, sig=sig)
    else:
        weighted = raw
    d1, d2, d3 = (_f16(w) for w in dec)
    h1 = _f16(np.maximum(_mm(weighted, d1.T), 0))
    h2 = _f16(np.maximum(_mm(h1, d2.T), 0))
    out = _f16(_mm(h2, d3.T))
    dy, squares = loss_grad(out, target)
    dh2 = _f16(np.where(h2 > 0, _mm(dy, d3), 0))
    dh1 = _f16(np.where(h1 > 0, _mm(dh2, d2), 0))
    dz = _f16(_mm(dh1, d1))
    # parameter order of the decoder: W1 [64][W], W2 [64][64], W3 [16][64]
    dec_grad = [dh1.astype(np.float64).T @ weighted.astype(np.float64), dh2.astype(np.float64).T @ h1.astype(np.float64),
                dy.astype(np.float64).T @ h2.astype(np.float64)]
    result.update(weighted=weighted, h1=h1, h2=h2, out=out, dy=dy, squares=squares, dz=dz)
    if router:
        direct, da = gate_backward(raw, sig, vis, dz, level_offset, level_dim, 16, k_fixed, softplus)
        dgh = _f16(np.where(gh > 0, _mm(da, g2), 0))
        dr = _f16(_mm(dgh, g1))
        values = grid_values(direct, dr, True)
        gate_grad = [dgh.astype(np.float64).T @ raw.astype(np.float64), da.astype(np.float64).T @ gh.astype(np.float64)]
        result.update(direct=direct, da=da, dgh=dgh, dr=dr)
    else:
        values = grid_values(dz, None, False)
        gate_grad = []
    result['values'] = values
    upstream = values.astype(np.float16)
    result['grid_grad'] = query_backward(xy, upstream, desc, layout['node_bitmap'], layout['node_prefix'],
                                         layout['bitmap'], grid.size)
    result['head_grad'] = np.concatenate([g.reshape(-1) for g in gate_grad + dec_grad]) if (gate_grad or dec_grad) \
        else np.zeros(0)
    return result


# ---------------------------------------------------------------- routed experts
def router_out(model_experts):
    """Logit rows of the router MLP: 16 for up to 16 experts, else 64 (router.cuh router_out)."""
    return 16 if model_experts <= 16 else 64


def router_shapes(width, model_experts=16):
    """Router W1, W2, W3 as (out, in)."""
    return [(32, width), (32, 32), (router_out(model_experts), 32)]


def expert_query(xy, tables16, expert, expert_stride, records, width, bitmap=None):
    """Per-coordinate expert tables: rows routed to expert e read tables16[e * stride : (e + 1) * stride]."""
    out = np.zeros((xy.shape[0], width), dtype=np.float16)
    for e in np.unique(expert):
        rows = np.nonzero(expert == e)[0]
        out[rows] = hash_query(xy[rows], tables16[e * expert_stride:(e + 1) * expert_stride], records, width, bitmap)
    return out


def expert_backward(xy, upstream, expert, expert_stride, records, params, bitmap=None):
    grad = np.zeros(params, dtype=np.float64)
    for e in np.unique(expert):
        rows = np.nonzero(expert == e)[0]
        grad[e * expert_stride:(e + 1) * expert_stride] += hash_backward(xy[rows], upstream[rows], records,
                                                                         expert_stride, bitmap)
    return grad


def reference_step_experts(rgb, ids, shape, tables, records, expert_stride, experts, router_table, router_records,
                           router_params, decoder_params, width=32, bitmap=None, banding=None, targets=None):
    """One routed-expert training step on the CPU (the restatement the CUDA path is checked against).

    Routing: router grid features -> router MLP with fp32 fma chains (bit-exact
    definition, `router`), top-1 over the coordinate's live experts, probability
    p.  banding (optional dict: bands, first_band, per_band, rows = full-image
    height, row_offset): spatial expert ownership -- a coordinate of global row y
    lies in band floor(y * bands / rows) and chooses among logit rows
    [band * per_band, (band + 1) * per_band); its local expert is (band -
    first_band) * per_band + choice.  Without banding every coordinate chooses
    among all `experts`.  Decoder input = fp16(expert features x fp16(p)).
    Decoder, loss and fp16 rounding points as in `reference_step`.  Backward:
    v = fp16(dz / 128); expert values = fp16(v x fp16(p)); dp = sum_c v_c f_c;
    dz_j = dp p (delta_je - p_j) with p_j the softmax of the live fp16 logits;
    da = fp16(fp16(dz_j) x 128) in the live columns, 0 elsewhere; router
    backward to dR; router values = fp16(dR / 128).  Head gradients (scale 16384)
    in the order router W1, W2, W3 | decoder W1, W2, W3; grid gradients (scale
    128) of the expert tables and of the router grid.  targets (optional u8 [n, 3]): the
    pixels of `ids`, given instead of reading them from rgb (for images too large to copy to the host).
    """
    height, img_width = shape
    b = dict(banding or dict(bands=1, first_band=0, per_band=experts, rows=height, row_offset=0), experts=experts)
    per = b['per_band']
    n = len(ids)
    xy = coords(ids, img_width, height, b.get('row_offset', 0), b['rows'])
    target = target_u8(rgb, ids) if targets is None else target_u8(targets, np.arange(n))
    rin = hash_query(xy, router_table.astype(np.float16), router_records, width)
    r1, r2, r3 = (_f16(w) for w in head_matrices(router_params, router_shapes(width, b['bands'] * per)))
    band = band_rows_of(ids, img_width, b) if b['bands'] > 1 else np.zeros(n, dtype=np.int64)
    first_row = (band * per).astype(np.int32)
    choice, prob, logits = router(rin, r1.reshape(-1), r2.reshape(-1), r3.reshape(-1), 32, per, first=first_row)
    expert = ((band - b['first_band']) * per + choice).astype(np.int32)
    live_cols = first_row[:, None] + np.arange(per)[None, :]
    live_logits = np.take_along_axis(logits, live_cols, axis=1)
    feats = expert_query(xy, tables.astype(np.float16), expert, expert_stride, records, width, bitmap)
    ph = prob.astype(np.float16)
    weighted = _f16(feats.astype(np.float64) * ph.astype(np.float64)[:, None])
    d1, d2, d3 = (_f16(w) for w in head_matrices(decoder_params, head_shapes(width, 64, 2, 16)))
    h1 = _f16(np.maximum(_mm(weighted, d1.T), 0))
    h2 = _f16(np.maximum(_mm(h1, d2.T), 0))
    out = _f16(_mm(h2, d3.T))
    dy, squares = loss_grad(out, target)
    dh2 = _f16(np.where(h2 > 0, _mm(dy, d3), 0))
    dh1 = _f16(np.where(h1 > 0, _mm(dh2, d2), 0))
    dz = _f16(_mm(dh1, d1))
    v = _f16(dz.astype(np.float64) / 128)
    values = _f16(v.astype(np.float64) * ph.astype(np.float64)[:, None])
    dp = (v.astype(np.float64) * feats.astype(np.float64)).sum(1)
    z = live_logits.astype(np.float64)
    ez = np.exp(z - z.max(1, keepdims=True))
    pj = ez / ez.sum(1, keepdims=True)
    onehot = np.zeros_like(pj)
    onehot[np.arange(n), choice] = 1
    da_live = _f16(_f16(dp[:, None] * prob.astype(np.float64)[:, None] * (onehot - pj)).astype(np.float64) * 128)
    da = np.zeros((n, r3.shape[0]), dtype=np.float16)
    np.put_along_axis(da, live_cols, da_live, axis=1)
    gh1 = _f16(np.maximum(_mm(rin, r1.T), 0))
    gh2 = _f16(np.maximum(_mm(gh1, r2.T), 0))
    dgh2 = _f16(np.where(gh2 > 0, _mm(da, r3), 0))
    dgh1 = _f16(np.where(gh1 > 0, _mm(dgh2, r2), 0))
    dr = _f16(_mm(dgh1, r1))
    router_values = _f16(dr.astype(np.float64) / 128)
    f64 = lambda a: a.astype(np.float64)  # noqa: E731
    head = [f64(dgh1).T @ f64(rin), f64(dgh2).T @ f64(gh1), f64(da).T @ f64(gh2),
            f64(dh1).T @ f64(weighted), f64(dh2).T @ f64(h1), f64(dy).T @ f64(h2)]
    return dict(xy=xy, target=target, router_features=rin, expert=expert, band=band, prob=prob, logits=logits,
                live_logits=live_logits, raw=feats, weighted=weighted, out=out, dy=dy, squares=squares, dz=dz,
                values=values.astype(np.float32), dp=dp, da=da, router_values=router_values.astype(np.float32),
                grid_grad=expert_backward(xy, values, expert, expert_stride, records, tables.size, bitmap),
                router_grid_grad=hash_backward(xy, router_values, router_records, router_table.size),
                head_grad=np.concatenate([g.reshape(-1) for g in head]))


# ---------------------------------------------------------------- stratified sampler (device variant)
def philox4x32_10(counter, key):
    """Philox4x32-10 (Salmon, Moraes, Dror and Shaw, SC 2011) on uint32 arrays: counter [4][...], key [2][...]."""
    c = [np.asarray(x, dtype=np.uint64) & 0xFFFFFFFF for x in counter]
    k0, k1 = (np.asarray(x, dtype=np.uint64) & 0xFFFFFFFF for x in key)
    mask = np.uint64(0xFFFFFFFF)
    for r in range(10):
        if r:
            k0 = (k0 + np.uint64(0x9E3779B9)) & mask
            k1 = (k1 + np.uint64(0xBB67AE85)) & mask
        p0 = c[0] * np.uint64(0xD2511F53)
        p1 = c[2] * np.uint64(0xCD9E8D57)
        hi0, lo0 = p0 >> np.uint64(32), p0 & mask
        hi1, lo1 = p1 >> np.uint64(32), p1 & mask
        c = [hi1 ^ c[1] ^ k0, lo1, hi0 ^ c[3] ^ k1, lo0]
    return [x.astype(np.uint32) for x in c]


def stratified_ids(seed, step, width, height, n):
    """The device stratified sampler (odie_stratified_ids) restated: slot j takes stratum (j mod side, j / side),
    r = (philox word >> 8) 2^-24 with key = seed, counter = (j, step); uv = r / side + stratum / side in fp32;
    pixel = trunc(uv (W, H)) clamped -- the form of the reference's stratified_batches (odie/data.py:63-80)."""
    side = int(round(n ** 0.5))
    assert side * side == n and n & (n - 1) == 0
    j = np.arange(n, dtype=np.uint64)
    words = philox4x32_10([j & 0xFFFFFFFF, j >> np.uint64(32), np.full(n, step & 0xFFFFFFFF, np.uint64),
                           np.full(n, step >> 32, np.uint64)],
                          [np.full(n, seed & 0xFFFFFFFF, np.uint64), np.full(n, seed >> 32, np.uint64)])
    inv = np.float32(1.0 / side)  # a power of two: exact
    r0 = (words[0] >> np.uint32(8)).astype(np.float32) * np.float32(2.0 ** -24)
    r1 = (words[1] >> np.uint32(8)).astype(np.float32) * np.float32(2.0 ** -24)
    sx = (j % np.uint64(side)).astype(np.float32)
    sy = (j // np.uint64(side)).astype(np.float32)
    ux = r0 * inv + sx * inv
    uy = r1 * inv + sy * inv
    x = np.minimum((ux * np.float32(width)).astype(np.int64), width - 1)
    y = np.minimum((uy * np.float32(height)).astype(np.int64), height - 1)
    return y * width + x


# ---------------------------------------------------------------- single fp32 hash grid
def uniform_xy(seed, step, n):
    """The fp32 hash grid's uniform coordinates: Philox4x32-10 with key = seed, counter = (slot, step);
    x = (word0 >> 8) 2^-24, y = (word1 >> 8) 2^-24, in [0, 1)."""
    j = np.arange(n, dtype=np.uint64)
    words = philox4x32_10([j & 0xFFFFFFFF, j >> np.uint64(32), np.full(n, step & 0xFFFFFFFF, np.uint64),
                           np.full(n, step >> 32, np.uint64)],
                          [np.full(n, seed & 0xFFFFFFFF, np.uint64), np.full(n, seed >> 32, np.uint64)])
    x = (words[0] >> np.uint32(8)).astype(np.float32) * np.float32(2.0 ** -24)
    y = (words[1] >> np.uint32(8)).astype(np.float32) * np.float32(2.0 ** -24)
    return np.stack([x, y], axis=1)


def hg32_bilinear(image, xy):
    """Bilinear fp32 targets [n, 3] of an fp32 [H, W, 3] image (oracle_hg32_bilinear)."""
    image = np.ascontiguousarray(image, dtype=np.float32)
    xy = np.ascontiguousarray(xy, dtype=np.float32)
    out = np.empty((xy.shape[0], 3), dtype=np.float32)
    lib().oracle_hg32_bilinear(_p(image), image.shape[1], image.shape[0], _p(xy), C.c_int64(xy.shape[0]), _p(out))
    return out


def hg32_features(xy, grid, records):
    """fp32 features [n, 2 levels] of the fp32 table (oracle_hg32_features)."""
    xy = np.ascontiguousarray(xy, dtype=np.float32)
    grid = np.ascontiguousarray(grid, dtype=np.float32)
    out = np.empty((xy.shape[0], 2 * len(records)), dtype=np.float32)
    lib().oracle_hg32_features(_p(xy), C.c_int64(xy.shape[0]), _p(grid), _hash_levels(records), len(records), _p(out))
    return out


def hg32_step(image, xy, grid, weights, records, loss_scale=None):
    """One step of the single fp32 hash grid restated: per-coordinate forward and backward in fp32 exactly as
    the kernels round them (oracle_hg32_step), the weight and grid gradients summed in fp64.  Returns a dict
    of every intermediate plus `head_grad` [6336] (W1 | W2 | W3) and `grid_grad` [grid size]."""
    xy = np.ascontiguousarray(xy, dtype=np.float32)
    n = xy.shape[0]
    loss_scale = np.float32(2.0 / (3.0 * n)) if loss_scale is None else np.float32(loss_scale)
    target = hg32_bilinear(image, xy)
    f = hg32_features(xy, grid, records)
    w = np.ascontiguousarray(weights, dtype=np.float32)
    out = {k: np.empty((n, d), dtype=np.float32) for k, d in
           (('h1', 64), ('h2', 64), ('z', 3), ('y', 3), ('dz', 3), ('dh2', 64), ('dh1', 64), ('dx', 32))}
    squares = np.empty(n, dtype=np.float32)
    lib().oracle_hg32_step(_p(f), _p(target), C.c_int64(n), _p(w), C.c_float(loss_scale), _p(out['h1']),
                           _p(out['h2']), _p(out['z']), _p(out['y']), _p(out['dz']), _p(squares), _p(out['dh2']),
                           _p(out['dh1']), _p(out['dx']))
    d = {k: v.astype(np.float64) for k, v in out.items()}
    f64 = f.astype(np.float64)
    head = np.concatenate([(d['dh1'].T @ f64).reshape(-1), (d['dh2'].T @ d['h1']).reshape(-1),
                           (d['dz'].T @ d['h2']).reshape(-1)])
    head_magnitude = np.concatenate([(np.abs(d['dh1']).T @ np.abs(f64)).reshape(-1),
                                     (np.abs(d['dh2']).T @ np.abs(d['h1'])).reshape(-1),
                                     (np.abs(d['dz']).T @ np.abs(d['h2'])).reshape(-1)])
    params = int(sum(r['capacity'] * r['features'] for r in records))
    grid_grad = hg32_scatter(xy, out['dx'], records, params)
    grid_magnitude = hg32_scatter(xy, np.abs(out['dx']), records, params)
    return dict(out, target=target, features=f, squares=squares, head_grad=head, head_magnitude=head_magnitude,
                grid_grad=grid_grad, grid_magnitude=grid_magnitude, loss_scale=loss_scale)


def hg32_scatter(xy, values, records, params):
    """sum_k w_k v over every coordinate's corners, in fp64 (the fp32 hash grid's grid gradient)."""
    xy = np.ascontiguousarray(xy, dtype=np.float32)
    values = np.asarray(values, dtype=np.float64)
    n, levels = xy.shape[0], len(records)
    idx = np.empty((n, levels, 4), dtype=np.int32)
    w = np.empty((n, levels, 4), dtype=np.float32)
    lib().oracle_hash_indices(_p(xy), C.c_int64(n), _hash_levels(records), levels, _p(idx), _p(w))
    grad = np.zeros(params, dtype=np.float64)
    for l, r in enumerate(records):
        rows = r['offset'] + 2 * idx[:, l, :].astype(np.int64)
        weights = w[:, l, :].astype(np.float64)
        for c in range(2):
            np.add.at(grad, (rows + c).reshape(-1), (weights * values[:, 2 * l + c, None]).reshape(-1))
    return grad
