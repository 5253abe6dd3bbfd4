"""PyTorch-CPU restatements of the training steps -- TEST/BENCH INFRASTRUCTURE ONLY.

Used only by bench.py as the CPU baseline and as the `--impl reference` arm:
the reference has no CPU path (its "reference" backend still needs CUDA and
TCNN, odie/optimizer.py:54-89), so its native step (odie/native/runtime.cu:
253-312) is restated here with vectorised torch CPU ops: index_select gathers
of the fp16-rounded corner values, autograd's index_add scatter, F.linear heads
with fp16 activations, the L2 loss with the reference's 128 x 128 loss scaling
and torch.optim.Adam (betas 0.9/0.999, eps 1e-15).  CpuExpertStep restates the
routed multi-expert step the same way, CpuHashGrid32Step the single fp32 hash grid's.
All run on the host threads torch is given.
"""
import time

import numpy as np
import torch
import torch.nn.functional as F


class CpuStep:
    def __init__(self, shape, rgb_u8, levels, grid, gate, decoder, width, router=True, lr=(1e-2, 1e-3, 1e-3)):
        """levels: list of dicts {scale, res, points, offset, F, col, kind, row_map (int64 node->row or None),
        cells (bool [R*R] visibility or None)}; grid/gate/decoder: fp32 numpy masters."""
        self.shape = shape
        self.rgb = torch.from_numpy(np.ascontiguousarray(rgb_u8))
        self.levels = levels
        self.width = width
        self.router = router
        self.grid = torch.nn.Parameter(torch.from_numpy(grid.copy()))
        self.gate = torch.nn.Parameter(torch.from_numpy(gate.copy())) if router else None
        self.decoder = torch.nn.Parameter(torch.from_numpy(decoder.copy()))
        groups = [{'params': [self.grid], 'lr': lr[0]}, {'params': [self.decoder], 'lr': lr[2]}]
        if router:
            groups.append({'params': [self.gate], 'lr': lr[1]})
        self.optimizer = torch.optim.Adam(groups, betas=(.9, .999), eps=1e-15, foreach=False)

    def _mats(self, params, shapes):
        out, offset = [], 0
        for o, i in shapes:
            out.append(params[offset:offset + o * i].view(o, i))
            offset += o * i
        return out

    def encode(self, xy):
        return encode_levels(self.grid, self.levels, xy, self.width)

    def step(self, ids):
        height, width = self.shape
        xy = torch.stack(((ids % width).float() * (1.0 / (width - 1)), (ids // width).float() * (1.0 / (height - 1))), 1)
        target = self.rgb[ids].float() / 255.
        self.optimizer.zero_grad(set_to_none=True)
        raw, vis = self.encode(xy)
        W = self.width
        if self.router:
            g1, g2 = self._mats(self.gate, [(32, W), (16, 32)])
            gh = F.relu(F.linear(raw, g1.half().float())).half().float()
            logits = F.linear(gh, g2.half().float()).half().float()
            gates = torch.sigmoid(logits[:, :len(self.levels)]) * vis.float()
            per_col = torch.cat([gates[:, l:l + 1].expand(-1, lv['F']) for l, lv in enumerate(self.levels)], 1)
            if per_col.shape[1] < W:
                per_col = torch.cat((per_col, torch.ones((raw.shape[0], W - per_col.shape[1]))), 1)
            x = (raw * per_col.half().float()).half().float()
        else:
            x = raw
        d1, d2, d3 = self._mats(self.decoder, [(64, W), (64, 64), (16, 64)])
        h1 = F.relu(F.linear(x, d1.half().float())).half().float()
        h2 = F.relu(F.linear(h1, d2.half().float())).half().float()
        out = F.linear(h2, d3.half().float()).half().float()[:, :3]
        loss = (out - target).square().mean()
        (loss * 128.).backward()
        for p in (self.grid, self.decoder, self.gate):
            if p is not None and p.grad is not None:
                p.grad.div_(128.)
        self.optimizer.step()
        return float(loss.detach())


def encode_levels(table, levels, xy, width, base=None):
    """fp16 features [n, width] (fp32 gradient path) and visibility [n, L] of `levels` over `table`;
    base (int64 [n] or None) offsets every row's parameters (one table per routed expert)."""
    n = xy.shape[0]
    cols = []
    vis_all = []
    for lv in levels:
        p = xy * lv['scale'] + 0.5
        i = torch.floor(p)
        f = p - i
        ix, iy = i[:, 0].long(), i[:, 1].long()
        fx, fy = f[:, 0], f[:, 1]
        w = torch.stack(((1 - fx) * (1 - fy), fx * (1 - fy), (1 - fx) * fy, fx * fy), 1)
        if lv['kind'] == 'plane':
            cell = ix + iy * lv['res']
            nodes = torch.stack((cell, cell + 1, cell + lv['res'], cell + lv['res'] + 1), 1) % lv['points']
            vis = lv['cells'][cell.clamp(0, lv['res'] ** 2 - 1)] if lv['cells'] is not None else torch.ones(n, dtype=torch.bool)
            rows = lv['row_map'][nodes] if lv['row_map'] is not None else nodes
        else:
            cx = torch.stack((ix, ix + 1, ix, ix + 1), 1)
            cy = torch.stack((iy, iy, iy + 1, iy + 1), 1)
            if lv['kind'] == 'hashed':
                idx = (cx ^ ((cy * 2654435761) & 0xffffffff)) & 0xffffffff
            else:
                idx = cx + cy * lv['res']
            rows = idx % lv['points']
            vis = torch.ones(n, dtype=torch.bool)
        rows = torch.where(vis.unsqueeze(1), rows, torch.zeros_like(rows)).clamp(min=0)  # hidden cells read row 0
        for c in range(lv['F']):
            values = table.index_select(0, ((lv['offset'] if base is None else lv['offset'] + base.unsqueeze(1)) + rows * lv['F'] + c).reshape(-1)).view(n, 4)
            values = values.half().float() + (values - values.detach())  # fp16-rounded corners, fp32 gradient
            cols.append((w.half().float() * values).sum(1) * vis)
        vis_all.append(vis)
    raw = torch.stack(cols, 1)
    if raw.shape[1] < width:
        raw = torch.cat((raw, torch.ones((n, width - raw.shape[1]))), 1)
    return raw.half().float() + (raw - raw.detach()), torch.stack(vis_all, 1)


class CpuExpertStep(CpuStep):
    """The routed multi-expert step (router grid -> top-1 router -> expert tables -> shared decoder) on the CPU.

    Same arithmetic as the CUDA path's definition: router MLP with fp16
    activations, top-1 of the fp16 logits, decoder input = fp16(features x
    fp16(p)); autograd through p (softmax probability) and both grids; Adam on
    expert tables, router grid, router MLP and decoder.  banding (dict: bands,
    first_band, per_band, rows = full-image height, row_offset): spatial expert
    ownership, each coordinate choosing among its row band's experts."""

    def __init__(self, shape, rgb_u8, levels, expert_stride, experts, router_levels, grid, router_grid, router, decoder,
                 width, lr=(1e-2, 1e-3, 1e-3), banding=None):
        super().__init__(shape, rgb_u8, levels, grid, router, decoder, width, router=True, lr=lr)
        self.router_levels, self.stride, self.experts = router_levels, expert_stride, experts
        self.banding = dict(banding or dict(bands=1, first_band=0, per_band=experts, rows=shape[0], row_offset=0))
        model_experts = self.banding['bands'] * self.banding['per_band']
        self.router_rows = 16 if model_experts <= 16 else 64
        self.router_grid = torch.nn.Parameter(torch.from_numpy(router_grid.copy()))
        self.optimizer.add_param_group({'params': [self.router_grid], 'lr': lr[0]})

    def step(self, ids):
        height, width = self.shape
        b = self.banding
        rows = ids // width + b.get('row_offset', 0)
        xy = torch.stack(((ids % width).float() * (1.0 / (width - 1)), rows.float() * (1.0 / (b['rows'] - 1))), 1)
        target = self.rgb[ids].float() / 255.
        self.optimizer.zero_grad(set_to_none=True)
        W = self.width
        rin, _ = encode_levels(self.router_grid, self.router_levels, xy, W)
        r1, r2, r3 = self._mats(self.gate, [(32, W), (32, 32), (self.router_rows, 32)])
        h = F.relu(F.linear(rin, r1.half().float())).half().float()
        h = F.relu(F.linear(h, r2.half().float())).half().float()
        per = b['per_band']
        if b['bands'] > 1:
            held = self.experts // per
            band = (rows * b['bands'] // b['rows']).clamp(b['first_band'], b['first_band'] + held - 1)
        else:
            band = torch.zeros_like(ids)
        live = band[:, None] * per + torch.arange(per)[None, :]
        logits = F.linear(h, r3.half().float()).half().float().gather(1, live)
        choice = logits.detach().argmax(1)
        expert = (band - b['first_band']) * per + choice
        prob = torch.softmax(logits, 1).gather(1, choice[:, None])
        raw, _ = encode_levels(self.grid, self.levels, xy, W, base=expert * self.stride)
        x = (raw * prob.half().float()).half().float()
        d1, d2, d3 = self._mats(self.decoder, [(64, W), (64, 64), (16, 64)])
        h1 = F.relu(F.linear(x, d1.half().float())).half().float()
        h2 = F.relu(F.linear(h1, d2.half().float())).half().float()
        out = F.linear(h2, d3.half().float()).half().float()[:, :3]
        loss = (out - target).square().mean()
        (loss * 128.).backward()
        for p in (self.grid, self.router_grid, self.decoder, self.gate):
            if p.grad is not None:
                p.grad.div_(128.)
        self.optimizer.step()
        return float(loss.detach())


def hash_levels_for_cpu(records):
    """Per-level dicts for CpuStep / CpuExpertStep from hash-grid level records."""
    return [dict(scale=r['scale'], res=r['resolution'], points=r['capacity'], offset=r['offset'], F=r['features'],
                 col=r['column'], kind='hashed' if r['hashed'] else 'dense', row_map=None, cells=None) for r in records]


def plane_levels_for_cpu(descriptors, node_bitmap, node_prefix, bitmap):
    """Per-level dicts for CpuStep from the reference descriptor tables (dense node->row maps for packed planes)."""
    levels = []
    nb = np.asarray(node_bitmap).view(np.uint64)
    for d in np.asarray(descriptors):
        r, points, offset, words, cells_off, f, col, direct = (int(v) for v in d)
        cells = np.unpackbits(np.asarray(bitmap)[cells_off:cells_off + (points // 8)], bitorder='little')[:r * r]
        row_map = None
        if not direct:
            bits = np.unpackbits(nb[words:words + (points + 63) // 64].view(np.uint8), bitorder='little')[:points]
            row_map = torch.from_numpy((np.cumsum(bits) - bits).astype(np.int64))
        levels.append(dict(scale=float(r - 1), res=r, points=points, offset=offset, F=f, col=col, kind='plane',
                           row_map=row_map, cells=torch.from_numpy(cells.astype(bool))))
    return levels


def time_steps(step, ids_batches, budget_seconds=20.0):
    """Run steps until the batches or the time budget run out; returns (coords, seconds)."""
    started = time.perf_counter()
    coords = 0
    for ids in ids_batches:
        step.step(ids)
        coords += ids.numel()
        if time.perf_counter() - started > budget_seconds:
            break
    return coords, time.perf_counter() - started


class CpuHashGrid32Step:
    """The single fp32 hash grid's step on the CPU: fp32 gathers (index_select), the fp32 MLP 32 -> 64 -> 64 -> 3
    with a sigmoid output, bilinear targets, mean squared error, autograd's index_add scatter and dense
    torch.optim.Adam (betas 0.9 / 0.99, eps 1e-15, lr 1e-2) over all 7.66 M table entries and the heads."""

    def __init__(self, image, records, grid, heads, lr=1e-2, seed=0):
        self.image = torch.from_numpy(np.ascontiguousarray(image, dtype=np.float32))
        self.levels = hash_levels_for_cpu(records)
        self.grid = torch.nn.Parameter(torch.from_numpy(np.array(grid, dtype=np.float32)))
        self.heads = torch.nn.Parameter(torch.from_numpy(np.array(heads, dtype=np.float32)))
        self.optimizer = torch.optim.Adam([self.grid, self.heads], lr=lr, betas=(.9, .99), eps=1e-15, foreach=False)
        self.generator = torch.Generator().manual_seed(seed)

    def features(self, xy):
        cols = []
        for lv in self.levels:
            p = xy * lv['scale'] + 0.5
            i = torch.floor(p)
            f = p - i
            ix, iy = i[:, 0].long(), i[:, 1].long()
            fx, fy = f[:, 0], f[:, 1]
            w = torch.stack(((1 - fx) * (1 - fy), fx * (1 - fy), (1 - fx) * fy, fx * fy), 1)
            cx = torch.stack((ix, ix + 1, ix, ix + 1), 1)
            cy = torch.stack((iy, iy, iy + 1, iy + 1), 1)
            idx = ((cx ^ ((cy * 2654435761) & 0xffffffff)) & 0xffffffff) if lv['kind'] == 'hashed' else cx + cy * lv['res']
            rows = lv['offset'] + 2 * (idx % lv['points'])
            for c in range(2):
                cols.append((w * self.grid.index_select(0, (rows + c).reshape(-1)).view(-1, 4)).sum(1))
        return torch.stack(cols, 1)

    def bilinear(self, xy):
        h, w = self.image.shape[:2]
        px, py = xy[:, 0] * (w - 1), xy[:, 1] * (h - 1)
        x0, y0 = px.long().clamp(0, w - 2), py.long().clamp(0, h - 2)
        fx, fy = (px - x0)[:, None], (py - y0)[:, None]
        im = self.image
        return (im[y0, x0] * (1 - fx) * (1 - fy) + im[y0, x0 + 1] * fx * (1 - fy) + im[y0 + 1, x0] * (1 - fx) * fy
                + im[y0 + 1, x0 + 1] * fx * fy)

    def step_uniform(self, n):
        xy = torch.rand((n, 2), generator=self.generator)
        target = self.bilinear(xy)
        self.optimizer.zero_grad(set_to_none=True)
        f = self.features(xy)
        w = self.heads
        h = F.relu(F.linear(f, w[:2048].view(64, 32)))
        h = F.relu(F.linear(h, w[2048:6144].view(64, 64)))
        y = torch.sigmoid(F.linear(h, w[6144:].view(3, 64)))
        loss = ((y - target) ** 2).mean()
        loss.backward()
        self.optimizer.step()
        return float(loss.detach())
