"""Data-parallel protocol (odie_b200.parallel) on 2 CPU ranks over gloo.

The GPU runtime is replaced by the CPU oracle of the routed-expert step: each
rank computes its own band's head gradient, DataParallelStep all-reduces it and
every rank applies the same update.  Checked: the row bands partition the image,
the ranks' heads stay identical, and they equal a single process that applies
the sum of both bands' gradients.
"""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from odie_b200 import parallel

SHAPE = (23, 17)
EXPERTS = 3
ENCODING = dict(n_levels=16, n_features_per_level=2, log2_hashmap_size=7, base_resolution=2, per_level_scale=1.3)
ROUTER_ENCODING = dict(n_levels=16, n_features_per_level=2, log2_hashmap_size=6, base_resolution=2,
                       per_level_scale=1.2)
LR = 1e-1


def case(seed=3):
    from odie_b200.layout import hash_levels
    rng = np.random.default_rng(seed)
    records, stride = hash_levels(ENCODING)
    rrecords, rtotal = hash_levels(ROUTER_ENCODING)
    image = rng.integers(0, 256, (SHAPE[0] * SHAPE[1], 3), dtype=np.uint8)
    tables = (rng.standard_normal(EXPERTS * stride) * .05).astype(np.float32)
    router_table = (rng.standard_normal(rtotal) * .5).astype(np.float32)
    heads = (rng.standard_normal(32 * 32 * 2 + 16 * 32 + 32 * 64 + 64 * 64 + 16 * 64) * .1).astype(np.float32)
    return image, records, stride, rrecords, tables, router_table, heads


class OracleRuntime:
    """step_grads / step_heads of one rank's band, computed by the CPU oracle."""

    def __init__(self, band, heads, head_grad, steps_ids):
        from oracle import oracle
        self.oracle = oracle
        self.image, self.records, self.stride, self.rrecords, self.tables, self.router_table, _ = case()
        first, last = parallel.band_rows(SHAPE[0], *band)
        self.shape = (last - first, SHAPE[1])
        self.rgb = self.image.reshape(SHAPE[0], SHAPE[1], 3)[first:last].reshape(-1, 3)
        self.heads, self.head_grad, self.ids = heads, head_grad, steps_ids

    def step_grads(self, ids):
        split = 32 * 32 * 2 + 16 * 32
        h = self.heads.detach().numpy()
        ref = self.oracle.reference_step_experts(self.rgb, ids.numpy(), self.shape, self.tables, self.records,
                                                 self.stride, EXPERTS, self.router_table, self.rrecords, h[:split],
                                                 h[split:])
        self.head_grad.copy_(torch.from_numpy(ref['head_grad'].astype(np.float32)))

    def step_heads(self):
        self.heads.sub_(LR * self.head_grad / 16384)


def band_ids(rank, ranks, step):
    first, last = parallel.band_rows(SHAPE[0], rank, ranks)
    g = torch.Generator().manual_seed(100 * step + rank)
    return torch.randint(0, (last - first) * SHAPE[1], (64,), generator=g)


def worker(rank, world, port, out_dir):
    os.environ.update(MASTER_ADDR='127.0.0.1', MASTER_PORT=str(port))
    dist.init_process_group('gloo', rank=rank, world_size=world)
    try:
        heads = torch.from_numpy(case()[-1].copy())
        if rank:
            heads.add_(1.0)  # deliberately different before the broadcast

        class Model:  # the two shared heads, as broadcast_heads sees them
            gate = type('H', (), {'params': heads[:32 * 32 * 2 + 16 * 32]})
            decoder = type('H', (), {'params': heads[32 * 32 * 2 + 16 * 32:]})
        parallel.broadcast_heads(Model)
        _, head_grad, _ = parallel.head_gradient_buffer(Model, device='cpu')
        step = parallel.DataParallelStep(OracleRuntime((rank, world), heads, head_grad, None), head_grad)
        for k in range(2):
            step(band_ids(rank, world, k))
        np.save(os.path.join(out_dir, f'heads{rank}.npy'), heads.numpy())
    finally:
        dist.destroy_process_group()


def free_port():
    with socket.socket() as s:
        s.bind(('127.0.0.1', 0))
        return s.getsockname()[1]


def test_band_rows_partition():
    for height in (1, 7, 1356):
        for ranks in (1, 2, 3, 8):
            if ranks > height:
                continue
            bands = [parallel.band_rows(height, r, ranks) for r in range(ranks)]
            assert bands[0][0] == 0 and bands[-1][1] == height
            assert all(a[1] == b[0] and a[0] < a[1] for a, b in zip(bands, bands[1:] + [(height, height + 1)]))


@pytest.mark.timeout(300)
def test_data_parallel_heads_match_single_process(tmp_path):
    world = 2
    mp.spawn(worker, args=(world, free_port(), str(tmp_path)), nprocs=world, join=True)
    got = [np.load(tmp_path / f'heads{r}.npy') for r in range(world)]
    assert np.array_equal(got[0], got[1]), 'ranks diverged'
    # single process: the same updates from the sum of both bands' gradients
    heads = torch.from_numpy(case()[-1].copy())
    grads = [torch.zeros_like(heads) for _ in range(world)]
    runtimes = [OracleRuntime((r, world), heads, grads[r], None) for r in range(world)]
    for k in range(2):
        for r in range(world):
            runtimes[r].step_grads(band_ids(r, world, k))
        total = grads[0] + grads[1]
        heads.sub_(LR * total / 16384)
    np.testing.assert_allclose(got[0], heads.numpy(), rtol=1e-6, atol=1e-7)


# ---------------------------------------------------------------- one fixed model split by bands
FULL = (24, 17)      # full image: 4 row bands of 6 rows
BANDS, PER = 4, 8    # 32 experts, 8 per band: the 64-row router
R_HEADS = 32 * 32 * 2 + 64 * 32


def banded_case(seed=5):
    from odie_b200.layout import hash_levels
    rng = np.random.default_rng(seed)
    records, stride = hash_levels(ENCODING)
    rrecords, rtotal = hash_levels(ROUTER_ENCODING)
    image = rng.integers(0, 256, (FULL[0] * FULL[1], 3), dtype=np.uint8)
    tables = (rng.standard_normal(BANDS * PER * stride) * .05).astype(np.float32)
    router_table = (rng.standard_normal(rtotal) * .5).astype(np.float32)
    heads = (rng.standard_normal(R_HEADS + 32 * 64 + 64 * 64 + 16 * 64) * .1).astype(np.float32)
    return image, records, stride, rrecords, tables, router_table, heads


class BandedOracleRuntime:
    """Rank `rank` of `ranks` holding bands [rank * k, (rank + 1) * k) (k = BANDS / ranks) of one fixed model: its
    own experts' tables, the shared router grid and heads.  Shared gradients go to `shared` (heads | router grid);
    its own tables take an SGD step in step_grads, the shared parameters one in step_heads."""

    def __init__(self, rank, ranks, heads, router_table, shared):
        from oracle import oracle
        self.oracle = oracle
        image, self.records, self.stride, self.rrecords, tables, _, _ = banded_case()
        held = BANDS // ranks
        self.first = rank * held
        rows = FULL[0] // BANDS
        self.row0, self.shape = self.first * rows, (held * rows, FULL[1])
        self.rgb = image.reshape(FULL[0], FULL[1], 3)[self.row0:self.row0 + held * rows].reshape(-1, 3)
        self.tables = tables[self.first * PER * self.stride:(self.first + held) * PER * self.stride].copy()
        self.heads, self.router_table, self.shared = heads, router_table, shared
        self.banding = dict(bands=BANDS, first_band=self.first, per_band=PER, rows=FULL[0], row_offset=self.row0)

    def step_grads(self, ids):
        h = self.heads.detach().numpy()
        ref = self.oracle.reference_step_experts(self.rgb, ids.numpy(), self.shape, self.tables, self.records,
                                                 self.stride, self.tables.size // self.stride, self.router_table.numpy(),
                                                 self.rrecords, h[:R_HEADS], h[R_HEADS:], banding=self.banding)
        heads = self.heads.numel()
        self.shared[:heads] = torch.from_numpy(ref['head_grad'].astype(np.float32))
        self.shared[heads:] = torch.from_numpy(ref['router_grid_grad'].astype(np.float32))
        self.tables -= (LR * ref['grid_grad'] / 128).astype(np.float32)

    def step_heads(self):
        heads = self.heads.numel()
        self.heads.sub_(LR * self.shared[:heads] / 16384)
        self.router_table.sub_(LR * self.shared[heads:] / 128)


def banded_ids(rank, ranks, step):
    rows = FULL[0] // BANDS * (BANDS // ranks)
    g = torch.Generator().manual_seed(10 * step + rank)
    return torch.randint(0, rows * FULL[1], (48,), generator=g)


def banded_worker(rank, world, port, out_dir):
    os.environ.update(MASTER_ADDR='127.0.0.1', MASTER_PORT=str(port))
    dist.init_process_group('gloo', rank=rank, world_size=world)
    try:
        case_ = banded_case()
        heads, router_table = torch.from_numpy(case_[-1].copy()), torch.from_numpy(case_[-2].copy())
        shared = torch.zeros(heads.numel() + router_table.numel())
        runtime = BandedOracleRuntime(rank, world, heads, router_table, shared)
        step = parallel.DataParallelStep(runtime, shared)
        for k in range(2):
            step(banded_ids(rank, world, k))
        np.save(os.path.join(out_dir, f'heads{rank}.npy'), heads.numpy())
        np.save(os.path.join(out_dir, f'router{rank}.npy'), router_table.numpy())
        np.save(os.path.join(out_dir, f'tables{rank}.npy'), runtime.tables)
    finally:
        dist.destroy_process_group()


@pytest.mark.timeout(300)
def test_banded_model_split_matches_single_process(tmp_path):
    """Two ranks holding bands 0-1 and 2-3 of one 32-expert model: the shared heads and router grid stay equal on
    both ranks and equal a single process applying the summed gradients; each rank's expert tables equal the
    single process's slice of them."""
    world = 2
    mp.spawn(banded_worker, args=(world, free_port(), str(tmp_path)), nprocs=world, join=True)
    heads = [np.load(tmp_path / f'heads{r}.npy') for r in range(world)]
    routers = [np.load(tmp_path / f'router{r}.npy') for r in range(world)]
    assert np.array_equal(heads[0], heads[1]) and np.array_equal(routers[0], routers[1]), 'ranks diverged'
    case_ = banded_case()
    h, rt = torch.from_numpy(case_[-1].copy()), torch.from_numpy(case_[-2].copy())
    shared = [torch.zeros(h.numel() + rt.numel()) for _ in range(world)]
    runtimes = [BandedOracleRuntime(r, world, h, rt, shared[r]) for r in range(world)]
    for k in range(2):
        for r in range(world):
            runtimes[r].step_grads(banded_ids(r, world, k))
        total = shared[0] + shared[1]
        h.sub_(LR * total[:h.numel()] / 16384)
        rt.sub_(LR * total[h.numel():] / 128)
    np.testing.assert_allclose(heads[0], h.numpy(), rtol=1e-6, atol=1e-7)
    np.testing.assert_allclose(routers[0], rt.numpy(), rtol=1e-6, atol=1e-7)
    for r in range(world):
        np.testing.assert_array_equal(np.load(tmp_path / f'tables{r}.npy'), runtimes[r].tables)
