"""Benchmark of the ODIE hot path on B200: train coords/s (fwd + bwd + Adam) and decode Gpix/s.

python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--workload c4-experts|...]

Workloads (odie_b200/workloads.py):
  c4-experts (default): the gigapixel benchmark -- a 32768 x 32768 procedural u8 image, 64 routed
    hash-grid experts under a 50 MiB fp16 budget (T = 2^14), owned spatially by 8 row bands of 8
    experts, a top-1 router (64 logits) on a coarse shared grid, the shared 64-wide decoder, 20 % of
    the 256 x 256 tiles allocated (exact top-k of the decoded residual), 2^22 coordinates per step and
    GPU, 70 % of them in the allocated tiles.  The decode line is the gigapixel reconstruction: every
    pixel of the image in launches of 2^24 pixels, u8 RGB out.
  c2-experts: 16 routed experts (T = 2^16) on a 2040 x 1356 image, 2^20 coords per step.
  c2-planes: the reference's own packed-plane method on the same image and batch.
  c3-experts: 8 routed experts (T = 2^17) on a 4096 x 4096 image with 30 % tile allocation, 2^21.
  c1-hash: the single fp32 hash grid (T = 2^19, 16 levels, fp32 MLP 32-64-64-3 with a sigmoid output) on a
    512 x 512 image, 2^18 uniform coordinates per step with bilinear targets, dense Adam (odie_hashgrid32_*).

One JSON line on rank 0.  `value` is whole-job coords/s with inputs resident in HBM (device-timed
with CUDA events, max over ranks); `e2e` is the same metric through the public API with the step's
pixel ids copied from pinned host memory and the loss read back every step (the next step's ids
upload on a copy stream while a step runs, as a training loop's loader prefetches).  Multi-GPU: one
process per GPU (torchrun).  c4: rank r of N holds 8/N bands of the one fixed model (their rows and
experts) and trains 2^22 coordinates of them per step (weak scaling); the router MLP, decoder and
router grid are shared, their gradients summed by one NCCL all-reduce per step that overlaps the
rank's expert-table scatter and update.  c2/c3: each rank trains the model of its own row band.
The `--impl reference` arm times the CPU restatement of the step (oracle/cpu_step.py; the reference
has no CPU path of its own) on the host's cores.
"""
import argparse
import json
import os
import subprocess
import sys
import threading
import time
from pathlib import Path

import numpy as np
import torch

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = 'train coords/s (fwd+bwd+Adam) & decode Gpix/s at 1/2/4/8 B200'
UNIT = 'coords/s'
WORKLOADS = ('c4-experts', 'c2-experts', 'c2-planes', 'c3-experts', 'c1-hash')
BATCHES = {'c4-experts': 1 << 22, 'c3-experts': 1 << 21, 'c2-experts': 1 << 20, 'c2-planes': 1 << 20, 'c1-hash': 1 << 18}
DECODE_LAUNCH = 1 << 24  # pixels per decode launch of the gigapixel reconstruction
CPU_WINDOW_ROWS = 1024   # rows of the gigapixel image the CPU legs sample from (their cost does not depend on it)


def parse():
    p = argparse.ArgumentParser()
    p.add_argument('--gpus', type=int, default=1)
    p.add_argument('--steps', type=int, default=20)
    p.add_argument('--warmup', type=int, default=5)
    p.add_argument('--impl', choices=['ours', 'reference'], default='ours')
    p.add_argument('--workload', default='c4-experts', choices=WORKLOADS)
    p.add_argument('--batch', type=int, default=None, help='coordinates per step and GPU (default: the workload\'s: '
                   '2^22 for c4, 2^21 for c3, 2^20 for the c2 workloads)')
    p.add_argument('--sampling', default='stratified', choices=['stratified', 'uniform'],
                   help='stratified: the reference default (odie/config.py:20, odie/data.py:63-80), one pixel per '
                        'stratum, strata in raster order; uniform: iid uniform pixel ids')
    p.add_argument('--no-cpu-baseline', action='store_true')
    p.add_argument('--shape', type=int, nargs=2, default=None, metavar=('H', 'W'),
                   help='c4 only: a smaller image of the same model and kernels (H a multiple of 2048), for profiling')
    p.add_argument('--decode-launch', type=int, default=DECODE_LAUNCH, help='c4: pixels per decode launch')
    return p.parse_args()


def workload(name, rank, ranks, batch, shape=None):
    """Model, target, planes, config and image of this rank's part of a workload."""
    from odie_b200 import workloads
    if name in ('c2-experts', 'c3-experts', 'c4-experts'):
        if name == 'c2-experts':
            config, rgb, shape = workloads.c2_experts(batch=batch, band=(rank, ranks))
        elif name == 'c3-experts':
            config, rgb, shape = workloads.c3_experts(batch=batch, band=(rank, ranks))
        else:
            config, rgb, shape = workloads.c4_experts(batch=batch, band=(rank, ranks),
                                                      shape=tuple(shape) if shape else workloads.C4_SHAPE)
        model, target, planes = workloads.build_expert_model(config, rgb)
        return dict(config=config, rgb=rgb, shape=shape, model=model, target=target, planes=planes)
    config, supports, dims, caps, rgb, shape = workloads.c2_planes(batch=batch, band=(rank, ranks))
    model, target, planes = workloads.build_plane_model(config, supports, dims, caps, rgb)
    return dict(config=config, rgb=rgb, shape=shape, model=model, target=target, planes=planes, supports=supports,
                dims=dims, caps=caps)


def c4_window(procedural=True):
    """The CPU legs' sample window of the gigapixel image: its first CPU_WINDOW_ROWS rows as u8 [rows * W, 3] on the
    host, drawn by this library's generator on the GPU (input data, not timed) when `procedural` and a GPU is
    there, else seeded random bytes of the same shape (the CPU step's cost does not depend on the pixel values)."""
    from odie_b200.workloads import C4_SHAPE
    if procedural and torch.cuda.is_available():
        from odie_b200.data import procedural_image
        return procedural_image(C4_SHAPE, 1729, 0, CPU_WINDOW_ROWS).cpu()
    g = torch.Generator().manual_seed(1729)
    return torch.randint(0, 256, (CPU_WINDOW_ROWS * C4_SHAPE[1], 3), dtype=torch.uint8, generator=g)


def cpu_step_of(name, batch, procedural=True):
    """The oracle's CPU restatement of one training step of the workload (same layout, seeded weights), and the
    (height, width) of the image window its coordinates are sampled from."""
    from oracle.cpu_step import CpuExpertStep, CpuHashGrid32Step, CpuStep, hash_levels_for_cpu, plane_levels_for_cpu
    from odie_b200 import layout as host_layout
    from odie_b200 import workloads
    rng = np.random.default_rng(0)
    if name == 'c1-hash':
        from odie_b200.data import blobs_and_gratings
        from odie_b200.hashgrid32 import c1_config, xavier_heads
        records, total = host_layout.hash_levels(c1_config()['hash_encoding'])
        image = blobs_and_gratings(512, 512, 1729).numpy()
        step = CpuHashGrid32Step(image, records, (rng.random(total, dtype=np.float32) * 2 - 1) * 1e-4,
                                 xavier_heads(1729).numpy())
        return step, (512, 512)
    if name in ('c2-experts', 'c3-experts', 'c4-experts'):
        banding = None
        if name == 'c2-experts':
            config, rgb, shape = workloads.c2_experts(batch=batch)
        elif name == 'c3-experts':
            config, rgb, shape = workloads.c3_experts(batch=batch,
                                                      device='cuda' if torch.cuda.is_available() else 'cpu')
        else:
            config = workloads.experts_config(experts=64, batch=batch, encoding=workloads.C4_ENCODING)
            rgb, shape = c4_window(procedural), (CPU_WINDOW_ROWS, workloads.C4_SHAPE[1])
            banding = dict(bands=workloads.C4_BANDS, first_band=0, per_band=workloads.C4_PER_BAND,
                           rows=workloads.C4_SHAPE[0], row_offset=0)
        records, stride = host_layout.hash_levels(config['hash_encoding'])
        router_records, router_total = host_layout.hash_levels(config['router_encoding'])
        width, experts = 32, config['experts']
        router_rows = 16 if experts <= 16 else 64
        step = CpuExpertStep(shape, rgb.cpu().numpy(), hash_levels_for_cpu(records), stride, experts,
                             hash_levels_for_cpu(router_records),
                             ((rng.random(experts * stride, dtype=np.float32) * 2 - 1) * 1e-4),
                             ((rng.random(router_total, dtype=np.float32) * 2 - 1) * 0.1),
                             (rng.standard_normal(32 * width + 32 * 32 + router_rows * 32) * .2).astype(np.float32),
                             (rng.standard_normal(width * 64 + 64 * 64 + 1024) * .1).astype(np.float32), width,
                             banding=banding)
        return step, shape
    config, supports, dims, caps, rgb, shape = workloads.c2_planes(batch=batch)
    lay = host_layout.make_layout(config, supports, dims, caps)
    levels = plane_levels_for_cpu(lay['descriptors'].numpy(), lay['node_bitmap'].numpy(), lay['node_prefix'].numpy(),
                                  lay['bitmap'].numpy())
    width = (lay['input_width'] + 15) // 16 * 16
    step = CpuStep(shape, rgb.numpy(), levels, (rng.standard_normal(lay['params']) * 1e-3).astype(np.float32),
                   (rng.standard_normal(width * 32 + 512) * .1).astype(np.float32),
                   (rng.standard_normal(width * 64 + 64 * 64 + 1024) * .1).astype(np.float32), width)
    return step, shape


class DeviceArray:
    """A raw device buffer of the runtime (pointer from odie_pointers) as a CUDA array interface, so torch can
    view it without a copy."""

    def __init__(self, pointer, count, typestr):
        self.__cuda_array_interface__ = {'shape': (count,), 'typestr': typestr, 'data': (int(pointer), False),
                                         'version': 3, 'stream': None}


class Clocks:
    """SM clocks and throttle reasons sampled during the timed region: NVML every 5 ms (read-only queries of the
    device that runs this rank, found by PCI bus id), else nvidia-smi every 200 ms."""
    QUERY = ('index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,'
             'clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,'
             'clocks_event_reasons.sw_power_cap')
    REASONS = ('hw_slowdown', 'hw_thermal_slowdown', 'sw_thermal_slowdown', 'sw_power_cap')

    def __init__(self, index):
        self.index, self.samples, self.stop, self.source = index, [], threading.Event(), 'nvidia-smi'
        self.nvml = self.handle = None
        try:
            import pynvml
            pynvml.nvmlInit()
            p = torch.cuda.get_device_properties(index)
            self.handle = pynvml.nvmlDeviceGetHandleByPciBusId(
                f'{p.pci_domain_id:08x}:{p.pci_bus_id:02x}:{p.pci_device_id:02x}.0')
            self.nvml, self.source = pynvml, 'nvml'
            self.bits = (pynvml.nvmlClocksEventReasonHwSlowdown, pynvml.nvmlClocksEventReasonHwThermalSlowdown,
                         pynvml.nvmlClocksEventReasonSwThermalSlowdown, pynvml.nvmlClocksEventReasonSwPowerCap)
            self.max_mhz = float(pynvml.nvmlDeviceGetMaxClockInfo(self.handle, pynvml.NVML_CLOCK_SM))
        except Exception:
            self.nvml = None
        self.thread = threading.Thread(target=self.run, daemon=True)

    def sample_nvml(self):
        n = self.nvml
        sm = float(n.nvmlDeviceGetClockInfo(self.handle, n.NVML_CLOCK_SM))
        mask = n.nvmlDeviceGetCurrentClocksEventReasons(self.handle)
        return sm, self.max_mhz, [name for name, bit in zip(self.REASONS, self.bits) if mask & bit]

    def sample_smi(self):
        out = subprocess.run(['nvidia-smi', f'--id={self.index}', f'--query-gpu={self.QUERY}',
                              '--format=csv,noheader,nounits'], capture_output=True, text=True, timeout=5)
        if out.returncode != 0 or not out.stdout.strip():
            return None
        f = [x.strip() for x in out.stdout.strip().split(',')]
        num = lambda x: float(x) if x.replace('.', '').isdigit() else None
        return num(f[1]), num(f[2]), [name for i, name in enumerate(self.REASONS) if len(f) > 5 + i and f[5 + i] == 'Active']

    def run(self):
        while not self.stop.is_set():
            try:
                s = self.sample_nvml() if self.nvml else self.sample_smi()
                if s:
                    self.samples.append(s)
            except Exception:
                pass
            self.stop.wait(0.005 if self.nvml else 0.2)

    def __enter__(self):
        self.thread.start()
        return self

    def __exit__(self, *a):
        self.stop.set()
        self.thread.join(timeout=10)

    def summary(self):
        if not self.samples:
            return {'sm_mhz': None, 'sm_max_mhz': None, 'reasons': ['unsampled'], 'samples': 0, 'source': self.source}
        sm = [s[0] for s in self.samples if s[0] is not None]
        mx = [s[1] for s in self.samples if s[1] is not None]
        return {'sm_mhz': float(np.median(sm)) if sm else None, 'sm_max_mhz': max(mx) if mx else None,
                'reasons': sorted({r for s in self.samples for r in s[2]}), 'samples': len(self.samples),
                'source': self.source}


def per_coordinate(name, model):
    """Algorithmic work per coordinate of a training step's stages (the figures the roofline divides):
    encode forward 8 + 4 L F 2 + L F 2 B per encoding (fp16 tables, fp16 features), encode backward
    8 + L F 2 B per encoding (the coordinate and its gradient values, read once; the touched table entries'
    read + write, 8 B each, are added per step by the caller), router 64 + 8 B (+ 2 live B per logit stored),
    heads 6 x sum(in x out) FLOP (forward, data and weight gradients).

    The backward's figure is the least traffic any scatter needs.  Counting each of the 4 L F corner updates
    of a coordinate as an fp32 read + write (8 L F 4 B more per encoding, the per-corner atomic algorithm)
    would exceed what the kernels move: their runs add a cell's updates in registers and write each run once,
    so that count is reported beside it (naive_atomics_per_step) but not divided."""
    L, F = model.n_levels, 2
    experts = name.endswith('experts')
    encodings = 2 if experts else 1  # the router grid and the routed expert
    decoder = 32 * 64 + 64 * 64 + 64 * 16
    if experts:
        live = 8 if model.per_band <= 8 else 16
        router_rows = 16 if model.experts <= 16 else 64
        # the heads recompute the router's hidden layers; the logit layer's products run 64 (or 16) wide
        gate = 32 * 32 + 32 * 32 + router_rows * 32
    else:
        live, gate = 0, 32 * 32 + 32 * 16
    return {'encode_forward': ('hbm', encodings * (8 + 4 * L * F * 2 + L * F * 2)),
            'encode_backward': ('hbm', encodings * (8 + L * F * 2)),
            'router': ('hbm', 64 + 8 + 2 * live) if experts else ('hbm', None),
            'mlp_train': ('tensor', 6 * (gate + decoder))}


def adam_bytes(total_params, touched):
    """Algorithmic bytes of the zero-skipping Adam sweep: every parameter's gradient read (4 B); for each touched
    one p, m, v read and written (24 B), its step counter read and written (8 B), the fp16 copy (2 B) and the
    gradient cleared (4 B)."""
    return 4 * total_params + 38 * touched


def decode_per_pixel(name, model):
    """(algorithmic bytes, FLOP) per decoded pixel: the fp16 corner reads of every encoding (4 L F 2 B each) plus the
    u8 RGB written; router (live logits only) and decoder products."""
    L, F = model.n_levels, 2
    experts = name.endswith('experts')
    encodings = 2 if experts else 1
    decoder = 32 * 64 + 64 * 64 + 64 * 16
    gate = (32 * 32 + 32 * 32 + model.per_band * 32) if experts else (32 * 32 + 32 * 16)
    return encodings * 4 * L * F * 2 + 3, 2 * (gate + decoder)


def traffic_of(name, stage):
    """DRAM bytes per step of a stage from the committed ncu summary (profiles/dram_traffic.json), or None."""
    path = ROOT / 'profiles' / 'dram_traffic.json'
    if not path.exists():
        return None
    entry = json.loads(path.read_text()).get(name, {}).get(stage)
    return entry['bytes_per_step'] if entry else None


def l2_probe(lib, table_mib=32, operations=1 << 27):
    """Measured L2 throughput for random 4/16-byte loads and 4/8-byte fp32 reductions over an L2-resident table
    (odie_l2_probe): context for the gather and scatter kernels, whose tables all fit in L2."""
    table = torch.zeros((table_mib << 20) // 4, device='cuda')
    sink = torch.zeros(1, device='cuda')
    stream = torch.cuda.current_stream()
    names = ['load4', 'load16', 'red4', 'red8']
    out = {'table_mib': table_mib, 'operations': operations, 'gops': {}}
    for mode, name in enumerate(names):
        best = float('inf')
        for _ in range(4):
            start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            start.record()
            rc = lib.odie_l2_probe(table.data_ptr(), table.numel() * 4, mode, operations, sink.data_ptr(),
                                   stream.cuda_stream)
            end.record()
            if rc:
                raise RuntimeError('odie_l2_probe failed')
            torch.cuda.synchronize()
            best = min(best, start.elapsed_time(end) / 1e3)
        out['gops'][name] = operations / best / 1e9
    return out


def peaks():
    path = ROOT / 'MEASURED_PEAKS.json'
    if path.exists():
        data = json.loads(path.read_text())
        return data['hbm_gbs'], data['bf16_tflops'], data.get('bf16_tflops_sustained', data['bf16_tflops']), 'measured'
    return 6650.0, 1590.0, 1400.0, 'fallback'


def cpu_legs(args, budget=10.0, threads_list=None):
    """The CPU restatement of the step on this host's cores (bounded samples of 2^14 uniform coordinates per step):
    once with every host thread, once with one (the reference pins one thread, odie/train.py:72)."""
    all_threads = os.cpu_count() or 1
    threads_list = threads_list or [all_threads, 1]
    step, shape = cpu_step_of(args.workload, args.batch)
    sample = 1 << 14
    pixels = shape[0] * shape[1]
    g = torch.Generator().manual_seed(1)

    def one_step():
        if args.workload == 'c1-hash':
            step.step_uniform(sample)
        else:
            step.step(torch.randint(0, pixels, (sample,), generator=g))
    legs = []
    for threads in threads_list:
        torch.set_num_threads(threads)
        one_step()  # warm-up
        started, coords, steps = time.perf_counter(), 0, 0
        while time.perf_counter() - started < budget or steps < 2:
            one_step()
            coords += sample
            steps += 1
        seconds = time.perf_counter() - started
        legs.append({'value': coords / seconds, 'unit': UNIT, 'cores': threads, 'kind': 'port',
                     'sample': f'{steps} steps of {sample} uniform coords of {args.workload} (full model and '
                               f'layout, coordinates from a {shape[0]} x {shape[1]} window), torch CPU, {threads} '
                               f'thread(s), {seconds:.1f} s'})
    torch.set_num_threads(all_threads)
    return legs


def run_reference(args):
    rank = int(os.environ.get('RANK', 0))
    if rank != 0:
        return
    steps, coords = 0, 0
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    # this arm runs none of this library's kernels: the gigapixel window is seeded random bytes
    step, shape = cpu_step_of(args.workload, args.batch, procedural=False)
    sample = 1 << 14
    g = torch.Generator().manual_seed(2)
    pixels = shape[0] * shape[1]

    def one_step():
        if args.workload == 'c1-hash':
            step.step_uniform(sample)
        else:
            step.step(torch.randint(0, pixels, (sample,), generator=g))
    for _ in range(args.warmup):
        one_step()
    started = time.perf_counter()
    for _ in range(args.steps):
        one_step()
        steps += 1
        coords += sample
    seconds = time.perf_counter() - started
    value = coords / seconds
    line = {'metric': METRIC, 'value': value, 'unit': UNIT, 'n_gpus': args.gpus, 'steps': args.steps,
            'warmup': args.warmup, 'ms_per_step': seconds / steps * 1e3, 'higher_is_better': True, 'scaling': 'weak',
            'vs_baseline': None, 'dtype': 'f32' if args.workload == 'c1-hash' else 'f32/f16', 'data': 'synthetic',
            'impl': 'reference',
            'config': {'workload': args.workload, 'batch_per_step': sample, 'full_batch': args.batch,
                       'note': 'bounded sample of the workload per step (full model and layout)'},
            'cpu_baseline': {'value': value, 'unit': UNIT, 'cores': threads, 'kind': 'port',
                             'sample': f'{steps} steps x {sample} coords, torch CPU restatement, {threads} threads'},
            'e2e': {'value': value, 'unit': UNIT, 'h2d_bytes_per_step': 0, 'd2h_bytes_per_step': 0}}
    print(json.dumps(line), flush=True)


def allocate(args, lib, opt, model, target, shape):
    """c3: the on-demand allocation stage on the current model: decode every pixel, the fp64 residual of every
    256 x 256 tile, the exact top 30 %, and the expert levels restricted to the chosen tiles' cells.  Timed with CUDA
    events; returns the tile mask and the timings."""
    from odie_b200 import _lib
    from odie_b200.workloads import C3_TILE
    height, width = shape
    tiles_y, tiles_x = -(-height // C3_TILE), -(-width // C3_TILE)
    count = tiles_x * tiles_y
    k = int(round(0.3 * count))
    stream = torch.cuda.current_stream()
    prediction = torch.empty((height * width, 3), device='cuda')
    scores = torch.empty(count, dtype=torch.float64, device='cuda')
    chosen = torch.empty(k, dtype=torch.int64, device='cuda')
    selected = torch.empty(count, dtype=torch.uint8, device='cuda')
    row_sums = torch.empty(count * C3_TILE, dtype=torch.float64, device='cuda')
    events = [torch.cuda.Event(enable_timing=True) for _ in range(5)]
    torch.cuda.synchronize()
    events[0].record()
    opt.decode(0, height * width, rgb=prediction)
    events[1].record()
    _lib.check(lib.odie_tile_topk(prediction.data_ptr(), target.data.data_ptr(), height, width, C3_TILE, k,
                                  row_sums.data_ptr(), scores.data_ptr(), chosen.data_ptr(), selected.data_ptr(),
                                  stream.cuda_stream))
    events[2].record()
    tiles = selected.reshape(tiles_y, tiles_x)
    model.set_allocation(tiles, C3_TILE, shape)
    events[3].record()
    opt.check(lib.odie_configure(opt.handle, json.dumps(opt.current_settings()).encode()))
    events[4].record()
    torch.cuda.synchronize()
    return {'tiles': tiles.bool(), 'tiles_allocated': k, 'tiles_total': count, 'tile_px': C3_TILE,
            'decode_ms': events[0].elapsed_time(events[1]), 'score_select_ms': events[1].elapsed_time(events[2]),
            'bitmaps_ms': events[2].elapsed_time(events[3]), 'configure_ms': events[3].elapsed_time(events[4]),
            'stage_ms': events[0].elapsed_time(events[4]),
            'sampling': ('70 % of coordinates on jittered strata spread evenly over the allocated tiles, 30 % on '
                         'jittered strata over the image, tile by tile' if args.sampling == 'stratified' else
                         '70 % of coordinates uniform in the allocated tiles, 30 % uniform over the image (iid)')}


def allocate_global(args, lib, opt, model, target, shape, dist):
    """c4: the allocation stage over the whole gigapixel image, split across ranks.  Each rank decodes its own rows
    one row of 256 x 256 tiles at a time and scores those tiles (fp64 residual, odie_tile_topk with k = 0); the
    ranks' scores are gathered in row order, every rank takes the same exact top 20 % of all tiles (odie_topk) and
    restricts the expert levels to the chosen tiles' cells with the full image's geometry, so the model is the same
    at every GPU count.  Returns the rank's own rows of the tile mask and the timings."""
    from odie_b200 import _lib
    from odie_b200.workloads import C4_ALLOCATED, C4_TILE
    tile = C4_TILE
    rows, width = shape
    row0 = int(opt.config.get('row_offset', 0))
    full_rows = model.image_rows
    if row0 % tile or rows % tile or full_rows % tile:
        raise ValueError('the rank rows must be whole rows of tiles')
    tiles_x, local_ty, full_ty = -(-width // tile), rows // tile, full_rows // tile
    stream = torch.cuda.current_stream()
    prediction = torch.empty((tile * width, 3), device='cuda')
    row_sums = torch.empty(tiles_x * tile, dtype=torch.float64, device='cuda')
    local = torch.empty(local_ty * tiles_x, dtype=torch.float64, device='cuda')
    events = [torch.cuda.Event(enable_timing=True) for _ in range(5)]
    torch.cuda.synchronize()
    events[0].record()
    for ty in range(local_ty):
        opt.decode(ty * tile * width, tile * width, rgb=prediction)
        _lib.check(lib.odie_tile_topk(prediction.data_ptr(), target.data.data_ptr() + ty * tile * width * 3, tile,
                                      width, tile, 0, row_sums.data_ptr(), local[ty * tiles_x:].data_ptr(), None, None,
                                      stream.cuda_stream))
    events[1].record()
    if dist is not None:
        gathered = [torch.empty_like(local) for _ in range(dist.get_world_size())]
        dist.all_gather(gathered, local)
        scores = torch.cat(gathered)
    else:
        scores = local
    count = full_ty * tiles_x
    k = int(round(C4_ALLOCATED * count))
    chosen = torch.empty(k, dtype=torch.int64, device='cuda')
    selected = torch.empty(count, dtype=torch.uint8, device='cuda')
    _lib.check(lib.odie_topk(scores.data_ptr(), count, k, chosen.data_ptr(), selected.data_ptr(), stream.cuda_stream))
    events[2].record()
    tiles = selected.reshape(full_ty, tiles_x)
    model.set_allocation(tiles, tile, (full_rows, width))
    events[3].record()
    opt.check(lib.odie_configure(opt.handle, json.dumps(opt.current_settings()).encode()))
    events[4].record()
    torch.cuda.synchronize()
    first = row0 // tile
    return {'tiles': tiles[first:first + local_ty].bool(), 'tiles_allocated': k, 'tiles_total': count, 'tile_px': tile,
            'decode_and_score_ms': events[0].elapsed_time(events[1]), 'select_ms': events[1].elapsed_time(events[2]),
            'bitmaps_ms': events[2].elapsed_time(events[3]), 'configure_ms': events[3].elapsed_time(events[4]),
            'stage_ms': events[0].elapsed_time(events[4]),
            'bitmap_bytes': int(model.allocation_bitmap.numel()),
            'sampling': ('70 % of coordinates on jittered strata spread evenly over the allocated tiles of the rank, '
                         '30 % on jittered strata over the rank\'s rows, tile by tile' if args.sampling == 'stratified'
                         else '70 % uniform in the rank\'s allocated tiles, 30 % uniform over its rows (iid)')}


def main():
    args = parse()
    if args.batch is None:
        args.batch = BATCHES[args.workload]
    if args.impl == 'reference':
        run_reference(args)
        return
    if args.workload == 'c1-hash':
        main_c1(args)
        return
    rank, world = int(os.environ.get('RANK', 0)), int(os.environ.get('WORLD_SIZE', 1))
    local = int(os.environ.get('LOCAL_RANK', 0))
    torch.cuda.set_device(local)
    torch.cuda.set_stream(torch.cuda.Stream())  # a dedicated training stream, as odie/train.py:73-75
    dist = None
    if world > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group('nccl', timeout=datetime.timedelta(seconds=300), device_id=torch.device('cuda', local))
    from odie_b200 import _lib, parallel
    from odie_b200.native_backend import NativeOptimizer
    from odie_b200.workloads import C4_TILE, allocated_ids, allocated_stratified_ids, fp16_payload_bytes
    lib = _lib.library()
    c4 = args.workload == 'c4-experts'
    experts = args.workload.endswith('experts')
    w = workload(args.workload, rank, world, args.batch, args.shape if c4 else None)
    config, shape, model = w['config'], w['shape'], w['model']
    shared = head_grad = router_grad = None
    if world > 1:
        # the shared parameters: every rank starts from rank 0's and applies the same summed gradient
        parallel.broadcast_heads(model)
        if c4:
            dist.broadcast(model.router_grid.data, 0)
        shared, head_grad, router_grad = parallel.head_gradient_buffer(model, router_grid=c4)
    # c4 decodes in launches of 2^24 pixels: the runtime's buffers hold that many coordinates
    capacity = max(args.batch, args.decode_launch) if c4 else args.batch
    # one GPU, routed experts: the runtime's pipeline mode (each step's backward branches overlap the next step's
    # forward; odie_join before every stop event)
    pipelined = world == 1 and experts
    opt = NativeOptimizer(model, w['target'], shape, config, w['planes'], batch=capacity, head_grad=head_grad,
                          router_grad=router_grad, pipeline=pipelined)
    runtime = parallel.NativeRuntime(opt)
    overlap = runtime.side_stream() if world > 1 else None
    dp_step = parallel.DataParallelStep(runtime, shared, overlap_stream=overlap)
    pixels = shape[0] * shape[1]
    gen = torch.Generator(device='cuda').manual_seed(1729 + rank)
    total_steps = args.warmup + args.steps
    allocation = None
    if args.workload in ('c3-experts', 'c4-experts'):
        if c4:
            allocation = allocate_global(args, lib, opt, model, w['target'], shape, dist)
        else:
            allocation = allocate(args, lib, opt, model, w['target'], shape)
        sampler = allocated_stratified_ids if args.sampling == 'stratified' else allocated_ids
        tile_px = allocation['tile_px']
        ids = torch.stack([sampler(allocation['tiles'], shape, args.batch, gen, tile_px=tile_px)
                           for _ in range(total_steps)])
        allocation = {k: v for k, v in allocation.items() if k != 'tiles'}
    elif args.sampling == 'stratified':
        from odie_b200.data import stratified_batches
        ids = torch.stack(list(stratified_batches(shape, args.batch, gen, steps=total_steps)))
    else:
        ids = torch.randint(0, pixels, (total_steps, args.batch), device='cuda', generator=gen)

    def step(batch_ids):
        if world == 1:
            opt.check(lib.odie_step(opt.handle, batch_ids.data_ptr(), batch_ids.numel(), 1))
        else:
            dp_step(batch_ids)

    def barrier():
        torch.cuda.synchronize()
        if dist is not None:
            dist.barrier()
        torch.cuda.synchronize()

    def view(name, count, typestr='<f4'):
        return torch.as_tensor(DeviceArray(opt.pointers[name], count, typestr), device='cuda')

    # warm-up; its first step keeps the grid gradients long enough to count the parameters a step touches
    # (the zero-skipping Adam reads p, m, v only for those)
    grid_params = model.grid.numel() + (model.router_grid.numel() if experts else 0)
    opt.check(lib.odie_step_grads(opt.handle, ids[0].data_ptr(), args.batch, 2))
    touched = int(torch.count_nonzero(view('grid_grad', model.grid.numel())))
    if experts:
        touched += int(torch.count_nonzero(view('router_grad', model.router_grid.numel())))
    opt.check(lib.odie_grid_update(opt.handle))
    if dist is not None:
        dist.all_reduce(shared)
    opt.check(lib.odie_step_heads(opt.handle))
    for k in range(1, args.warmup):
        step(ids[k])
    barrier()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with Clocks(local) as clocks:
        barrier()
        launches_before = lib.odie_launch_count()
        start.record()
        for k in range(args.steps):
            step(ids[args.warmup + k])
        opt.check(lib.odie_join(opt.handle))
        end.record()
        launches = lib.odie_launch_count() - launches_before
        barrier()
    ms = start.elapsed_time(end)
    # Stage timers (the roofline's kernel durations): a second pass of the same K steps with CUDA events between
    # the stages and the step's two branches serialised on one stream, so that each stage's time is its own
    # kernels' (concurrent branches would charge each other's waits).  Not part of `value`.
    dp_step.overlap_stream = None
    opt.check(lib.odie_profile(opt.handle, 2))
    barrier()
    for k in range(args.steps):
        step(ids[args.warmup + k])
    barrier()
    report = json.loads(lib.odie_profile_report(opt.handle))
    opt.check(lib.odie_profile(opt.handle, 0))
    dp_step.overlap_stream = overlap
    ms_t = torch.tensor([ms], device='cuda')
    if dist is not None:
        dist.all_reduce(ms_t, op=dist.ReduceOp.MAX)
    ms = float(ms_t)
    value = world * args.batch * args.steps / (ms / 1e3)

    # end to end through the public API: pinned host ids in, loss out, every step.  As a training
    # loop's data loader does, step k + 1's ids upload on a copy stream (double buffer) while
    # step k runs; every copy is inside the timed region.
    host_ids = ids[args.warmup:].cpu().pin_memory()
    device_ids = [torch.empty(args.batch, dtype=torch.int64, device='cuda') for _ in range(2)]
    loss_host = torch.empty(args.steps, dtype=torch.float64).pin_memory()
    # the runtime's per-sample squared errors, viewed in place: the loss is their fp64 mean.  Each step's
    # errors are copied (device to device) on a loss stream, and the next step waits only for that copy;
    # the reduction and the 8-byte read to the host run beside the next step.
    squares = view('squares', args.batch)
    main_stream, copy_stream, loss_stream = torch.cuda.current_stream(), torch.cuda.Stream(), torch.cuda.Stream()
    uploaded = [torch.cuda.Event() for _ in range(2)]
    released = [torch.cuda.Event() for _ in range(2)]
    stepped = [torch.cuda.Event() for _ in range(2)]
    copied = [torch.cuda.Event() for _ in range(2)]
    snapshots = [torch.empty(args.batch, device='cuda') for _ in range(2)]

    def read_loss(k):
        buf = k % 2
        stepped[buf].record(main_stream)
        with torch.cuda.stream(loss_stream):
            loss_stream.wait_event(stepped[buf])
            snapshots[buf].copy_(squares)
            copied[buf].record(loss_stream)
            loss_host[k:k + 1].copy_((snapshots[buf].sum(dtype=torch.float64) / args.batch).reshape(1),
                                     non_blocking=True)

    def upload(k):
        buf = k % 2
        with torch.cuda.stream(copy_stream):
            if k >= 2:
                copy_stream.wait_event(released[buf])  # step k - 2 has consumed this buffer
            device_ids[buf].copy_(host_ids[k], non_blocking=True)
            uploaded[buf].record(copy_stream)

    # warm-up of the loop's own operations (the loss read's torch kernels load lazily on first use)
    read_loss(0)
    upload(0)
    barrier()
    e_start, e_end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e_start.record()
    copy_stream.wait_event(e_start)
    upload(0)
    for k in range(args.steps):
        buf = k % 2
        if k + 1 < args.steps:
            upload(k + 1)
        main_stream.wait_event(uploaded[buf])
        if k >= 1:
            main_stream.wait_event(copied[(k - 1) % 2])  # step k - 1's errors are copied out
        step(device_ids[buf])
        released[buf].record(main_stream)
        read_loss(k)
    main_stream.wait_stream(loss_stream)  # the last loss has reached the host buffer
    opt.check(lib.odie_join(opt.handle))
    e_end.record()
    barrier()
    e_ms = torch.tensor([e_start.elapsed_time(e_end)], device='cuda')
    if dist is not None:
        dist.all_reduce(e_ms, op=dist.ReduceOp.MAX)
    e2e = world * args.batch * args.steps / (float(e_ms) / 1e3)
    losses = loss_host.numpy()

    # the sampler of a training loop, per step: the reference's stratified_batches (torch RNG and
    # arithmetic kernels) against the device sampler, and the step with the sampler fused in
    sampler = None
    if world == 1 and args.workload in ('c2-experts', 'c2-planes') and args.sampling == 'stratified':
        from odie_b200.data import device_stratified_ids, stratified_batches
        reps = 10
        s_events = [torch.cuda.Event(enable_timing=True) for _ in range(6)]
        batches = stratified_batches(shape, args.batch, torch.Generator(device='cuda').manual_seed(7), steps=2 * reps)
        next(batches)
        device_stratified_ids(shape, args.batch, 7, 0)
        barrier()
        s_events[0].record()
        for _ in range(reps):
            next(batches)
        s_events[1].record()
        for k in range(reps):
            device_stratified_ids(shape, args.batch, 7, k)
        s_events[2].record()
        for k in range(args.steps):
            opt.check(lib.odie_step_stratified(opt.handle, 7, k, args.batch, 1))
        opt.check(lib.odie_join(opt.handle))
        s_events[3].record()
        barrier()
        sampler = {'torch_stratified_ms': s_events[0].elapsed_time(s_events[1]) / reps,
                   'device_stratified_ms': s_events[1].elapsed_time(s_events[2]) / reps,
                   'fused_step_ms': s_events[2].elapsed_time(s_events[3]) / args.steps,
                   'step_ms': ms / args.steps,
                   'note': 'stratified_batches (odie/data.py:63-80) as the reference runs it each step, vs '
                           'odie_stratified_ids; odie_step_stratified = odie_step with the sampler fused in'}

    # decode of this rank's rows, every pixel (c4: the gigapixel reconstruction in launches of 2^24 pixels)
    rgb8 = torch.empty((pixels, 3), dtype=torch.uint8, device='cuda')
    opt.decode(0, pixels, rgb8=rgb8)
    barrier()
    d_start, d_end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    repeats = 2 if c4 else 5
    d_start.record()
    for _ in range(repeats):
        opt.decode(0, pixels, rgb8=rgb8)
    d_end.record()
    barrier()
    d_ms = torch.tensor([d_start.elapsed_time(d_end)], device='cuda')
    if dist is not None:
        dist.all_reduce(d_ms, op=dist.ReduceOp.MAX)
    d_seconds = float(d_ms) / 1e3
    decode_gpix = world * pixels * repeats / d_seconds / 1e9
    del rgb8

    probe = l2_probe(lib) if rank == 0 else None
    if rank == 0:
        hbm, tensor_burst, tensor_sustained, peak_kind = peaks()
        units = per_coordinate(args.workload, model)
        stages = {k: v for k, v in report.items() if v['launches']}
        per_stage = {}
        for k, v in stages.items():
            seconds = v['ms'] / args.steps / 1e3
            bound, work = units.get(k, ('hbm', None))
            if work is not None:
                work = work * args.batch
            if k == 'adam_grid':
                work = adam_bytes(grid_params, touched)
            if k == 'encode_backward':
                work += 8 * touched  # each touched gradient entry read and written once
            if k == 'input_batch':
                work = (8 + 3 + 8 + 12) * args.batch  # id, u8 target in; xy, fp32 target out
            achieved = (work / seconds / (1e12 if bound == 'tensor' else 1e9)) if work else None
            peak = tensor_sustained if bound == 'tensor' else hbm
            per_stage[k] = {'ms_per_step': v['ms'] / args.steps, 'launches_per_step': v['launches'] / args.steps,
                            'bound': bound, 'algorithmic_per_step': work, 'achieved': achieved,
                            'unit': 'TFLOP/s' if bound == 'tensor' else 'GB/s',
                            'frac': (achieved / peak) if achieved else None}
            if k == 'encode_backward':
                # the per-corner atomic algorithm's reductions, and their time at the probe's L2 reduction rate
                atomics = (2 if experts else 1) * model.n_levels * 4 * args.batch
                per_stage[k]['naive_atomics_per_step'] = atomics
                per_stage[k]['naive_atomics_ms_at_l2_probe'] = atomics / (probe['gops']['red8'] * 1e9) * 1e3
        dominant = max(stages, key=lambda k: stages[k]['ms'])
        d = per_stage[dominant]
        peak = tensor_sustained if d['bound'] == 'tensor' else hbm
        roofline = {'kernel': dominant, 'bound': d['bound'], 'achieved': d['achieved'], 'peak': peak,
                    'unit': d['unit'], 'frac': d['frac'], 'traffic': traffic_of(args.workload, dominant),
                    'traffic_unit': 'DRAM bytes per step (ncu, profiles/dram_traffic.json)',
                    'algorithmic_per_step': d['algorithmic_per_step'],
                    'peak_source': f'{peak_kind} ({"sustained dense bf16" if d["bound"] == "tensor" else "HBM copy"})',
                    'timing': 'stage events with the step branches serialised (kernel time)',
                    'share': stages[dominant]['ms'] / sum(v['ms'] for v in stages.values()),
                    'touched_params_per_step': touched, 'grid_params': grid_params,
                    'stages': per_stage, 'l2_probe_gops': probe['gops']}
        dec_bytes, dec_flop = decode_per_pixel(args.workload, model)
        dec_rate = pixels * repeats / d_seconds
        decode = {'value': decode_gpix, 'unit': 'Gpix/s', 'pixels_per_rank': pixels,
                  'launch_pixels': min(capacity, pixels), 'launches_per_pass': -(-pixels // capacity),
                  'roofline': {'bound': 'hbm', 'algorithmic_bytes_per_pixel': dec_bytes,
                               'achieved': dec_rate * dec_bytes / 1e9, 'peak': hbm, 'unit': 'GB/s',
                               'frac': dec_rate * dec_bytes / 1e9 / hbm, 'flop_per_pixel': dec_flop,
                               'tflops': dec_rate * dec_flop / 1e12,
                               'note': 'table corner reads of both encodings + u8 out; the tables are L2-resident'}}
        base = None
        if world == 1 and not args.no_cpu_baseline:
            legs = cpu_legs(args)
            base = dict(legs[0], one_thread=legs[1])
        payload = fp16_payload_bytes(model) if experts else 2 * (model.grid.numel() + model.decoder.params.numel())
        line = {'metric': METRIC, 'value': value, 'unit': UNIT, 'n_gpus': world, 'steps': args.steps,
                'warmup': args.warmup, 'ms_per_step': ms / args.steps, 'higher_is_better': True, 'scaling': 'weak',
                'vs_baseline': None, 'dtype': 'f16 (fp32 masters, fp32 accumulate)', 'data': 'synthetic',
                'config': {'workload': args.workload,
                           'image_hw': [model.image_rows, shape[1]] if c4 else list(shape),
                           'rows_per_rank': shape[0], 'global_batch': world * args.batch,
                           'batch_per_gpu': args.batch, 'levels': model.n_levels,
                           'grid_params_per_rank': model.grid.numel(),
                           'experts': getattr(model, 'experts', None),
                           'experts_per_rank': getattr(model, 'experts_held', None),
                           'bands': getattr(model, 'bands', None),
                           'fp16_payload_mib': payload / 2 ** 20,
                           'parallelism': (f'dp{world} (one model: 8 row bands of 8 experts split over ranks; '
                                           'all-reduce of router MLP + decoder + router grid)' if c4 else
                                           f'dp{world} (row bands, head all-reduce)'),
                           'sampling': (args.sampling + (' (reference default, odie/config.py:20)'
                                                         if args.sampling == 'stratified' else ' (iid)')
                                        + (', 70 % in the allocated tiles' if allocation else '')),
                           'l2': 'per-step inputs and activations (c4: > 1 GB) larger than L2; model tables '
                                 'L2-resident',
                           'schedule': ('pipelined: each step\'s backward branches overlap the next step\'s forward '
                                        '(odie_join before the stop event)' if pipelined else 'one step at a time')},
                'e2e': {'value': e2e, 'unit': UNIT, 'h2d_bytes_per_step': args.batch * 8, 'd2h_bytes_per_step': 8},
                'gpu_launches': launches, 'roofline': roofline, 'cpu_baseline': base, 'decode': decode,
                'loss_first_last': [float(losses[0]), float(losses[-1])], 'clocks': clocks.summary()}
        if allocation:
            line['allocation'] = allocation
        if sampler:
            line['sampler'] = sampler
        print(json.dumps(line), flush=True)
    opt.close()
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()


def fma_peak(lib, iterations=1 << 16):
    """Measured fp32 FMA throughput of this GPU (TFLOP/s; odie_fma_probe, best of 3)."""
    sink = torch.zeros(1, device='cuda')
    stream = torch.cuda.current_stream()
    lib.odie_fma_probe(iterations, sink.data_ptr(), stream.cuda_stream)  # warm-up
    best = float('inf')
    for _ in range(3):
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record()
        flop = lib.odie_fma_probe(iterations, sink.data_ptr(), stream.cuda_stream)
        end.record()
        end.synchronize()
        best = min(best, start.elapsed_time(end))
    return flop / (best / 1e3) / 1e12


def main_c1(args):
    """c1-hash: the single fp32 hash grid through odie_hashgrid32_* (one GPU per process; each rank trains its
    own replica on its own coordinates, no exchange)."""
    rank, world = int(os.environ.get('RANK', 0)), int(os.environ.get('WORLD_SIZE', 1))
    local = int(os.environ.get('LOCAL_RANK', 0))
    torch.cuda.set_device(local)
    torch.cuda.set_stream(torch.cuda.Stream())
    dist = None
    if world > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group('nccl', timeout=datetime.timedelta(seconds=300), device_id=torch.device('cuda', local))
    from odie_b200 import _lib
    from odie_b200.hashgrid32 import HEAD_PARAMS, HashGrid32, HashGrid32Trainer, c1_config, c1_image
    lib = _lib.library()
    n = args.batch
    config = c1_config(seed=1729 + rank, batch=n)
    model = HashGrid32(config)
    image = c1_image(1729)
    trainer = HashGrid32Trainer(model, image, n)
    seed = 1729 + rank

    def barrier():
        torch.cuda.synchronize()
        if dist is not None:
            dist.barrier()
        torch.cuda.synchronize()

    # a first step whose gradient is kept for inspection counts the table entries a step touches (the entries the
    # scatter writes); its update then runs as a warm-up step's would
    trainer.step(step=0, seed=seed, update=False)
    touched = int(torch.count_nonzero(trainer.read('grid_grad', model.total)))
    trainer.update()
    for k in range(args.warmup):
        trainer.step(step=k, seed=seed)
    barrier()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with Clocks(local) as clocks:
        barrier()
        launches_before = lib.odie_launch_count()
        start.record()
        for k in range(args.steps):
            trainer.step(step=args.warmup + k, seed=seed)
        end.record()
        launches = lib.odie_launch_count() - launches_before
        barrier()
    ms_t = torch.tensor([start.elapsed_time(end)], device='cuda')
    if dist is not None:
        dist.all_reduce(ms_t, op=dist.ReduceOp.MAX)
    ms = float(ms_t)
    value = world * n * args.steps / (ms / 1e3)
    # stage times: CUDA events around each stage's launches (one stream, so each is its kernels' own time)
    _lib.check(lib.odie_hashgrid32_profile(trainer.handle, 1))
    for k in range(args.steps):
        trainer.step(step=args.warmup + k, seed=seed)
    report = json.loads(lib.odie_hashgrid32_profile_report(trainer.handle))
    _lib.check(lib.odie_hashgrid32_profile(trainer.handle, 0))
    # end to end: each step's coordinates from pinned host memory (uploaded on a copy stream one step ahead) and
    # its mean loss read back to the host
    host_xy = torch.rand((args.steps, n, 2), generator=torch.Generator().manual_seed(seed)).pin_memory()
    device_xy = [torch.empty((n, 2), device='cuda') for _ in range(2)]
    loss_host = torch.empty(args.steps, dtype=torch.float64).pin_memory()
    main_stream, copy_stream = torch.cuda.current_stream(), torch.cuda.Stream()
    uploaded = [torch.cuda.Event() for _ in range(2)]
    released = [torch.cuda.Event() for _ in range(2)]
    squares = trainer.read('squares', n)

    def upload(k):
        with torch.cuda.stream(copy_stream):
            if k >= 2:
                copy_stream.wait_event(released[k % 2])
            device_xy[k % 2].copy_(host_xy[k], non_blocking=True)
            uploaded[k % 2].record(copy_stream)
    def read_loss(k):
        _lib.check(lib.odie_copy(squares.data_ptr(), int(trainer.buffers['squares']), 4 * n, main_stream.cuda_stream))
        loss_host[k:k + 1].copy_((squares.sum(dtype=torch.float64) / n).reshape(1), non_blocking=True)
    # warm-up of the loop's own operations (torch loads the reduction's kernels on first use)
    upload(0)
    main_stream.wait_event(uploaded[0])
    trainer.step(step=0, xy=device_xy[0])
    read_loss(0)
    barrier()
    e_start, e_end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e_start.record()
    copy_stream.wait_event(e_start)
    upload(0)
    for k in range(args.steps):
        if k + 1 < args.steps:
            upload(k + 1)
        main_stream.wait_event(uploaded[k % 2])
        trainer.step(step=k, xy=device_xy[k % 2])
        released[k % 2].record(main_stream)
        read_loss(k)
    e_end.record()
    barrier()
    e_ms = torch.tensor([e_start.elapsed_time(e_end)], device='cuda')
    if dist is not None:
        dist.all_reduce(e_ms, op=dist.ReduceOp.MAX)
    e2e = world * n * args.steps / (float(e_ms) / 1e3)
    # decode of the whole image, fp32 RGB
    pixels = image.shape[0] * image.shape[1]
    rgb = torch.empty((pixels, 3), device='cuda')
    trainer.decode(begin=0, n=pixels, out=rgb)
    barrier()
    d_start, d_end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    repeats = 20
    d_start.record()
    for _ in range(repeats):
        trainer.decode(begin=0, n=pixels, out=rgb)
    d_end.record()
    barrier()
    d_seconds = d_start.elapsed_time(d_end) / 1e3
    if rank == 0:
        hbm, _, _, peak_kind = peaks()
        fma = fma_peak(lib)
        flop_per_coord = 2 * 3 * (32 * 64 + 64 * 64 + 64 * 3)  # forward, data backward, weight gradients
        total = model.total
        work = {'fused_step': ('fp32', flop_per_coord * n),
                # xy and the fp32 feature-gradient row read once, each touched table entry read and written once
                'encode_backward': ('hbm', (8 + 4 * 32) * n + 8 * touched),
                'reduce_partials': ('hbm', None),
                'adam_grid': ('hbm', 40 * total),  # g, p, m, v, step read; p, m, v, step written; g cleared
                'adam_heads': ('hbm', None)}
        per_stage = {}
        for k, v in report.items():
            if not v['launches']:
                continue
            seconds = v['ms'] / args.steps / 1e3
            bound, amount = work[k]
            achieved = (amount / seconds / (1e12 if bound == 'fp32' else 1e9)) if amount else None
            peak = fma if bound == 'fp32' else hbm
            per_stage[k] = {'ms_per_step': v['ms'] / args.steps, 'bound': bound, 'algorithmic_per_step': amount,
                            'achieved': achieved, 'unit': 'TFLOP/s' if bound == 'fp32' else 'GB/s',
                            'frac': achieved / peak if achieved else None}
        dominant = max(per_stage, key=lambda k: per_stage[k]['ms_per_step'])
        d = per_stage[dominant]
        roofline = {'kernel': dominant, 'bound': 'fp32 CUDA-core FMA' if d['bound'] == 'fp32' else 'hbm',
                    'achieved': d['achieved'], 'peak': fma if d['bound'] == 'fp32' else hbm, 'unit': d['unit'],
                    'frac': d['frac'], 'traffic': traffic_of('c1-hash', dominant),
                    'peak_source': ('measured (odie_fma_probe, fp32 FMA)' if d['bound'] == 'fp32'
                                    else f'{peak_kind} (HBM copy)'),
                    'timing': 'stage events on one stream (kernel time)', 'touched_params_per_step': touched,
                    'stages': per_stage}
        dec_bytes = 16 * 4 * 8 + 8 + 12
        base = None
        if world == 1 and not args.no_cpu_baseline:
            legs = cpu_legs(args)
            base = dict(legs[0], one_thread=legs[1])
        losses = loss_host.numpy()
        line = {'metric': METRIC, 'value': value, 'unit': UNIT, 'n_gpus': world, 'steps': args.steps,
                'warmup': args.warmup, 'ms_per_step': ms / args.steps, 'higher_is_better': True, 'scaling': 'weak',
                'vs_baseline': None, 'dtype': 'f32', 'data': 'synthetic',
                'config': {'workload': 'c1-hash', 'image_hw': list(image.shape[:2]), 'global_batch': world * n,
                           'batch_per_gpu': n, 'levels': 16, 'log2_hashmap_size': 19, 'grid_params': total,
                           'head_params': HEAD_PARAMS, 'sampling': 'uniform (Philox on the device), bilinear targets',
                           'parallelism': f'replicas{world} (each GPU its own model and coordinates)',
                           'l2': 'per-step activations (dx rows 32 MB) and the 30.6 MB table; dense Adam state '
                                 '92 MB: inputs larger than L2 across the step'},
                'e2e': {'value': e2e, 'unit': UNIT, 'h2d_bytes_per_step': 8 * n, 'd2h_bytes_per_step': 8},
                'gpu_launches': launches, 'roofline': roofline, 'cpu_baseline': base,
                'decode': {'value': pixels * repeats / d_seconds / 1e9, 'unit': 'Gpix/s', 'pixels': pixels,
                           'roofline': {'bound': 'hbm', 'algorithmic_bytes_per_pixel': dec_bytes,
                                        'achieved': pixels * repeats / d_seconds * dec_bytes / 1e9, 'peak': hbm,
                                        'frac': pixels * repeats / d_seconds * dec_bytes / 1e9 / hbm,
                                        'note': 'fp32 corner reads (L2-resident table) + fp32 RGB out'}},
                'fma_peak_tflops': fma, 'loss_first_last': [float(losses[0]), float(losses[-1])],
                'clocks': clocks.summary()}
        print(json.dumps(line), flush=True)
    trainer.close()
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == '__main__':
    main()
