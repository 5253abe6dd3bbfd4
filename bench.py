"""Benchmark of the ODIE hot path on B200: train coords/s (fwd + bwd + Adam) and decode Gpix/s.

python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--workload c2-planes]

One JSON line on rank 0.  `value` is whole-job coords/s with inputs resident in
HBM (device-timed with CUDA events, max over ranks); `e2e` is the same metric
through the public API with the step's pixel ids copied from pinned host memory
and the loss read back every step.  Multi-GPU: one process per GPU (torchrun),
each rank trains the model of its own row band of the image (weak scaling),
and only the shared head gradients cross GPUs (NCCL all-reduce).  The
`--impl reference` arm times the CPU restatement of the reference step
(oracle/cpu_step.py; the reference has no CPU path of its own).
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
BATCH = 1 << 20


def parse():
    p = argparse.ArgumentParser()
    p.add_argument('--gpus', type=int, default=1)
    p.add_argument('--steps', type=int, default=20)
    p.add_argument('--warmup', type=int, default=5)
    p.add_argument('--impl', choices=['ours', 'reference'], default='ours')
    p.add_argument('--workload', default='c2-planes')
    p.add_argument('--batch', type=int, default=BATCH)
    p.add_argument('--no-cpu-baseline', action='store_true')
    return p.parse_args()


def workload(name, rank, ranks, batch):
    from odie_b200 import workloads
    if name != 'c2-planes':
        raise SystemExit(f'unknown workload {name}')
    return workloads.c2_planes(batch=batch, band=(rank, ranks))


class Clocks:
    """nvidia-smi sampling of SM clocks and throttle reasons during the timed region."""
    QUERY = ('index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,'
             'clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,'
             'clocks_event_reasons.sw_power_cap')

    def __init__(self, index):
        self.index, self.samples, self.stop = index, [], threading.Event()
        self.thread = threading.Thread(target=self.run, daemon=True)

    def run(self):
        while not self.stop.is_set():
            try:
                out = subprocess.run(['nvidia-smi', f'--id={self.index}', f'--query-gpu={self.QUERY}',
                                      '--format=csv,noheader,nounits'], capture_output=True, text=True, timeout=5)
                if out.returncode == 0 and out.stdout.strip():
                    self.samples.append([s.strip() for s in out.stdout.strip().split(',')])
            except Exception:
                pass
            self.stop.wait(0.2)

    def __enter__(self):
        self.thread.start()
        return self

    def __exit__(self, *a):
        self.stop.set()
        self.thread.join(timeout=10)

    def summary(self):
        if not self.samples:
            return {'sm_mhz': None, 'sm_max_mhz': None, 'reasons': ['unsampled'], 'samples': 0}
        sm = [float(s[1]) for s in self.samples if s[1].replace('.', '').isdigit()]
        mx = [float(s[2]) for s in self.samples if s[2].replace('.', '').isdigit()]
        names = ['hw_slowdown', 'hw_thermal_slowdown', 'sw_thermal_slowdown', 'sw_power_cap']
        reasons = sorted({names[i] for s in self.samples for i in range(4) if len(s) > 5 + i and s[5 + i] == 'Active'})
        return {'sm_mhz': float(np.median(sm)) if sm else None, 'sm_max_mhz': max(mx) if mx else None,
                'reasons': reasons, 'samples': len(self.samples)}


def algorithmic(stage, levels, features, n, params, head_flops):
    """Algorithmic bytes (or FLOPs) of one launch of a stage, per the per-unit figures in DESIGN.md."""
    L, F = levels, features
    if stage == 'encode_forward':
        return 'hbm', (8 + 4 * L * F * 2 + L * F * 2) * n
    if stage == 'encode_backward':
        return 'hbm', (8 + L * F * 2 + 8 * L * F * 4) * n
    if stage == 'mlp_train':
        return 'tensor', head_flops * n
    if stage == 'adam_grid':
        return 'hbm', 30 * params
    return 'hbm', None


def peaks():
    path = ROOT / 'MEASURED_PEAKS.json'
    if path.exists():
        data = json.loads(path.read_text())
        return data['hbm_gbs'], data['bf16_tflops'], 'measured'
    return 6650.0, 1590.0, 'fallback'


def cpu_baseline(args, budget=12.0):
    """The CPU restatement of the reference step on this host's cores (bounded sample)."""
    from oracle.cpu_step import CpuStep, plane_levels_for_cpu
    from odie_b200 import layout as host_layout
    config, supports, dims, caps, rgb, shape = workload(args.workload, 0, 1, args.batch)
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    lay = host_layout.make_layout(config, supports, dims, caps)
    levels = plane_levels_for_cpu(lay['descriptors'].numpy(), lay['node_bitmap'].numpy(), lay['node_prefix'].numpy(),
                                  lay['bitmap'].numpy())
    rng = np.random.default_rng(0)
    grid = (rng.standard_normal(lay['params']) * 1e-3).astype(np.float32)
    width = (lay['input_width'] + 15) // 16 * 16
    gate = (rng.standard_normal(width * 32 + 32 * 16) * .1).astype(np.float32)
    decoder = (rng.standard_normal(width * 64 + 64 * 64 + 64 * 16) * .1).astype(np.float32)
    step = CpuStep(shape, rgb.numpy(), levels, grid, gate, decoder, width)
    sample = 1 << 14
    pixels = shape[0] * shape[1]
    g = torch.Generator().manual_seed(1)
    step.step(torch.randint(0, pixels, (sample,), generator=g))  # warm-up
    started, coords = time.perf_counter(), 0
    while time.perf_counter() - started < budget:
        step.step(torch.randint(0, pixels, (sample,), generator=g))
        coords += sample
    seconds = time.perf_counter() - started
    return {'value': coords / seconds, 'unit': UNIT, 'cores': threads, 'kind': 'port',
            'sample': f'{coords // sample} steps of {sample} coords of {args.workload} (same layout, batch scaled '
                      f'down), torch CPU, {threads} threads, {seconds:.1f} s'}


def run_reference(args):
    rank = int(os.environ.get('RANK', 0))
    if rank != 0:
        return
    steps, coords, seconds = 0, 0, 0.0
    from oracle.cpu_step import CpuStep, plane_levels_for_cpu
    from odie_b200 import layout as host_layout
    config, supports, dims, caps, rgb, shape = workload(args.workload, 0, 1, args.batch)
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    lay = host_layout.make_layout(config, supports, dims, caps)
    levels = plane_levels_for_cpu(lay['descriptors'].numpy(), lay['node_bitmap'].numpy(), lay['node_prefix'].numpy(),
                                  lay['bitmap'].numpy())
    rng = np.random.default_rng(0)
    width = (lay['input_width'] + 15) // 16 * 16
    step = CpuStep(shape, rgb.numpy(), levels, (rng.standard_normal(lay['params']) * 1e-3).astype(np.float32),
                   (rng.standard_normal(width * 32 + 512) * .1).astype(np.float32),
                   (rng.standard_normal(width * 64 + 64 * 64 + 1024) * .1).astype(np.float32), width)
    sample = 1 << 14
    g = torch.Generator().manual_seed(2)
    pixels = shape[0] * shape[1]
    for _ in range(args.warmup):
        step.step(torch.randint(0, pixels, (sample,), generator=g))
    started = time.perf_counter()
    for _ in range(args.steps):
        step.step(torch.randint(0, pixels, (sample,), generator=g))
        steps += 1
        coords += sample
    seconds = time.perf_counter() - started
    value = coords / seconds
    line = {'metric': METRIC, 'value': value, 'unit': UNIT, 'n_gpus': args.gpus, 'steps': args.steps,
            'warmup': args.warmup, 'ms_per_step': seconds / steps * 1e3, 'higher_is_better': True, 'scaling': 'weak',
            'vs_baseline': None, 'dtype': 'f32/f16', 'data': 'synthetic', 'impl': 'reference',
            'config': {'workload': args.workload, 'batch_per_step': sample, 'full_batch': args.batch,
                       'note': 'bounded sample of the workload per step'},
            'cpu_baseline': {'value': value, 'unit': UNIT, 'cores': threads, 'kind': 'port',
                             'sample': f'{steps} steps x {sample} coords, torch CPU restatement, {threads} threads'},
            'e2e': {'value': value, 'unit': UNIT, 'h2d_bytes_per_step': 0, 'd2h_bytes_per_step': 0}}
    print(json.dumps(line), flush=True)


def main():
    args = parse()
    if args.impl == 'reference':
        run_reference(args)
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
    from odie_b200 import _lib
    from odie_b200 import workloads
    from odie_b200.native_backend import NativeOptimizer
    lib = _lib.library()
    config, supports, dims, caps, rgb, shape = workload(args.workload, rank, world, args.batch)
    model, target, planes = workloads.build_plane_model(config, supports, dims, caps, rgb)
    head_grad = None
    if world > 1:
        width = (model.input_width + 15) // 16 * 16
        head_grad = torch.zeros(width * 32 + 512 + width * 64 + 64 * 64 + 1024, device='cuda')
    opt = NativeOptimizer(model, target, shape, config, planes, batch=args.batch, head_grad=head_grad)
    pixels = shape[0] * shape[1]
    gen = torch.Generator(device='cuda').manual_seed(1729 + rank)
    total_steps = args.warmup + args.steps
    ids = torch.randint(0, pixels, (total_steps, args.batch), device='cuda', generator=gen)

    def step(batch_ids):
        if world == 1:
            opt.check(lib.odie_step(opt.handle, batch_ids.data_ptr(), batch_ids.numel(), 1))
        else:
            opt.check(lib.odie_step_grads(opt.handle, batch_ids.data_ptr(), batch_ids.numel(), 1))
            dist.all_reduce(head_grad)
            opt.check(lib.odie_step_heads(opt.handle))

    def barrier():
        torch.cuda.synchronize()
        if dist is not None:
            dist.barrier()
        torch.cuda.synchronize()

    for w in range(args.warmup):
        step(ids[w])
    barrier()
    opt.check(lib.odie_profile(opt.handle, 1))
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with Clocks(local) as clocks:
        barrier()
        start.record()
        for k in range(args.steps):
            step(ids[args.warmup + k])
        end.record()
        barrier()
    ms = start.elapsed_time(end)
    report = json.loads(lib.odie_profile_report(opt.handle))
    opt.check(lib.odie_profile(opt.handle, 0))
    ms_t = torch.tensor([ms], device='cuda')
    if dist is not None:
        dist.all_reduce(ms_t, op=dist.ReduceOp.MAX)
    ms = float(ms_t)
    value = world * args.batch * args.steps / (ms / 1e3)

    # end to end through the public API: pinned host ids in, loss out, every step
    host_ids = ids[args.warmup:].cpu().pin_memory()
    device_ids = torch.empty(args.batch, dtype=torch.int64, device='cuda')
    loss_host = torch.empty(args.steps, dtype=torch.float64).pin_memory()
    squares = torch.empty(args.batch, device='cuda')
    barrier()
    e_start, e_end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e_start.record()
    for k in range(args.steps):
        device_ids.copy_(host_ids[k], non_blocking=True)
        step(device_ids)
        opt.check(lib.odie_copy(squares.data_ptr(), opt.pointers['squares'], args.batch * 4,
                                torch.cuda.current_stream().cuda_stream))
        loss_host[k:k + 1].copy_(squares.double().mean().reshape(1), non_blocking=True)
    e_end.record()
    barrier()
    e_ms = torch.tensor([e_start.elapsed_time(e_end)], device='cuda')
    if dist is not None:
        dist.all_reduce(e_ms, op=dist.ReduceOp.MAX)
    e2e = world * args.batch * args.steps / (float(e_ms) / 1e3)
    losses = loss_host.numpy()

    # decode of this rank's band (all pixels), Gpix/s
    rgb8 = torch.empty((pixels, 3), dtype=torch.uint8, device='cuda')
    opt.decode(0, pixels, rgb8=rgb8)
    barrier()
    d_start, d_end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    repeats = 5
    d_start.record()
    for _ in range(repeats):
        opt.decode(0, pixels, rgb8=rgb8)
    d_end.record()
    barrier()
    d_ms = torch.tensor([d_start.elapsed_time(d_end)], device='cuda')
    if dist is not None:
        dist.all_reduce(d_ms, op=dist.ReduceOp.MAX)
    decode_gpix = world * pixels * repeats / (float(d_ms) / 1e3) / 1e9

    if rank == 0:
        hbm, tensor_peak, peak_kind = peaks()
        stages = {k: v for k, v in report.items() if v['launches']}
        dominant = max(stages, key=lambda k: stages[k]['ms'])
        total_ms = sum(v['ms'] for v in stages.values())
        width = (model.input_width + 15) // 16 * 16
        head_flops = 6 * (width * 32 + 32 * 16 + width * 64 + 64 * 64 + 64 * 16)
        bound, work = algorithmic(dominant, model.n_levels, 2, args.batch, model.grid.numel(), head_flops)
        per_launch_s = stages[dominant]['ms'] / stages[dominant]['launches'] / 1e3
        if bound == 'tensor':
            achieved, peak, unit = work / per_launch_s / 1e12, tensor_peak, 'TFLOP/s'
        else:
            achieved, peak, unit = (work / per_launch_s / 1e9 if work else None), hbm, 'GB/s'
        roofline = {'kernel': dominant, 'bound': bound, 'achieved': achieved, 'peak': peak, 'unit': unit,
                    'frac': (achieved / peak) if achieved else None, 'traffic': None, 'peak_source': peak_kind,
                    'share': stages[dominant]['ms'] / total_ms,
                    'stages_ms_per_step': {k: v['ms'] / args.steps for k, v in stages.items()}}
        base = None
        if world == 1 and not args.no_cpu_baseline:
            base = cpu_baseline(args)
        line = {'metric': METRIC, 'value': value, 'unit': UNIT, 'n_gpus': world, 'steps': args.steps,
                'warmup': args.warmup, 'ms_per_step': ms / args.steps, 'higher_is_better': True, 'scaling': 'weak',
                'vs_baseline': None, 'dtype': 'f16 (fp32 masters, fp32 accumulate)', 'data': 'synthetic',
                'config': {'workload': args.workload, 'image_hw': list(shape), 'global_batch': world * args.batch,
                           'batch_per_gpu': args.batch, 'levels': model.n_levels, 'grid_params': model.grid.numel(),
                           'parallelism': f'dp{world} (row bands, head all-reduce)',
                           'l2': 'per-step inputs/activations (~200 MB) larger than L2; model tables L2-resident'},
                'e2e': {'value': e2e, 'unit': UNIT, 'h2d_bytes_per_step': args.batch * 8, 'd2h_bytes_per_step': 8},
                'gpu_launches': 8 * args.steps, 'roofline': roofline, 'cpu_baseline': base,
                'decode': {'value': decode_gpix, 'unit': 'Gpix/s', 'pixels_per_rank': pixels},
                'loss_first_last': [float(losses[0]), float(losses[-1])], 'clocks': clocks.summary()}
        print(json.dumps(line), flush=True)
    opt.close()
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == '__main__':
    main()
