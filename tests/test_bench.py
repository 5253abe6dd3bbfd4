"""bench.py's one-line JSON contract: the reference arm (CPU) and this library's arm (GPU), small runs."""
import json
import subprocess
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]


def run_bench(*args, timeout=600):
    out = subprocess.run([sys.executable, str(ROOT / 'bench.py'), *args], cwd=ROOT, capture_output=True, text=True,
                         timeout=timeout)
    assert out.returncode == 0, out.stderr[-2000:]
    lines = [line for line in out.stdout.splitlines() if line.startswith('{')]
    assert len(lines) == 1, out.stdout[-2000:]
    return json.loads(lines[0])


BASE_KEYS = {'metric', 'value', 'unit', 'n_gpus', 'steps', 'warmup', 'ms_per_step', 'higher_is_better', 'scaling',
             'vs_baseline', 'dtype', 'data', 'config', 'e2e', 'cpu_baseline'}


def test_reference_arm_line():
    line = run_bench('--impl', 'reference', '--steps', '1', '--warmup', '1')
    assert BASE_KEYS <= set(line)
    assert line['impl'] == 'reference' and line['unit'] == 'coords/s' and line['value'] > 0
    assert line['higher_is_better'] is True and line['config']['workload'] == 'c4-experts'
    assert line['e2e'] == {'value': line['value'], 'unit': line['unit'], 'h2d_bytes_per_step': 0,
                           'd2h_bytes_per_step': 0}
    base = line['cpu_baseline']
    assert base['kind'] in ('port', 'reference') and base['cores'] >= 1 and base['value'] == line['value']


@pytest.mark.gpu
@pytest.mark.parametrize('workload', ['c4-experts', 'c2-experts', 'c2-planes', 'c3-experts'])
def test_our_arm_line(cuda, workload):
    batch = 1 << 16
    line = run_bench('--workload', workload, '--steps', '3', '--warmup', '3', '--batch', str(batch),
                     '--no-cpu-baseline')
    assert BASE_KEYS - {'cpu_baseline'} <= set(line)
    assert line['n_gpus'] == 1 and line['steps'] == 3 and line['warmup'] == 3
    assert line['value'] > 0 and line['ms_per_step'] > 0 and line['config']['workload'] == workload
    assert line['config']['batch_per_gpu'] == batch
    e2e = line['e2e']
    assert e2e['value'] > 0 and e2e['h2d_bytes_per_step'] == batch * 8 and e2e['d2h_bytes_per_step'] == 8
    roof = line['roofline']
    assert {'bound', 'achieved', 'peak', 'unit', 'frac', 'traffic'} <= set(roof)
    assert roof['bound'] in ('hbm', 'tensor') and roof['peak'] > 0
    assert line['gpu_launches'] > 0, 'the library counted none of its own launches'
    clocks = line['clocks']
    assert {'sm_mhz', 'sm_max_mhz', 'reasons'} <= set(clocks)
    assert line['decode']['value'] > 0
    first, last = line['loss_first_last']
    assert last == last and first == first, 'loss is NaN'
    if workload in ('c3-experts', 'c4-experts'):
        allocation = line['allocation']
        fraction = 0.3 if workload == 'c3-experts' else 0.2
        assert allocation['tiles_allocated'] == round(fraction * allocation['tiles_total'])
    if workload == 'c4-experts':
        config = line['config']
        assert config['experts'] == 64 and config['bands'] == 8 and config['image_hw'] == [32768, 32768]
        assert config['fp16_payload_mib'] <= 50
        assert line['decode']['launch_pixels'] == 1 << 24 and line['decode']['launches_per_pass'] == 64
