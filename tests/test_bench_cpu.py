"""CPU: the benchmark's reference arm (the reference's own source compiled for
the CPU) prints one JSON line with the keys the benchmark contract names, and
ranks other than 0 exit quietly."""
import json
import os
import subprocess
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
REF = ROOT / 'oracle' / '_ref'


def _run(args, env_extra=None):
    env = dict(os.environ, **(env_extra or {}))
    out = subprocess.run([sys.executable, str(ROOT / 'bench.py'), *args], cwd=ROOT, env=env, capture_output=True,
                         text=True, timeout=300)
    assert out.returncode == 0, out.stderr[-2000:]
    return [line for line in out.stdout.splitlines() if line.startswith('{')]


@pytest.mark.parametrize('config,library', [('decode1', 'routed_storage_n32'), ('dense_qkvz1', 'dense_n32'),
                                            ('head_vocab1', 'head_i8')])
def test_reference_arm_line(config, library):
    if not (REF / f'libref_{library}.so').exists():
        pytest.skip(f'oracle/_ref/libref_{library}.so not built')
    lines = _run(['--impl', 'reference', '--config', config, '--steps', '1', '--warmup', '0'])
    assert len(lines) == 1
    line = json.loads(lines[0])
    for key in ('impl', 'metric', 'value', 'unit', 'n_gpus', 'steps', 'warmup', 'ms_per_step', 'higher_is_better',
                'config', 'cpu_baseline', 'e2e'):
        assert key in line, key
    assert line['impl'] == 'reference' and line['value'] > 0
    assert line['cpu_baseline']['kind'] == 'reference' and line['cpu_baseline']['cores'] >= 1
    assert line['e2e']['value'] == line['value']
    assert line['e2e']['h2d_bytes_per_step'] == line['e2e']['d2h_bytes_per_step'] == 0


def test_reference_arm_other_ranks_print_nothing():
    assert _run(['--impl', 'reference', '--steps', '1', '--warmup', '0'], {'RANK': '1', 'WORLD_SIZE': '2'}) == []


def test_default_workload_follows_the_launcher():
    """A plain process measures decode B=1; under
    torch.distributed.run, at any world size, the expert-parallel prefill
    (configs[4]) is the default, so a scaling run compares one workload."""
    if not (REF / 'libref_routed_storage_n32.so').exists():
        pytest.skip('oracle/_ref/libref_routed_storage_n32.so not built')
    sys.path.insert(0, str(ROOT))
    import bench
    plain = json.loads(_run(['--impl', 'reference', '--steps', '1', '--warmup', '0'])[0])
    assert plain['config']['workload'] == bench.CONFIGS['decode1']['name']
    launched = json.loads(_run(['--impl', 'reference', '--steps', '1', '--warmup', '0'],
                               {'TORCHELASTIC_RUN_ID': 'test', 'LOCAL_WORLD_SIZE': '1', 'RANK': '0',
                                'WORLD_SIZE': '1'})[0])
    assert launched['config']['workload'] == bench.CONFIGS['ep_prefill8192']['name']
