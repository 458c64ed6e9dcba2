"""CPU: the benchmark's reference arm (the reference's own source compiled for
the CPU) prints one JSON line with the keys the benchmark contract names, and
ranks other than 0 exit quietly; the benchmark's and the package's GPU-only
code reads no unbound name."""
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


def _unbound_names(path):
    """Names read inside the functions of a module that no scope binds: not a
    parameter or local of the function or of an enclosing one, not a module
    global, not a builtin.  The GPU-only legs of the benchmark (the
    expert-parallel and layer measurements) never run on the CPU, so a
    misspelt or misplaced name there would surface only on a GPU box."""
    import builtins
    import symtable
    top = symtable.symtable(Path(path).read_text(), str(path), 'exec')
    module_names = set(top.get_identifiers())
    missing = []

    def walk(table, enclosing):
        bound = set(enclosing)
        if table.get_type() == 'function':
            bound |= {s.get_name() for s in table.get_symbols() if s.is_assigned() or s.is_parameter()
                      or s.is_imported() or s.is_local()}
            for s in table.get_symbols():
                name = s.get_name()
                if s.is_referenced() and not (name in bound or name in module_names or hasattr(builtins, name)):
                    missing.append(f'{table.get_name()}:{table.get_lineno()}: {name}')
        for child in table.get_children():
            walk(child, bound if table.get_type() == 'function' else set())

    walk(top, set())
    return missing


@pytest.mark.parametrize('path', ['bench.py', '__graft_entry__.py', 'ornith-ciru-halo-agent_b200/ep.py',
                                  'ornith-ciru-halo-agent_b200/native.py', 'ornith-ciru-halo-agent_b200/method.py'])
def test_functions_read_only_bound_names(path):
    assert _unbound_names(ROOT / path) == []
