"""Shared fixtures.  GPU tests carry @pytest.mark.gpu; everything else runs on CPU."""
import importlib
import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parents[1]
sys.path.insert(0, str(ROOT))
import __graft_entry__ as graft  # noqa: E402

graft.load_package()
GOLDEN = ROOT / 'tests' / 'golden'


def pytest_configure(config):
    config.addinivalue_line('markers', 'gpu: needs a CUDA device (B200)')


# GPU files in run order: the routed parity suite first, then the other
# single-GPU files that have passed on a B200, then files not yet run on one,
# the expert-parallel ones (two GPUs) and the allocation-free entry last, so
# that a run stopped at its first failure has always checked what came before.
GPU_ORDER = ['test_parity_gpu.py', 'test_dense_gpu.py', 'test_head_gpu.py', 'test_shared_dense_gpu.py',
             'test_weights_gpu.py', 'test_debug_bounds_gpu.py', 'test_ep_plan_gpu.py', 'test_ep_gpu.py',
             'test_zz_no_alloc.py']


def pytest_collection_modifyitems(config, items):
    def rank(item):
        name = item.path.name
        if name in GPU_ORDER:
            return GPU_ORDER.index(name)
        # an unlisted GPU file runs just before the allocation-free entry; CPU files keep their place
        return len(GPU_ORDER) - 1.5 if name.endswith('_gpu.py') else -1
    items.sort(key=rank)   # stable: file order otherwise


@pytest.fixture(scope='session')
def S():
    return importlib.import_module('ornith_b200.synthetic')


@pytest.fixture(scope='session')
def O():
    from oracle import oracle
    return oracle


@pytest.fixture(scope='session')
def native():
    return importlib.import_module('ornith_b200.native')


@pytest.fixture(scope='session')
def golden():
    return np.load(GOLDEN / 'routed_reference_outputs.npz')


@pytest.fixture(scope='session')
def dense_golden():
    return np.load(GOLDEN / 'dense_reference_outputs.npz')


@pytest.fixture(scope='session')
def head_golden():
    return np.load(GOLDEN / 'head_reference_outputs.npz')


@pytest.fixture(scope='session')
def tables():
    return np.load(GOLDEN / 'shared_math_tables.npz')


@pytest.fixture(scope='session')
def make_golden():
    spec = importlib.util.spec_from_file_location('make_golden', GOLDEN / 'make_golden.py')
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


@pytest.fixture(scope='session')
def layer1(S):
    """The layer every golden case uses (seed 1)."""
    return S.make_layer(np.random.default_rng(1))
