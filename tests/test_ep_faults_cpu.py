"""CPU: expert parallelism when a peer fails (gloo ranks, world size 2).

A rank that dies or raises between steps must not leave the other ranks
waiting forever: with a short process-group timeout their next collective
ends with an error, which the layer passes to its caller.  The failures are
made on the host (a rank that exits without joining the exchange, a rank whose
expert compute raises), never on a GPU."""
import datetime
import os
import socket
import sys
import time
from pathlib import Path

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

ROOT = Path(__file__).resolve().parents[1]
sys.path.insert(0, str(Path(__file__).resolve().parent))
from test_ep_cpu import fake_combine_gathered, fake_rows, _inputs  # noqa: E402

TIMEOUT_S = 5


def _port():
    with socket.socket() as s:
        s.bind(('127.0.0.1', 0))
        return s.getsockname()[1]


def _report(q, item, code):
    """Send a result and end the process without teardown collectives (a
    failed peer could not take part in them); the queue is flushed first,
    since os._exit does not wait for its feeder thread."""
    q.put(item)
    q.close()
    q.join_thread()
    os._exit(code)


def _worker(rank, world, port, q, failure):
    try:
        os.environ['MASTER_ADDR'] = '127.0.0.1'
        os.environ['MASTER_PORT'] = str(port)
        dist.init_process_group('gloo', rank=rank, world_size=world,
                                timeout=datetime.timedelta(seconds=TIMEOUT_S))
        sys.path.insert(0, str(ROOT))
        import __graft_entry__ as g
        g.load_package()
        from ornith_b200 import ep
        placement = ep.contiguous_placement(world)
        table = torch.tensor(placement.experts_of(rank))
        x, ids, weights = _inputs(rank, 12, 99)

        def compute(xr, ir, n_valid):
            if failure == 'raise' and rank == 1:
                raise RuntimeError('expert compute failed on rank 1')
            return fake_rows(xr, ir, table)[ir >= 0] if xr.shape[0] else torch.zeros((0, 2048))

        # one healthy step first
        ep.ep_layer(None, world, x, ids, weights, compute if failure != 'raise' else
                    (lambda xr, ir, n: fake_rows(xr, ir, table)[ir >= 0]), fake_combine_gathered, placement)
        if failure == 'exit' and rank == 1:
            _report(q, (rank, 'exited', 0.0), 0)   # dies between steps, with nothing in flight
        t0 = time.monotonic()
        try:
            ep.ep_layer(None, world, x, ids, weights, compute, fake_combine_gathered, placement)
            outcome = 'completed'
        except Exception as exc:            # noqa: BLE001 - the test inspects what surfaced
            outcome = f'error: {type(exc).__name__}'
        _report(q, (rank, outcome, time.monotonic() - t0), 0)
    except Exception as exc:                # noqa: BLE001
        _report(q, (rank, f'setup error: {exc!r}', 0.0), 1)


@pytest.mark.parametrize('failure', ['exit', 'raise'])
def test_a_failed_peer_ends_the_others_step_with_an_error(failure):
    ctx = mp.get_context('spawn')
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q, failure)) for r in range(2)]
    for p in procs:
        p.start()
    results = {}
    for _ in range(2):
        rank, what, seconds = q.get(timeout=120)
        results[rank] = (what, seconds)
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    what, seconds = results[0]
    # the surviving rank got an error, not a hang, and within a bounded time
    assert what.startswith('error'), results
    assert seconds < 6 * TIMEOUT_S, results
    if failure == 'raise':
        assert results[1][0].startswith('error'), results
