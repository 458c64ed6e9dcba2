"""GPU: the bounded waits on other ranks give up, raise flag 64 and return.

One GPU, no peer memory: the flag arrays a wait reads are local device
buffers that nothing raises (or that a test raises before the wait), so no
kernel ever waits on another kernel that runs at the same time.  The wait
limit is the library's setting, cut to a few milliseconds here and restored
afterwards."""
import time

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu
DEV = torch.device('cuda:0')
FLAG_TIMEOUT = 64
LIMIT_NS = 5_000_000   # 5 ms


@pytest.fixture
def short_wait(native):
    native.set_peer_wait_limit_ns(LIMIT_NS)
    yield
    native.set_peer_wait_limit_ns(1_000_000_000)


def timed(fn):
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    fn()
    torch.cuda.synchronize()
    return time.perf_counter() - t0


@pytest.mark.parametrize('world,me', [(2, 0), (8, 3)])
def test_wait_signals_runs_out(native, short_wait, world, me):
    """No rank ever raises its epoch: the wait ends after about the limit
    with flag 64, and the context stays usable."""
    sig = torch.zeros(2 * world, dtype=torch.int32, device=DEV)
    flags = torch.zeros(1, dtype=torch.int32, device=DEV)
    dt = timed(lambda: native.ep_wait_signals(sig.data_ptr(), world, me, 1, flags))
    assert int(flags.item()) == FLAG_TIMEOUT
    assert dt < 0.5, f'the wait took {dt:.3f} s against a limit of {LIMIT_NS / 1e9} s'
    assert torch.ones(4, device=DEV).sum().item() == 4.0   # the context still works


def test_wait_epoch_runs_out(native, short_wait):
    """The device-counter form (fixed exchange): epoch 5 in device memory,
    rank 0 has raised it, rank 2 has not: flag 64."""
    world, me = 4, 1
    sig = torch.zeros(2 * world, dtype=torch.int32, device=DEV)
    sig[0] = 5
    sig[3] = 5
    epoch = torch.full((1,), 5, dtype=torch.int32, device=DEV)
    flags = torch.zeros(1, dtype=torch.int32, device=DEV)
    dt = timed(lambda: native.ep_wait_epoch(sig.data_ptr(), world, me, epoch, flags))
    assert int(flags.item()) == FLAG_TIMEOUT and dt < 0.5


def test_wait_returns_when_raised_and_takes_the_senders_timeout_bit(native, short_wait):
    """Every epoch raised: the wait returns at once; its flags pick up a
    sender's status bit (that sender's own wait ran out) and nothing else."""
    world, me = 3, 2
    sig = torch.zeros(2 * world, dtype=torch.int32, device=DEV)
    sig[0:2] = 7
    flags = torch.zeros(1, dtype=torch.int32, device=DEV)
    native.ep_wait_signals(sig.data_ptr(), world, me, 7, flags)
    torch.cuda.synchronize()
    assert int(flags.item()) == 0
    sig[world + 1] = FLAG_TIMEOUT | 1          # rank 1's status word; only bit 64 travels
    native.ep_wait_signals(sig.data_ptr(), world, me, 7, flags)
    torch.cuda.synchronize()
    assert int(flags.item()) == FLAG_TIMEOUT


def test_sender_publishes_its_timeout_bit(native, short_wait):
    """The fixed dispatch stores its rank's timeout bit beside the epoch in
    the other ranks' arrays.  Rank 0 of two, with rank 1's buffers standing in
    as local memory; rank 0's flags carry 64 from an earlier wait that ran
    out.  Rank 1's wait (run after the dispatch, on the same stream) then
    reports 64 too."""
    import ctypes as C
    world, T = 2, 4
    x = torch.randn((T, 2048), device=DEV).to(torch.bfloat16)
    lids = torch.full((world, T, 8), -1, dtype=torch.int32, device=DEV)
    tok = [torch.zeros((world * T, 2048), dtype=torch.bfloat16, device=DEV) for _ in range(2 * world)]
    ids = [torch.zeros((world * T, 8), dtype=torch.int32, device=DEV) for _ in range(2 * world)]
    sig = [torch.zeros(2 * world, dtype=torch.int32, device=DEV) for _ in range(world)]
    dst_x = (C.c_void_p * (2 * world))(*[t.data_ptr() for t in tok])
    dst_ids = (C.c_void_p * (2 * world))(*[t.data_ptr() for t in ids])
    signals = (C.c_void_p * world)(*[s.data_ptr() for s in sig])
    epoch0 = torch.zeros(1, dtype=torch.int32, device=DEV)
    counter = torch.zeros(1, dtype=torch.int32, device=DEV)
    flags0 = torch.full((1,), FLAG_TIMEOUT, dtype=torch.int32, device=DEV)
    native.ep_fixed_dispatch(x, lids, dst_x, dst_ids, world * T, signals, world, 0, epoch0, counter, flags0)
    torch.cuda.synchronize()
    assert sig[1].cpu().numpy().tolist() == [1, 0, FLAG_TIMEOUT, 0]   # epoch 1 and status 64 from rank 0
    assert int(epoch0.item()) == 1
    # call 1 uses set 1: rank 1's token buffer of that set holds rank 0's rows first
    np.testing.assert_array_equal(tok[1 * world + 1][:T].view(torch.int16).cpu().numpy(),
                                  x.view(torch.int16).cpu().numpy())
    epoch1 = torch.ones(1, dtype=torch.int32, device=DEV)
    flags1 = torch.zeros(1, dtype=torch.int32, device=DEV)
    dt = timed(lambda: native.ep_wait_epoch(sig[1].data_ptr(), world, 1, epoch1, flags1))
    assert int(flags1.item()) == FLAG_TIMEOUT and dt < 0.5
