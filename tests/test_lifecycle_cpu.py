"""CPU: the worker lifecycle's failure detection (per-step flag checks and
poisoning), with a fake binding and a fake flag transport, so every failure
is made on the host: a flag value the fake reports, or an error the fake
raises."""
import importlib

import pytest


@pytest.fixture(scope='module')
def L():
    return importlib.import_module('ornith_b200.lifecycle')


class FakeBinding:
    def __init__(self, n=3):
        self.layer_prefixes = tuple(f'layer{i}' for i in range(n))
        self.current = [0] * n
        self.reset_error = None
        self.resets = 0

    def reset_error_flags(self):
        if self.reset_error:
            raise self.reset_error
        self.current = [0] * len(self.layer_prefixes)
        self.resets += 1


class FakeTransport:
    """Copies the binding's current flags at queue() time, as the device copy
    enqueued behind a step's work would."""

    def __init__(self, binding):
        self.binding = binding
        self.queue_error = self.finish_error = None
        self.width = None

    def allocate_slot(self):
        from ornith_b200.lifecycle import FlagSlot
        return FlagSlot(host=None)

    def queue(self, slot):
        if self.queue_error:
            raise self.queue_error
        slot.host = list(self.binding.current)

    def finish(self, slot):
        if self.finish_error:
            raise self.finish_error
        return slot.host if self.width is None else slot.host[:self.width]


def _make(L, inflight=2, n=3):
    b = FakeBinding(n)
    t = FakeTransport(b)
    return L.WorkerStepLifecycle(b, inflight, _transport=t), b, t


def test_clean_steps_cycle_the_slots(L):
    lc, b, _ = _make(L)
    for i in range(5):
        tk = lc.begin(f'step{i}')
        lc.queue(tk)
        assert lc.complete(tk) == (0, 0, 0)
    assert (lc.resets, lc.copies, lc.completions, b.resets) == (5, 5, 5, 5)


def test_flag_poisons_the_worker(L):
    lc, b, _ = _make(L)
    tk = lc.begin('decode')
    b.current[1] = 4                    # invalid expert id in layer1
    lc.queue(tk)
    with pytest.raises(L.OrnithWorkerFault, match='layer1'):
        lc.complete(tk)
    with pytest.raises(L.OrnithWorkerFault):
        lc.begin('next')                # poisoned: no more steps


def test_later_clean_step_cannot_hide_an_earlier_fault(L):
    lc, b, _ = _make(L)
    t1 = lc.begin('a')
    b.current[0] = 8
    lc.queue(t1)
    t2 = lc.begin('b')                  # resets the flags: its own copy is clean
    lc.queue(t2)
    with pytest.raises(L.OrnithWorkerFault, match="step 0 \\(a\\)"):
        lc.complete(t2)
    assert t1.completed and t1.flags == (8, 0, 0)


def test_slot_pool_is_bounded(L):
    lc, _, _ = _make(L, inflight=2)
    a, _b = lc.begin('a'), lc.begin('b')
    with pytest.raises(RuntimeError, match='flag slots'):
        lc.begin('c')
    lc.queue(a)
    lc.complete(a)
    lc.begin('c')                       # a slot came back
    with pytest.raises(ValueError):
        L.WorkerStepLifecycle(FakeBinding(), 0, _transport=FakeTransport(FakeBinding()))
    with pytest.raises(ValueError):
        L.WorkerStepLifecycle(FakeBinding(), True, _transport=FakeTransport(FakeBinding()))


@pytest.mark.parametrize('where', ['reset', 'queue', 'finish', 'width'])
def test_boundary_failures_poison(L, where):
    lc, b, t = _make(L)
    boom = RuntimeError(f'{where} failed')
    if where == 'reset':
        b.reset_error = boom
        with pytest.raises(RuntimeError, match='reset failed'):
            lc.begin('x')
    else:
        tk = lc.begin('x')
        if where == 'queue':
            t.queue_error = boom
            with pytest.raises(RuntimeError, match='queue failed'):
                lc.queue(tk)
        else:
            lc.queue(tk)
            if where == 'finish':
                t.finish_error = boom
            else:
                t.width = 2
            with pytest.raises(RuntimeError):
                lc.complete(tk)
    with pytest.raises(L.OrnithWorkerFault):
        lc.begin('y')


def test_complete_requires_the_copy(L):
    lc, _, _ = _make(L)
    tk = lc.begin('x')
    with pytest.raises(RuntimeError, match='never queued'):
        lc.complete(tk)


def test_abort_keeps_the_cause(L):
    lc, b, _ = _make(L)
    tk = lc.begin('x')
    with pytest.raises(ValueError, match='model error'):
        lc.abort(tk, ValueError('model error'))          # clean flags: the error itself
    with pytest.raises(L.OrnithWorkerFault):
        lc.begin('y')
    lc, b, _ = _make(L)
    tk = lc.begin('x')
    b.current[2] = 16
    with pytest.raises(L.OrnithWorkerFault) as info:
        lc.abort(tk, ValueError('model error'))          # flags set: the fault, caused by the error
    assert isinstance(info.value.__cause__, ValueError)


def test_checked_async_output(L):
    class Async:
        def __init__(self, value, error=None):
            self.value, self.error = value, error

        def get_output(self):
            if self.error:
                raise self.error
            return self.value

    lc, b, _ = _make(L)
    tk = lc.begin('x')
    lc.queue(tk)
    out = lc.checked_output(Async(42), tk)
    assert out.get_output() == 42
    with pytest.raises(RuntimeError, match='already taken'):
        out.get_output()
    tk = lc.begin('y')
    b.current[0] = 1                    # raised by y's work, before y's copy
    lc.queue(tk)
    tk2 = lc.begin('z')                 # not needed for the check of y
    lc.queue(tk2)
    with pytest.raises(L.OrnithWorkerFault):
        lc.checked_output(Async(1), tk).get_output()
    lc, _, _ = _make(L)
    tk = lc.begin('w')
    lc.queue(tk)
    with pytest.raises(KeyError):
        lc.checked_output(Async(0, KeyError('copy failed')), tk).get_output()
    with pytest.raises(L.OrnithWorkerFault):
        lc.begin('v')


def test_plain_output_and_drain(L):
    lc, b, _ = _make(L, inflight=3)
    tk = lc.begin('x')
    lc.queue(tk)
    assert lc.checked_output('tokens', tk) == 'tokens'
    lc.begin('a')
    lc.begin('b')                       # drain queues and checks both
    lc.drain()
    assert lc.completions == 3
    lc.begin('c')
    b.current[0] = 32
    with pytest.raises(L.OrnithWorkerFault):
        lc.drain()


def test_cuda_transport_needs_a_cuda_runtime(L):
    class CpuRuntime:
        device = __import__('torch').device('cpu')
        layer_prefixes = ('a',)
    with pytest.raises(ValueError, match='CUDA'):
        L.CudaFlagTransport(CpuRuntime())
