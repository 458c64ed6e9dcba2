"""Per-step error-flag checks and worker poisoning (failure detection).

The interface of the reference plugin's worker lifecycle
(plugin-site/ornith_g256/lifecycle.py: WorkerStepLifecycle with begin / queue /
complete / abort / checked_output / drain, OrnithWorkerFault, a flag
transport), without vLLM:

  * begin(name) resets the runtime's sticky per-layer flags (never inside a
    graph capture) and opens a step;
  * queue(ticket) enqueues one asynchronous copy of the flags to pinned host
    memory behind the step's work;
  * complete(ticket) checks that step and every older open step, oldest
    first, so a clean later step cannot hide a fault of an earlier one;
  * the first non-zero flag, and any failure of a reset, copy or check,
    poisons the worker: every later call raises OrnithWorkerFault, since a
    native error leaves outputs unusable and the process has to be replaced
    (lifecycle.py:17-19,110-116).

The copies go through a transport object; CudaFlagTransport does them on a
GPU, and tests pass a fake one, so the whole state machine is exercised on
CPU without any GPU fault.
"""
import threading
from collections import deque
from contextlib import contextmanager
from dataclasses import dataclass

import torch


class OrnithWorkerFault(RuntimeError):
    """The worker hit a native error and must not deliver further outputs."""


def _refuse_during_capture(device):
    if device.type == 'cuda':
        with torch.cuda.device(device):
            if torch.cuda.is_current_stream_capturing():
                raise RuntimeError('Error flags are not reset or read while a CUDA graph is being captured')


@dataclass(eq=False)
class FlagSlot:
    """Host landing place of one step's flags and the event that marks it filled."""
    host: object
    event: object = None


@dataclass(eq=False)
class StepTicket:
    sequence: int
    name: str
    slot: FlagSlot
    queued: bool = False
    completed: bool = False
    flags: tuple = None


class CudaFlagTransport:
    """Flag copies of a Runtime on a CUDA device: one pinned int32 vector and
    one event per in-flight step, allocated once."""

    def __init__(self, binding):
        self.binding = binding
        self.device = binding.device
        if self.device.type != 'cuda':
            raise ValueError('CudaFlagTransport needs a runtime on a CUDA device')
        self.fallback_synchronizations = 0   # checks that had to wait for their copy

    def allocate_slot(self):
        _refuse_during_capture(self.device)
        host = torch.empty(len(self.binding.layer_prefixes), dtype=torch.int32, pin_memory=True)
        return FlagSlot(host, torch.cuda.Event(blocking=True))

    def queue(self, slot):
        _refuse_during_capture(self.device)
        with torch.cuda.device(self.device):
            stream = torch.cuda.current_stream(self.device)
            slot.host.copy_(self.binding.error_flags, non_blocking=True)
            slot.event.record(stream)

    def finish(self, slot):
        _refuse_during_capture(self.device)
        with torch.cuda.device(self.device):
            if not slot.event.query():
                # the step's own output copy usually waited past this already
                self.fallback_synchronizations += 1
                slot.event.synchronize()
        return tuple(slot.host.tolist())


class WorkerStepLifecycle:
    """Bounded per-step flag checks for one worker.  `binding` is a Runtime
    (error_flags, layer_prefixes, reset_error_flags); at most `max_inflight`
    steps (1..64) may be open, i.e. begun and not yet checked."""

    def __init__(self, binding, max_inflight, *, _transport=None):
        if isinstance(max_inflight, bool) or not isinstance(max_inflight, int) or not 1 <= max_inflight <= 64:
            raise ValueError('max_inflight must be an int in 1..64')
        self.binding = binding
        self.transport = CudaFlagTransport(binding) if _transport is None else _transport
        self._spare = [self.transport.allocate_slot() for _ in range(max_inflight)]
        self._open = deque()          # begun, unchecked steps, oldest first
        self._next_sequence = 0
        self._fault = None
        self._lock = threading.RLock()
        self.resets = self.copies = self.completions = 0

    # -- failure handling -------------------------------------------------------
    def raise_if_failed(self):
        if self._fault is not None:
            raise self._fault

    def poison(self, error):
        """Record the first failure; every later call raises it."""
        with self._lock:
            if self._fault is None:
                fault = OrnithWorkerFault(f'worker poisoned by {type(error).__name__}: {error}')
                fault.__cause__ = error
                self._fault = fault

    @contextmanager
    def _poison_on_error(self):
        try:
            yield
        except BaseException as error:
            self.poison(error)
            raise

    # -- step protocol ----------------------------------------------------------
    def begin(self, name):
        """Open a step: reset the sticky flags and reserve a flag slot."""
        with self._lock:
            self.raise_if_failed()
            if not self._spare:
                raise RuntimeError(f'all {len(self._open)} flag slots are held by unchecked steps')
            slot = self._spare.pop()
            try:
                with self._poison_on_error():
                    self.binding.reset_error_flags()
            except BaseException:
                self._spare.append(slot)
                raise
            ticket = StepTicket(self._next_sequence, str(name), slot)
            self._next_sequence += 1
            self._open.append(ticket)
            self.resets += 1
            return ticket

    def queue(self, ticket):
        """Enqueue the copy of the step's flags behind the work issued so far."""
        with self._lock:
            if ticket.completed or ticket not in self._open:
                raise RuntimeError(f'step {ticket.sequence} is not open')
            if not ticket.queued:
                with self._poison_on_error():
                    self.transport.queue(ticket.slot)
                ticket.queued = True
                self.copies += 1

    def complete(self, ticket):
        """Check every open step up to this one, oldest first; returns this
        step's flags.  A non-zero flag poisons the worker and raises."""
        with self._lock:
            while self._open and self._open[0].sequence <= ticket.sequence:
                step = self._open[0]
                if not step.queued:
                    raise RuntimeError(f'step {step.sequence} ({step.name}) was never queued for its flag copy')
                with self._poison_on_error():
                    flags = tuple(int(v) for v in self.transport.finish(step.slot))
                    if len(flags) != len(self.binding.layer_prefixes):
                        raise RuntimeError(f'flag copy has {len(flags)} slots, expected '
                                           f'{len(self.binding.layer_prefixes)}')
                self._open.popleft()
                self._spare.append(step.slot)
                step.flags, step.completed = flags, True
                self.completions += 1
                bad = {p: v for p, v in zip(self.binding.layer_prefixes, flags) if v}
                if bad and self._fault is None:
                    self._fault = OrnithWorkerFault(f'step {step.sequence} ({step.name}) raised native flags {bad}')
            self.raise_if_failed()
            if not ticket.completed:
                raise RuntimeError(f'step {ticket.sequence} is unknown')
            return ticket.flags

    def abort(self, ticket, error):
        """A step ended in `error`: check its flags anyway, poison the worker
        and re-raise, keeping `error` as the cause of any flag fault."""
        try:
            self.queue(ticket)
            self.complete(ticket)
        except OrnithWorkerFault as fault:
            if fault is error:
                raise
            raise fault from error
        except BaseException as flag_error:
            error.add_note(f'the flag check after it failed too: {type(flag_error).__name__}: {flag_error}')
        self.poison(error)
        raise error

    def checked_output(self, output, ticket):
        """Return `output` once its step's flags are clean; an output with a
        get_output() method (an asynchronous runner output) is wrapped, and
        the check runs when get_output() is called."""
        if callable(getattr(output, 'get_output', None)):
            return CheckedAsyncOutput(output, self, ticket)
        self.complete(ticket)
        return output

    def drain(self):
        """Check every open step (shutdown, or a path that returns without output)."""
        with self._lock:
            for step in list(self._open):
                self.queue(step)
            if self._open:
                self.complete(self._open[-1])
            self.raise_if_failed()


class CheckedAsyncOutput:
    """An asynchronous output whose get_output() also checks its step: the
    wrapped output first (it waits for its own copy, queued after the flag
    copy), then the flags; the result is handed out only if both succeed."""

    def __init__(self, delegate, lifecycle, ticket):
        self._delegate, self._lifecycle, self._ticket = delegate, lifecycle, ticket
        self._consumed = False

    def get_output(self):
        if self._consumed:
            raise RuntimeError('this output was already taken')
        self._consumed = True
        try:
            result = self._delegate.get_output()
        except BaseException as error:
            self._lifecycle.abort(self._ticket, error)
        self._lifecycle.complete(self._ticket)
        return result
