"""ctypes binding of libornith_moe_b200.so and the torch custom operators.

Mirrors the reference plugin's binding (plugin-site/ornith_g256/native.py):
  * `configure(settings, capacity)` checks the routed activation settings the
    way native.py:28-44 does and selects the launch symbol
    (`ornith_routed_direct_launch`, `_a4` or `_a4_prefill`);
  * `ornith_b200::routed_out` has the argument order, validation and mutation
    set of `ornith_g256::routed_out` (native.py:156-186), including the
    per-phase segmentation of mixed prefill/decode batches;
  * `ornith_b200::routed_shared_out` is the fused shared-slot launch that
    moe_shared.py:130-174 drives;
  * `ornith_b200::routed_from_logits` is the north-star operator (hidden
    states + router logits -> combined hidden states);
  * `ornith_b200::dense_out` has the arguments and the A8 / bf16-prefill
    split of `ornith_g256::dense_out` (native.py:121-153), and
    `dense_n32_out` is the one-row N32 shadow launch of dense_n32.py:45-53;
  * `ornith_b200::head_out` is the W8 LM head launch of
    `ornith_g256::head_out` (native.py:205-212).
All launches go to the caller's current CUDA stream.  There is no CPU
fallback: every operator raises if the CUDA library is missing.
"""
import ctypes as C
import os
from pathlib import Path

import torch

HERE = Path(__file__).resolve().parent
# ORNITH_MOE_B200_LIB selects another build of the library (a variant written
# by build.py --out; relative paths are taken from this package's directory)
LIB_PATH = HERE / os.environ.get('ORNITH_MOE_B200_LIB', 'libornith_moe_b200.so')

_lib = None
_PHASE_SEGMENTS = ()
_SETTINGS = {'launch': 'ornith_routed_direct_launch'}


class RoutedLayout(C.Structure):
    """OrnithRoutedDirectLayout (include/ornith_moe_b200.h; reference native.py:16-20)."""
    _fields_ = [(n, C.c_size_t) for n in
                ('workspace_bytes', 'gate_x', 'gate_low', 'gate_high', 'gate_scales',
                 'gate_sums', 'gate_y', 'middle', 'down_x', 'down_low', 'down_high',
                 'down_scales', 'down_sums', 'route_out', 'final_f32')]


class DenseLayout(C.Structure):
    """OrnithDenseG256Layout (include/ornith_moe_b200.h; reference native.py:11-13)."""
    _fields_ = [(n, C.c_size_t) for n in
                ('workspace_bytes', 'transformed', 'low', 'high', 'scales', 'sums', 'projection')]


class HeadLayout(C.Structure):
    """OrnithHeadI8Layout (include/ornith_moe_b200.h; reference native.py:23-25)."""
    _fields_ = [(n, C.c_size_t) for n in
                ('workspace_bytes', 'transformed', 'activation_words', 'activation_scales', 'projection')]


_DENSE_ARGS = [C.c_void_p] * 4 + [C.c_size_t] + [C.c_void_p] * 2 + [C.c_int] * 7 + [C.c_void_p]
_LAUNCH_ARGS = [C.c_void_p] * 8 + [C.c_size_t] + [C.c_void_p] * 2 + [C.c_int] * 2 + [C.c_void_p]
SIGNATURES = {
    'ornith_routed_direct_get_layout': ([C.c_int, C.POINTER(RoutedLayout)], C.c_int),
    'ornith_routed_direct_launch': (_LAUNCH_ARGS, C.c_int),
    'ornith_routed_direct_launch_a4': (_LAUNCH_ARGS, C.c_int),
    'ornith_routed_direct_launch_a4_prefill': (_LAUNCH_ARGS, C.c_int),
    'ornith_routed_storage_n32': ([], C.c_int),
    'ornith_routed_prefill_output_tile': ([], C.c_int),
    'ornith_routed_shared_get_layout': ([C.c_int, C.POINTER(RoutedLayout)], C.c_int),
    'ornith_routed_direct_launch_shared_tables': (
        [C.c_void_p] * 15 + [C.c_size_t] + [C.c_void_p] * 3 + [C.c_int] * 2 + [C.c_void_p], C.c_int),
    'ornith_moe_b200_abi_version': ([], C.c_uint32),
    'ornith_moe_b200_kernel_launches': ([], C.c_ulonglong),
    'ornith_moe_b200_route_topk': ([C.c_void_p, C.c_int, C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p], C.c_int),
    'ornith_moe_b200_launch_from_logits': (
        [C.c_void_p] * 14 + [C.c_size_t] + [C.c_void_p] * 3 + [C.c_int] * 3 + [C.c_void_p], C.c_int),
    'ornith_moe_b200_get_layout': ([C.c_int, C.POINTER(C.c_size_t)], C.c_int),
    'ornith_moe_b200_router_logits': ([C.c_void_p, C.c_void_p, C.c_int, C.c_void_p, C.c_void_p], C.c_int),
    'ornith_moe_b200_launch_from_hidden': (
        [C.c_void_p] * 15 + [C.c_size_t] + [C.c_void_p] * 3 + [C.c_int] * 3 + [C.c_void_p], C.c_int),
    'ornith_moe_b200_combine': ([C.c_void_p] * 3 + [C.c_int] + [C.c_void_p] * 3, C.c_int),
    'ornith_moe_b200_combine_gathered': ([C.c_void_p, C.c_int] + [C.c_void_p] * 3 + [C.c_int] + [C.c_void_p] * 3,
                                         C.c_int),
    'ornith_moe_b200_gather_route_rows': ([C.c_void_p, C.c_size_t, C.c_int, C.c_int, C.c_void_p, C.c_int]
                                          + [C.c_void_p] * 3, C.c_int),
    'ornith_moe_b200_scatter_route_rows': ([C.c_void_p, C.c_size_t, C.c_int, C.c_int, C.c_void_p, C.c_void_p],
                                           C.c_int),
    'ornith_moe_b200_repack_n16_to_n32': ([C.c_void_p] * 4 + [C.c_int] * 3 + [C.c_void_p], C.c_int),
    'ornith_moe_b200_ep_plan': ([C.c_void_p, C.c_int, C.c_void_p, C.c_void_p, C.c_int] + [C.c_void_p] * 7, C.c_int),
    'ornith_moe_b200_ep_buffer_alloc': ([C.c_size_t, C.POINTER(C.c_void_p)], C.c_int),
    'ornith_moe_b200_ep_buffer_free': ([C.c_void_p], C.c_int),
    'ornith_moe_b200_ep_ipc_handle': ([C.c_void_p, C.c_void_p], C.c_int),
    'ornith_moe_b200_ep_ipc_open': ([C.c_void_p, C.POINTER(C.c_void_p)], C.c_int),
    'ornith_moe_b200_ep_ipc_close': ([C.c_void_p], C.c_int),
    'ornith_moe_b200_ep_return_p2p': ([C.c_void_p, C.c_size_t, C.c_int, C.c_int, C.c_void_p, C.c_int,
                                       C.POINTER(C.c_int32), C.POINTER(C.c_void_p), C.POINTER(C.c_int64), C.c_int64,
                                       C.POINTER(C.c_void_p), C.c_int, C.c_int, C.c_uint32, C.c_void_p, C.c_void_p,
                                       C.c_void_p], C.c_int),
    'ornith_moe_b200_ep_dispatch_p2p': ([C.c_void_p, C.c_int, C.c_void_p, C.c_void_p, C.c_int, C.POINTER(C.c_int32),
                                         C.POINTER(C.c_void_p), C.POINTER(C.c_void_p), C.POINTER(C.c_int64), C.c_int64,
                                         C.POINTER(C.c_void_p), C.c_int, C.c_int, C.c_uint32, C.c_void_p, C.c_void_p,
                                         C.c_void_p], C.c_int),
    'ornith_moe_b200_ep_fixed_dispatch': ([C.c_void_p, C.c_void_p, C.c_int] + [C.POINTER(C.c_void_p)] * 2
                                          + [C.c_int64, C.POINTER(C.c_void_p)]
                                          + [C.c_int, C.c_int] + [C.c_void_p] * 4, C.c_int),
    'ornith_moe_b200_ep_fixed_return': ([C.c_void_p, C.c_size_t, C.c_int, C.c_int, C.c_void_p]
                                        + [C.POINTER(C.c_void_p), C.c_int64, C.POINTER(C.c_void_p)]
                                        + [C.c_int, C.c_int] + [C.c_void_p] * 4, C.c_int),
    'ornith_moe_b200_ep_fixed_dispatch_weights': ([C.c_void_p, C.c_void_p, C.c_void_p, C.c_int]
                                                  + [C.POINTER(C.c_void_p)] * 3
                                                  + [C.c_int64, C.POINTER(C.c_void_p)]
                                                  + [C.c_int, C.c_int] + [C.c_void_p] * 4, C.c_int),
    'ornith_moe_b200_ep_fixed_return_partial': ([C.c_void_p, C.c_size_t, C.c_int, C.c_int, C.c_void_p]
                                                + [C.POINTER(C.c_void_p), C.c_int64, C.POINTER(C.c_void_p)]
                                                + [C.c_int, C.c_int] + [C.c_void_p] * 4, C.c_int),
    'ornith_moe_b200_set_peer_wait_limit_ns': ([C.c_uint64], C.c_int),
    'ornith_moe_b200_peer_wait_limit_ns': ([], C.c_uint64),
    'ornith_moe_b200_ep_wait_epoch': ([C.c_void_p, C.c_int, C.c_int, C.c_void_p, C.c_void_p, C.c_void_p], C.c_int),
    'ornith_moe_b200_ep_wait_signals': ([C.c_void_p, C.c_int, C.c_int, C.c_uint32, C.c_void_p, C.c_void_p], C.c_int),
    'ornith_routed_direct_launch_noalloc': ([C.c_void_p] * 9 + [C.c_int, C.c_void_p], C.c_int),
    'ornith_dense_g256_abi_version': ([], C.c_uint32),
    'ornith_dense_g256_get_layout': ([C.c_int] * 4 + [C.POINTER(DenseLayout)], C.c_int),
    'ornith_dense_g256_launch': (_DENSE_ARGS, C.c_int),
    'ornith_dense_g256_launch_n32': (_DENSE_ARGS, C.c_int),
    'ornith_dense_g256_n32_rows': ([], C.c_int),
    'ornith_dense_g256_prepare_bf16': ([C.c_void_p] * 6 + [C.c_int] * 3 + [C.c_void_p], C.c_int),
    'ornith_head_i8_tile_abi_version': ([], C.c_uint32),
    'ornith_head_i8_tile_get_layout': ([C.c_int, C.c_int, C.POINTER(HeadLayout)], C.c_int),
    'ornith_head_i8_tile_launch': ([C.c_void_p] * 4 + [C.c_size_t] + [C.c_void_p] * 2 + [C.c_size_t]
                                   + [C.c_void_p] + [C.c_int] * 4 + [C.c_void_p], C.c_int),
    'ornith_head_i8_tile_shortlist': ([], C.c_int),
}


def load(path):
    """A ctypes handle of a build of the library at `path`, with the
    signatures of every exported entry point set."""
    path = Path(path)
    if not path.exists():
        raise RuntimeError(f'{path} is missing: build it with `python {HERE / "build.py"}` '
                           '(or __graft_entry__.build()); the MoE operators have no CPU fallback')
    handle = C.CDLL(str(path))
    for name, (args, res) in SIGNATURES.items():
        fn = getattr(handle, name)
        fn.argtypes, fn.restype = args, res
    if handle.ornith_routed_storage_n32() != 32:
        raise RuntimeError(f'{path} does not report N32 expert storage (marker 32)')
    return handle


def lib():
    """Load the CUDA library (raises if it was not built: there is no fallback)."""
    global _lib
    if _lib is None:
        _lib = load(LIB_PATH)
    return _lib


def ptr(t):
    return C.c_void_p(t.data_ptr()) if t is not None else C.c_void_p(0)


def stream(x):
    return C.c_void_p(torch.cuda.current_stream(x.device).cuda_stream)


def check(status, operation):
    if status:
        raise RuntimeError(f'{operation} failed with native status {status}')


def get_layout(capacity):
    layout = RoutedLayout()
    check(lib().ornith_routed_direct_get_layout(capacity, C.byref(layout)), 'routed layout')
    return layout


def workspace_bytes(capacity):
    n = C.c_size_t()
    check(lib().ornith_moe_b200_get_layout(capacity, C.byref(n)), 'layout')
    return max(n.value, get_layout(capacity).workspace_bytes)


def configure(settings, capacity):
    """Select the routed launch symbol from the plugin settings (native.py:28-44)
    and return the workspace bytes for `capacity` rows."""
    bits = settings.get('routed_activation_bits', 8)
    prefill_bits = settings.get('routed_prefill_activation_bits', 8)
    if bits not in (4, 8) or prefill_bits not in (4, 8):
        raise ValueError('routed_activation_bits and routed_prefill_activation_bits take 4 or 8')
    if bits == prefill_bits == 4:
        raise ValueError('A4 everywhere and A4 for prefill only are exclusive: set one of the two to 8')
    suffix = '_a4' if bits == 4 else '_a4_prefill' if prefill_bits == 4 else ''
    _SETTINGS['launch'] = 'ornith_routed_direct_launch' + suffix
    return workspace_bytes(capacity)


def set_phase_segments(segments):
    """Mixed prefill/decode segmentation (phase_dispatch.py:13-34): a tuple of
    (start, end, prefill) row ranges; prefill segments use A4, decode ones A8."""
    global _PHASE_SEGMENTS
    _PHASE_SEGMENTS = tuple((int(a), int(b), bool(p)) for a, b, p in segments)


def _phase_plan(rows):
    """Row ranges (lo, hi, prefill) of a mixed prefill/decode batch: the
    configured segments, then any rows past them as prefill; None when the
    batch is not segmented (no segments, or fewer rows than they cover).
    The rule of the plugin's phase dispatch (native.py:124-135,162-168)."""
    if not _PHASE_SEGMENTS or rows < _PHASE_SEGMENTS[-1][1]:
        return None
    plan = list(_PHASE_SEGMENTS)
    covered = plan[-1][1]
    if covered < rows:
        plan.append((covered, rows, True))
    return plan


def validate(x, out, capacity, k):
    if (x.ndim != 2 or x.shape[1] != k or not 0 <= x.shape[0] <= capacity
            or x.dtype != torch.bfloat16 or x.device.type != 'cuda'
            or out.dtype != x.dtype or out.device != x.device
            or not x.is_contiguous() or not out.is_contiguous()):
        raise ValueError(f'expected contiguous CUDA bf16 rows [M <= {capacity}, {k}] '
                         'and a bf16 output on the same device')


def _validate_routes(x, routes, ids):
    if (routes.dtype != torch.float32 or ids.dtype != torch.int32
            or routes.shape != (x.shape[0], 8) or ids.shape != routes.shape
            or routes.device != x.device or ids.device != x.device
            or not routes.is_contiguous() or not ids.is_contiguous()):
        raise ValueError('routing weights must be contiguous fp32 [T, 8] and ids int32 [T, 8] on the input device')


def _routed_launch(symbol, x, routes, ids, gate, gate_meta, down, down_meta, workspace, out, flags, capacity):
    validate(x, out, capacity, 2048)
    _validate_routes(x, routes, ids)
    fn = getattr(lib(), symbol)
    check(fn(*[ptr(t) for t in (x, routes, ids, gate, gate_meta, down, down_meta, workspace)],
             workspace.numel(), ptr(out), ptr(flags), x.shape[0], capacity, stream(x)), 'G256 ' + symbol)


@torch.library.custom_op('ornith_b200::routed_out', mutates_args={'workspace', 'out', 'flags'}, device_types='cuda')
def routed_out(x: torch.Tensor, routes: torch.Tensor, ids: torch.Tensor,
               gate: torch.Tensor, gate_meta: torch.Tensor, down: torch.Tensor, down_meta: torch.Tensor,
               workspace: torch.Tensor, out: torch.Tensor, flags: torch.Tensor, capacity: int) -> None:
    plan = _phase_plan(x.shape[0])
    if plan is None:
        _routed_launch(_SETTINGS['launch'], x, routes, ids, gate, gate_meta, down, down_meta, workspace, out, flags,
                       capacity)
        return
    for lo, hi, prefill in plan:
        symbol = 'ornith_routed_direct_launch_a4' if prefill else 'ornith_routed_direct_launch'
        _routed_launch(symbol, x[lo:hi], routes[lo:hi], ids[lo:hi], gate, gate_meta, down, down_meta, workspace,
                       out[lo:hi], flags, capacity)


@routed_out.register_fake
def _routed_fake(x, routes, ids, gate, gate_meta, down, down_meta, workspace, out, flags, capacity):
    return None


@torch.library.custom_op('ornith_b200::routed_shared_out',
                         mutates_args={'workspace', 'out', 'shared_out', 'flags'}, device_types='cuda')
def routed_shared_out(x: torch.Tensor, routes: torch.Tensor, ids: torch.Tensor,
                      gate: torch.Tensor, gate_meta: torch.Tensor, down: torch.Tensor, down_meta: torch.Tensor,
                      shared_gate: torch.Tensor, shared_gate_meta: torch.Tensor,
                      shared_down: torch.Tensor, shared_down_meta: torch.Tensor,
                      logit: torch.Tensor, silu_table: torch.Tensor, sigmoid_table: torch.Tensor,
                      workspace: torch.Tensor, out: torch.Tensor, shared_out: torch.Tensor,
                      flags: torch.Tensor, capacity: int) -> None:
    validate(x, out, capacity, 2048)
    validate(x, shared_out, capacity, 2048)
    _validate_routes(x, routes, ids)
    if (silu_table.dtype != torch.float32 or sigmoid_table.dtype != torch.bfloat16
            or silu_table.shape != (65536,) or sigmoid_table.shape != (65536,)
            or logit.dtype != torch.bfloat16 or logit.numel() != x.shape[0]):
        raise ValueError('Invalid shared reference table geometry')
    check(lib().ornith_routed_direct_launch_shared_tables(
        *[ptr(t) for t in (x, routes, ids, gate, gate_meta, down, down_meta, shared_gate, shared_gate_meta,
                           shared_down, shared_down_meta, logit, silu_table, sigmoid_table, workspace)],
        workspace.numel(), ptr(out), ptr(shared_out), ptr(flags), x.shape[0], capacity, stream(x)),
        'G256 routed shared')


@routed_shared_out.register_fake
def _routed_shared_fake(x, routes, ids, gate, gate_meta, down, down_meta, shared_gate, shared_gate_meta,
                        shared_down, shared_down_meta, logit, silu_table, sigmoid_table, workspace, out,
                        shared_out, flags, capacity):
    return None


@torch.library.custom_op('ornith_b200::route_topk', mutates_args={'weights', 'ids', 'flags'}, device_types='cuda')
def route_topk(logits: torch.Tensor, weights: torch.Tensor, ids: torch.Tensor, flags: torch.Tensor) -> None:
    if (logits.dtype != torch.float32 or logits.ndim != 2 or logits.shape[1] != 256 or not logits.is_contiguous()
            or weights.shape != (logits.shape[0], 8) or ids.shape != weights.shape
            or weights.dtype != torch.float32 or ids.dtype != torch.int32):
        raise ValueError('route_topk requires FP32 logits [T,256] and [T,8] outputs')
    check(lib().ornith_moe_b200_route_topk(ptr(logits), logits.shape[0], ptr(weights), ptr(ids), ptr(flags),
                                           stream(logits)), 'route_topk')


@route_topk.register_fake
def _route_topk_fake(logits, weights, ids, flags):
    return None


@torch.library.custom_op('ornith_b200::routed_from_logits',
                         mutates_args={'workspace', 'out', 'shared_out', 'flags'}, device_types='cuda')
def routed_from_logits(x: torch.Tensor, logits: torch.Tensor,
                       gate: torch.Tensor, gate_meta: torch.Tensor, down: torch.Tensor, down_meta: torch.Tensor,
                       shared_gate: torch.Tensor | None, shared_gate_meta: torch.Tensor | None,
                       shared_down: torch.Tensor | None, shared_down_meta: torch.Tensor | None,
                       shared_gate_weight: torch.Tensor | None, silu_table: torch.Tensor | None,
                       sigmoid_table: torch.Tensor | None, workspace: torch.Tensor, out: torch.Tensor,
                       shared_out: torch.Tensor | None, flags: torch.Tensor, capacity: int, act_bits: int) -> None:
    validate(x, out, capacity, 2048)
    if logits.dtype != torch.float32 or logits.shape != (x.shape[0], 256) or not logits.is_contiguous():
        raise ValueError('routed_from_logits requires FP32 router logits [T,256]')
    check(lib().ornith_moe_b200_launch_from_logits(
        *[ptr(t) for t in (x, logits, gate, gate_meta, down, down_meta, shared_gate, shared_gate_meta,
                           shared_down, shared_down_meta, shared_gate_weight, silu_table, sigmoid_table,
                           workspace)],
        workspace.numel(), ptr(out), ptr(shared_out), ptr(flags), x.shape[0], capacity, act_bits, stream(x)),
        'routed_from_logits')


@routed_from_logits.register_fake
def _routed_from_logits_fake(x, logits, gate, gate_meta, down, down_meta, shared_gate, shared_gate_meta,
                             shared_down, shared_down_meta, shared_gate_weight, silu_table, sigmoid_table,
                             workspace, out, shared_out, flags, capacity, act_bits):
    return None


def router_logits(x, router_weight, logits):
    """Router linear: bf16 x [T,2048] and bf16 W [256,2048] -> fp32 logits [T,256]."""
    T = x.shape[0]
    if (x.dtype != torch.bfloat16 or x.shape != (T, 2048) or not x.is_contiguous()
            or router_weight.dtype != torch.bfloat16 or router_weight.shape != (256, 2048)
            or not router_weight.is_contiguous() or logits.dtype != torch.float32 or logits.shape != (T, 256)
            or not logits.is_contiguous()):
        raise ValueError('router_logits requires BF16 x [T,2048], BF16 W [256,2048] and FP32 logits [T,256]')
    check(lib().ornith_moe_b200_router_logits(ptr(x), ptr(router_weight), T, ptr(logits), stream(x)), 'router_logits')


@torch.library.custom_op('ornith_b200::routed_from_hidden',
                         mutates_args={'logits', 'workspace', 'out', 'shared_out', 'flags'}, device_types='cuda')
def routed_from_hidden(x: torch.Tensor, router_weight: torch.Tensor, logits: torch.Tensor,
                       gate: torch.Tensor, gate_meta: torch.Tensor, down: torch.Tensor, down_meta: torch.Tensor,
                       shared_gate: torch.Tensor | None, shared_gate_meta: torch.Tensor | None,
                       shared_down: torch.Tensor | None, shared_down_meta: torch.Tensor | None,
                       shared_gate_weight: torch.Tensor | None, silu_table: torch.Tensor | None,
                       sigmoid_table: torch.Tensor | None, workspace: torch.Tensor, out: torch.Tensor,
                       shared_out: torch.Tensor | None, flags: torch.Tensor, capacity: int, act_bits: int) -> None:
    """The router linear, then routed_from_logits; `logits` receives the router output."""
    validate(x, out, capacity, 2048)
    if (router_weight.dtype != torch.bfloat16 or router_weight.shape != (256, 2048)
            or not router_weight.is_contiguous() or logits.dtype != torch.float32
            or logits.shape != (x.shape[0], 256) or not logits.is_contiguous()):
        raise ValueError('routed_from_hidden requires BF16 router weight [256,2048] and FP32 logits [T,256]')
    check(lib().ornith_moe_b200_launch_from_hidden(
        *[ptr(t) for t in (x, router_weight, logits, gate, gate_meta, down, down_meta, shared_gate, shared_gate_meta,
                           shared_down, shared_down_meta, shared_gate_weight, silu_table, sigmoid_table,
                           workspace)],
        workspace.numel(), ptr(out), ptr(shared_out), ptr(flags), x.shape[0], capacity, act_bits, stream(x)),
        'routed_from_hidden')


@routed_from_hidden.register_fake
def _routed_from_hidden_fake(x, router_weight, logits, gate, gate_meta, down, down_meta, shared_gate,
                             shared_gate_meta, shared_down, shared_down_meta, shared_gate_weight, silu_table,
                             sigmoid_table, workspace, out, shared_out, flags, capacity, act_bits):
    return None


def combine_rows(route_rows, weights, ids, out, flags):
    """Slot-ordered combine of per-route fp32 rows [T*8, 2048] into bf16 out [T, 2048]."""
    T = ids.shape[0]
    if (route_rows.dtype != torch.float32 or route_rows.shape != (T * 8, 2048) or not route_rows.is_contiguous()
            or out.dtype != torch.bfloat16 or out.shape != (T, 2048) or not out.is_contiguous()):
        raise ValueError('combine_rows requires FP32 rows [T*8,2048] and a BF16 output [T,2048]')
    _validate_routes(out, weights, ids)
    check(lib().ornith_moe_b200_combine(ptr(route_rows), ptr(weights), ptr(ids), T, ptr(out), ptr(flags),
                                        stream(out)), 'combine')


def combine_gathered(rows, row_index, weights, ids, out, flags):
    """Slot-ordered combine from gathered fp32 rows [n, 2048]; row_index int32 [T, 8]
    names the row of each valid slot."""
    T = ids.shape[0]
    if (rows.dtype != torch.float32 or rows.dim() != 2 or rows.shape[1] != 2048 or not rows.is_contiguous()
            or row_index.dtype != torch.int32 or row_index.shape != (T, 8) or not row_index.is_contiguous()
            or out.dtype != torch.bfloat16 or out.shape != (T, 2048) or not out.is_contiguous()):
        raise ValueError('combine_gathered requires FP32 rows [n,2048], INT32 row_index [T,8], BF16 out [T,2048]')
    _validate_routes(out, weights, ids)
    check(lib().ornith_moe_b200_combine_gathered(ptr(rows), rows.shape[0], ptr(row_index), ptr(weights), ptr(ids), T,
                                                 ptr(out), ptr(flags), stream(out)), 'combine_gathered')


def gather_route_rows(workspace, T, capacity, route_index, rows, flags):
    """fp32 down projections of the routes route_index (8*token + slot) of the
    last layer call of T tokens on `workspace`, into rows [n, 2048]."""
    n = route_index.numel()
    if (route_index.dtype != torch.int32 or not route_index.is_contiguous() or rows.dtype != torch.float32
            or rows.shape != (n, 2048) or not rows.is_contiguous()):
        raise ValueError('gather_route_rows requires INT32 route indices [n] and FP32 rows [n,2048]')
    check(lib().ornith_moe_b200_gather_route_rows(ptr(workspace), workspace.numel(), T, capacity, ptr(route_index), n,
                                                  ptr(rows), ptr(flags), stream(rows)), 'gather_route_rows')


def ep_plan(ids, owner, local, world):
    """The expert-parallel dispatch plan of ids int32 [T, 8] in one launch
    (owner, local: int32 [256] placement tables).  Returns device tensors
    (counts int64 [world, 2], token_index int64, dest int64, local_ids int32
    [., 8], slot_mask bool [., 8], row_index int32 [T, 8]); the row buffers
    hold T * world rows, of which the first counts[:, 0].sum() are the plan."""
    T = ids.shape[0]
    dev = ids.device
    if (ids.dtype != torch.int32 or ids.dim() != 2 or ids.shape[1] != 8 or not ids.is_contiguous()
            or dev.type != 'cuda' or not 1 <= world <= 8 or T > 8192):
        raise ValueError('ep_plan takes contiguous CUDA int32 ids [T <= 8192, 8] and 1..8 ranks')
    for t in (owner, local):
        if t.dtype != torch.int32 or t.shape != (256,) or not t.is_contiguous() or t.device != dev:
            raise ValueError('ep_plan takes int32 [256] placement tables on the ids device')
    n = T * world
    counts = torch.empty((world, 2), dtype=torch.int64, device=dev)
    token_index = torch.empty(n, dtype=torch.int64, device=dev)
    dest = torch.empty(n, dtype=torch.int64, device=dev)
    local_ids = torch.empty((n, 8), dtype=torch.int32, device=dev)
    slot_mask = torch.empty((n, 8), dtype=torch.bool, device=dev)
    row_index = torch.empty((T, 8), dtype=torch.int32, device=dev)
    check(lib().ornith_moe_b200_ep_plan(ptr(ids), T, ptr(owner), ptr(local), world, ptr(counts), ptr(token_index),
                                        ptr(dest), ptr(local_ids), ptr(slot_mask), ptr(row_index), stream(ids)),
          'expert-parallel dispatch plan')
    return counts, token_index, dest, local_ids, slot_mask, row_index


def ep_buffer_alloc(nbytes):
    """A zeroed device allocation for a peer-memory receive buffer; its address."""
    p = C.c_void_p()
    check(lib().ornith_moe_b200_ep_buffer_alloc(int(nbytes), C.byref(p)), 'expert-parallel buffer allocation')
    return int(p.value)


def ep_buffer_free(address):
    check(lib().ornith_moe_b200_ep_buffer_free(C.c_void_p(address)), 'expert-parallel buffer release')


def ep_ipc_handle(address):
    """The 64-byte CUDA IPC handle of an ep_buffer_alloc allocation."""
    h = (C.c_uint8 * 64)()
    check(lib().ornith_moe_b200_ep_ipc_handle(C.c_void_p(address), h), 'IPC handle')
    return bytes(h)


def ep_ipc_open(handle):
    """Map another rank's buffer from its IPC handle; the local address."""
    if len(handle) != 64:
        raise ValueError('an IPC handle has 64 bytes')
    h = (C.c_uint8 * 64).from_buffer_copy(handle)
    p = C.c_void_p()
    check(lib().ornith_moe_b200_ep_ipc_open(h, C.byref(p)), 'IPC open')
    return int(p.value)


def ep_ipc_close(address):
    check(lib().ornith_moe_b200_ep_ipc_close(C.c_void_p(address)), 'IPC close')


def ep_return_p2p(workspace, T, capacity, route_index, seg, dst, offsets, cap_rows, signals, world, me, epoch,
                  counter, flags):
    """Store the fp32 down projections of route_index (rows [seg[h], seg[h+1])
    to home rank h) into the home ranks' receive buffers (dst: ctypes array of
    world addresses) at rows offsets[h]..., then raise `epoch` in their flag
    arrays (signals)."""
    n = route_index.numel()
    if (route_index.dtype != torch.int32 or not route_index.is_contiguous() or len(seg) != world + 1
            or len(offsets) != world or len(dst) != world or len(signals) != world):
        raise ValueError('ep_return_p2p takes INT32 route indices and per-rank segments, offsets and addresses')
    seg_a = (C.c_int32 * (world + 1))(*seg)
    off_a = (C.c_int64 * world)(*offsets)
    check(lib().ornith_moe_b200_ep_return_p2p(ptr(workspace), workspace.numel(), T, capacity, ptr(route_index), n,
                                              seg_a, dst, off_a, cap_rows, signals, world, me, epoch, ptr(counter),
                                              ptr(flags), stream(workspace)), 'expert-parallel peer return')


def ep_dispatch_p2p(x, token_index, local_ids, seg, dst_x, dst_ids, offsets, cap_tokens, signals, world, me, epoch,
                    counter, flags):
    """Store the sent token rows (x[token_index[i]], local_ids[i]; rows
    [seg[d], seg[d+1]) to expert rank d) into the expert ranks' receive
    buffers (dst_x, dst_ids: ctypes arrays of world addresses) at rows
    offsets[d]..., then raise `epoch` in their dispatch flag arrays."""
    n = token_index.numel()
    if (x.dtype != torch.bfloat16 or x.dim() != 2 or x.shape[1] != 2048 or not x.is_contiguous()
            or token_index.dtype != torch.int64 or not token_index.is_contiguous()
            or local_ids.dtype != torch.int32 or local_ids.shape != (n, 8) or not local_ids.is_contiguous()
            or len(seg) != world + 1 or len(offsets) != world):
        raise ValueError('ep_dispatch_p2p takes bf16 rows [T, 2048], INT64 token indices and INT32 local ids [n, 8]')
    seg_a = (C.c_int32 * (world + 1))(*seg)
    off_a = (C.c_int64 * world)(*offsets)
    check(lib().ornith_moe_b200_ep_dispatch_p2p(ptr(x), x.shape[0], ptr(token_index), ptr(local_ids), n, seg_a, dst_x,
                                                dst_ids, off_a, cap_tokens, signals, world, me, epoch, ptr(counter),
                                                ptr(flags), stream(x)), 'expert-parallel peer dispatch')


def ep_fixed_dispatch(x, local_ids, dst_x, dst_ids, cap_rows, signals, world, me, epoch, counter, flags):
    """Fixed-size dispatch over peer memory: x bf16 [T, 2048] and local_ids
    int32 [world, T, 8] into every rank's receive set of this call (dst_x,
    dst_ids: ctypes arrays [2 * world], cap_rows rows per set); epoch: the
    int32 call counter; flags: this rank's flag word, whose timeout bit goes
    with the epoch."""
    T = x.shape[0]
    if (x.dtype != torch.bfloat16 or x.shape != (T, 2048) or not x.is_contiguous() or local_ids.dtype != torch.int32
            or local_ids.shape != (world, T, 8) or not local_ids.is_contiguous()):
        raise ValueError('ep_fixed_dispatch takes bf16 rows [T, 2048] and INT32 ids [world, T, 8]')
    check(lib().ornith_moe_b200_ep_fixed_dispatch(ptr(x), ptr(local_ids), T, dst_x, dst_ids, cap_rows, signals,
                                                  world, me, ptr(epoch), ptr(counter), ptr(flags), stream(x)),
          'expert-parallel fixed dispatch')


def ep_fixed_return(workspace, T, capacity, ids, dst_rows, cap_rows, signals, world, me, epoch, counter, flags):
    """Fixed-size return over peer memory after a layer call on ids int32
    [world * T, 8] (local ids; -1 where another rank owns the slot); every
    set of dst_rows holds cap_rows rows."""
    if ids.dtype != torch.int32 or ids.shape != (world * T, 8) or not ids.is_contiguous():
        raise ValueError('ep_fixed_return takes the INT32 local ids [world * T, 8] of the layer call')
    check(lib().ornith_moe_b200_ep_fixed_return(ptr(workspace), workspace.numel(), T, capacity, ptr(ids), dst_rows,
                                                cap_rows, signals, world, me, ptr(epoch), ptr(counter), ptr(flags),
                                                stream(ids)), 'expert-parallel fixed return')


def ep_fixed_dispatch_weights(x, local_ids, local_w, dst_x, dst_ids, dst_w, cap_rows, signals, world, me, epoch,
                              counter, flags):
    """ep_fixed_dispatch that also carries local_w fp32 [world, T, 8] (the
    weights of each rank's slots, 0 elsewhere) into dst_w, for the
    rank-partial combine."""
    T = x.shape[0]
    if (x.dtype != torch.bfloat16 or x.shape != (T, 2048) or not x.is_contiguous() or local_ids.dtype != torch.int32
            or local_ids.shape != (world, T, 8) or not local_ids.is_contiguous() or local_w.dtype != torch.float32
            or local_w.shape != (world, T, 8) or not local_w.is_contiguous()):
        raise ValueError('ep_fixed_dispatch_weights takes bf16 rows [T, 2048], INT32 ids and FP32 weights '
                         '[world, T, 8]')
    check(lib().ornith_moe_b200_ep_fixed_dispatch_weights(ptr(x), ptr(local_ids), ptr(local_w), T, dst_x, dst_ids,
                                                          dst_w, cap_rows, signals, world, me, ptr(epoch),
                                                          ptr(counter), ptr(flags), stream(x)),
          'expert-parallel fixed dispatch with weights')


def ep_fixed_return_partial(workspace, T, capacity, ids, dst_part, cap_rows, signals, world, me, epoch, counter,
                            flags):
    """Rank-partial return over peer memory after a layer call on ids int32
    [world * T, 8]: each token's fp32 sum over this rank's slots goes to its
    home rank's partial buffer (every set of dst_part holds cap_rows rows)."""
    if ids.dtype != torch.int32 or ids.shape != (world * T, 8) or not ids.is_contiguous():
        raise ValueError('ep_fixed_return_partial takes the INT32 local ids [world * T, 8] of the layer call')
    check(lib().ornith_moe_b200_ep_fixed_return_partial(ptr(workspace), workspace.numel(), T, capacity, ptr(ids),
                                                        dst_part, cap_rows, signals, world, me, ptr(epoch),
                                                        ptr(counter), ptr(flags), stream(ids)),
          'expert-parallel fixed partial return')


def set_peer_wait_limit_ns(limit_ns):
    """Limit of the bounded waits on other ranks (ns; 1 s by default)."""
    check(lib().ornith_moe_b200_set_peer_wait_limit_ns(int(limit_ns)), 'peer wait limit')


def peer_wait_limit_ns():
    return int(lib().ornith_moe_b200_peer_wait_limit_ns())


def ep_wait_epoch(signals_address, world, me, epoch, flags):
    check(lib().ornith_moe_b200_ep_wait_epoch(C.c_void_p(signals_address), world, me, ptr(epoch), ptr(flags),
                                              stream(flags)), 'expert-parallel peer wait')


def ep_wait_signals(signals_address, world, me, epoch, flags):
    check(lib().ornith_moe_b200_ep_wait_signals(C.c_void_p(signals_address), world, me, epoch, ptr(flags),
                                                stream(flags)), 'expert-parallel peer wait')


def scatter_route_rows(workspace, T, capacity, rows):
    """Route-ordered fp32 down projections [8T, 2048] of the last layer call of
    T tokens on `workspace` (rows of padding slots hold unspecified values)."""
    if rows.dtype != torch.float32 or rows.shape != (T * 8, 2048) or not rows.is_contiguous():
        raise ValueError('scatter_route_rows requires FP32 rows [8T,2048]')
    check(lib().ornith_moe_b200_scatter_route_rows(ptr(workspace), workspace.numel(), T, capacity, ptr(rows),
                                                   stream(rows)), 'scatter_route_rows')


def repack_n16_to_n32(codes16, meta16, N, K):
    """Device repack of checkpoint N16 banks to N32 storage (method.py:124-158)."""
    e = codes16.shape[0]
    codes32 = torch.empty((e, N // 32, K // 256, 32, 32), dtype=torch.uint32, device=codes16.device)
    meta32 = torch.empty((e, N // 32, K // 256, 32), dtype=torch.uint32, device=codes16.device)
    check(lib().ornith_moe_b200_repack_n16_to_n32(ptr(codes16.contiguous()), ptr(meta16.contiguous()),
                                                  ptr(codes32), ptr(meta32), e, N, K, stream(codes16)), 'repack')
    return codes32, meta32


# ---------------------------------------------------------------------------
# Dense G256 projections (reference native.py:121-153, dense_n32.py:37-53)
# ---------------------------------------------------------------------------

def dense_get_layout(capacity, n, k):
    layout = DenseLayout()
    check(lib().ornith_dense_g256_get_layout(capacity, n, k, 8, C.byref(layout)), 'dense layout')
    return layout


def dense_workspace_bytes(capacity, shapes):
    """Arena bytes for dense calls of up to `capacity` rows over (n, k) shapes:
    the A8 workspace, or the bf16 prefill buffers [capacity,k] + [n,k]
    (native.py:87-91)."""
    sizes = []
    for n, k in shapes:
        sizes.append(dense_get_layout(capacity, n, k).workspace_bytes)
        sizes.append((capacity * k + n * k) * 2)
    return max(sizes)


def _bf16_prefill_views(workspace, capacity, m, n, k):
    """The arena as the bf16 prefill path uses it (the plugin sizes it for
    this, native.py:87-91): bf16 H128(x) [m, k] from byte 0, the dequantised
    bf16 weights [n, k] from byte capacity*k*2."""
    w0 = capacity * k * 2
    if workspace.numel() < w0 + n * k * 2:
        raise ValueError('G256 dense workspace too small for the bf16 prefill path')
    xt = workspace[:m * k * 2].view(torch.bfloat16).view(m, k)
    w = workspace[w0:w0 + n * k * 2].view(torch.bfloat16).view(n, k)
    return xt, w


def _dense_impl(x, codes, metadata, workspace, out, flags, capacity, n, k, geometry, a8_max_rows):
    validate(x, out, capacity, k)
    m = x.shape[0]
    if out.shape != (m, n):
        raise ValueError('Native G256 dense output must be [M, N]')
    if m <= a8_max_rows:
        check(lib().ornith_dense_g256_launch(ptr(x), ptr(codes), ptr(metadata), ptr(workspace), workspace.numel(),
                                             ptr(out), ptr(flags), m, capacity, n, k, 8, 128, geometry, stream(x)),
              'G256 dense')
        return
    # longer batches: bf16 operands prepared in the arena, then a bf16 GEMM
    xt, w = _bf16_prefill_views(workspace, capacity, m, n, k)
    check(lib().ornith_dense_g256_prepare_bf16(ptr(x), ptr(codes), ptr(metadata), ptr(xt), ptr(w), ptr(flags), m,
                                                n, k, stream(x)), 'G256 BF16 prefill preparation')
    torch.mm(xt, w.t(), out=out)


@torch.library.custom_op('ornith_b200::dense_out', mutates_args={'workspace', 'out', 'flags'}, device_types='cuda')
def dense_out(x: torch.Tensor, codes: torch.Tensor, metadata: torch.Tensor,
              workspace: torch.Tensor, out: torch.Tensor, flags: torch.Tensor,
              capacity: int, n: int, k: int, geometry: int, a8_max_rows: int) -> None:
    """out[M,n] = x[M,k] projected by an N16 G256 bank: A8 for M <= a8_max_rows,
    else the bf16 prefill path; a mixed batch follows the phase segments
    (decode rows A8, prefill rows bf16)."""
    plan = _phase_plan(x.shape[0])
    if plan is None:
        _dense_impl(x, codes, metadata, workspace, out, flags, capacity, n, k, geometry, a8_max_rows)
        return
    for lo, hi, prefill in plan:
        _dense_impl(x[lo:hi], codes, metadata, workspace, out[lo:hi], flags, capacity, n, k, geometry,
                    0 if prefill else capacity)


@dense_out.register_fake
def _dense_fake(x, codes, metadata, workspace, out, flags, capacity, n, k, geometry, a8_max_rows):
    return None


def dense_n32_out(x, codes32, metadata32, workspace, out, flags, capacity, n, k):
    """A8 projection of 1..16 rows from an N32 shadow bank (dense_n32.py:45-53)."""
    validate(x, out, capacity, k)
    check(lib().ornith_dense_g256_launch_n32(ptr(x), ptr(codes32), ptr(metadata32), ptr(workspace),
                                             workspace.numel(), ptr(out), ptr(flags), x.shape[0], capacity,
                                             n, k, 8, 128, 2, stream(x)), 'G256 dense N32')


def dense_n32_shadow(codes, metadata, n, k):
    """N32 shadow of an N16 dense bank on the device (dense_n32.py:30-31),
    through the repack kernel with one bank."""
    codes32, meta32 = repack_n16_to_n32(codes.reshape(1, n // 16, k // 256, 32, 16),
                                        metadata.reshape(1, n // 16, k // 256, 16), n, k)
    return codes32[0], meta32[0]


# ---------------------------------------------------------------------------
# W8 LM head (reference native.py:205-212)
# ---------------------------------------------------------------------------
HEAD_VOCAB, HEAD_ROWS = 248320, 64


def head_get_layout(capacity, n=HEAD_VOCAB):
    layout = HeadLayout()
    check(lib().ornith_head_i8_tile_get_layout(capacity, n, C.byref(layout)), 'head layout')
    return layout


@torch.library.custom_op('ornith_b200::head_out', mutates_args={'workspace', 'out', 'flags'}, device_types='cuda')
def head_out(x: torch.Tensor, codes: torch.Tensor, scales: torch.Tensor,
             workspace: torch.Tensor, out: torch.Tensor, flags: torch.Tensor, geometry: int) -> None:
    """Logits bf16 [M, 248320] of up to 64 rows x bf16 [M, 2048] through the
    int8 head bank (codes uint32 [15520, 128, 4, 16], scales fp16 [248320, 16])."""
    validate(x, out, HEAD_ROWS, 2048)
    check(lib().ornith_head_i8_tile_launch(ptr(x), ptr(codes), ptr(scales), ptr(workspace), workspace.numel(),
                                           ptr(out), None, 0, ptr(flags), x.shape[0], HEAD_ROWS, out.shape[1],
                                           geometry, stream(x)), 'W8 head')


@head_out.register_fake
def _head_fake(x, codes, scales, workspace, out, flags, geometry):
    return None


def head_launch(x, codes, scales, workspace, out, flags, n, capacity=HEAD_ROWS, geometry=2, group_dots=None):
    """The head launch for any supported vocabulary size n, optionally storing
    the raw group dots int32 [M, n, 16]."""
    validate(x, out, capacity, 2048)
    nbytes = group_dots.numel() * group_dots.element_size() if group_dots is not None else 0
    check(lib().ornith_head_i8_tile_launch(ptr(x), ptr(codes), ptr(scales), ptr(workspace), workspace.numel(),
                                           ptr(out), ptr(group_dots) if group_dots is not None else None, nbytes,
                                           ptr(flags), x.shape[0], capacity, n, geometry, stream(x)), 'W8 head')


# ---------------------------------------------------------------------------
# Shared expert in the reference's dense decode form
# (plugin-site/ornith_g256/iu4_correctness/shared_kernel.py:33-62, `fixed8`)
# ---------------------------------------------------------------------------
SHARED_DENSE_ROWS = 16  # rows per dense N32 launch (ornith_dense_g256_n32_rows)


def shared_dense_workspace_bytes():
    """Workspace for shared_dense_out: the dense N32 launches of 16 rows."""
    return max(dense_get_layout(SHARED_DENSE_ROWS, 1024, 2048).workspace_bytes,
               dense_get_layout(SHARED_DENSE_ROWS, 2048, 512).workspace_bytes)


def shared_dense_out(x, gate_codes, gate_meta, down_codes, down_meta, gate_weight, workspace, gate_flags,
                     down_flags):
    """The shared expert as the reference's production decode computes it
    (shared_kernel.py:33-62, which overwrites the fused ninth slot's decode
    rows, shared_live.py:125-137): gate/up = the dense A8 projection of x by
    the shared expert's N32 gate/up bank (bf16 [M, 1024]); act =
    bf16(bf16(silu(gate)) * up) in the arithmetic of vLLM's silu_and_mul;
    down = the dense A8 projection of act by the N32 down bank (bf16
    [M, 2048]); out = bf16(sigmoid(bf16(sum_k x*w_gate)) * down), the gate
    logit summed in fp32.  The projections are this library's dense N32
    launches (16 rows at a time: rows are independent, so the reference's
    padding to 8 rows changes nothing); the elementwise tail and the logit are
    torch operations, as the reference's are vLLM and torch operations.
    gate_flags / down_flags receive the dense flag bits of the two launches."""
    if (x.ndim != 2 or x.shape[1] != 2048 or x.dtype != torch.bfloat16 or x.device.type != 'cuda'
            or not x.is_contiguous()):
        raise ValueError('shared_dense_out requires contiguous CUDA BF16 rows [M, 2048]')
    if gate_weight.dtype != torch.bfloat16 or gate_weight.numel() != 2048:
        raise ValueError('shared_dense_out requires a BF16 shared gate weight of 2048 values')
    result = torch.empty_like(x)
    M = x.shape[0]
    if M == 0:
        return result
    logit = (x.float() @ gate_weight.reshape(2048, 1).float()).to(torch.bfloat16)   # [M, 1]
    gate = torch.sigmoid(logit)
    for first in range(0, M, SHARED_DENSE_ROWS):
        chunk = x[first:first + SHARED_DENSE_ROWS]
        m = chunk.shape[0]
        gu = torch.empty((m, 1024), dtype=torch.bfloat16, device=x.device)
        dense_n32_out(chunk, gate_codes, gate_meta, workspace, gu, gate_flags, SHARED_DENSE_ROWS, 1024, 2048)
        act = torch.nn.functional.silu(gu[:, :512].float()).to(torch.bfloat16) * gu[:, 512:]
        down = torch.empty((m, 2048), dtype=torch.bfloat16, device=x.device)
        dense_n32_out(act, down_codes, down_meta, workspace, down, down_flags, SHARED_DENSE_ROWS, 2048, 512)
        result[first:first + m] = gate[first:first + m] * down
    return result
