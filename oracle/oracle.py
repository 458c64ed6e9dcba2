"""ctypes front-end of the CPU oracle (test infrastructure only).

Two checkers live here:
  * `liboracle.so`, the C restatement of the reference's routed-MoE arithmetic
    (oracle/ornith_oracle.c);
  * the reference's own HIP sources compiled for the CPU (oracle/build_ref.py),
    called through the reference's exported C ABI
    (kernels/routed_storage/routed_direct_api.h:13-33,
    routed_storage_n32_consumer.cpp:309-401).

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg may
import this module.  The product path never does.
"""
import ctypes as C
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIB_PATH = HERE / '_build' / 'liboracle.so'
REF_DIR = HERE / '_ref'

E, TOP, H, I, G = 256, 8, 2048, 512, 256

_lib = None
_refs = {}


def build():
    """Compile liboracle.so (and the reference libraries when the reference checkout exists)."""
    subprocess.run(['make', '-s', '-C', str(HERE)], check=True)
    from . import build_ref  # noqa: WPS433
    ref = build_ref.reference_root()
    if ref is not None:
        build_ref.build(ref)


def _p(a):
    return a.ctypes.data_as(C.c_void_p)


def lib():
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            subprocess.run(['make', '-s', '-C', str(HERE)], check=True)
        _lib = C.CDLL(str(LIB_PATH))
        _lib.orc_bf16_rne.restype = C.c_uint16
        _lib.orc_bf16_rne.argtypes = [C.c_float]
        _lib.orc_f32_to_half_rne.restype = C.c_uint16
        _lib.orc_f32_to_half_rne.argtypes = [C.c_float]
        _lib.orc_half_to_f32.restype = C.c_float
        _lib.orc_half_to_f32.argtypes = [C.c_uint16]
        _lib.orc_portable_exp.restype = C.c_float
        _lib.orc_portable_exp.argtypes = [C.c_float]
        _lib.orc_silu.restype = C.c_float
        _lib.orc_silu.argtypes = [C.c_float]
        _lib.orc_set_threads.restype = C.c_int
        _lib.orc_set_threads.argtypes = [C.c_int]
        for name in ('orc_routed_layer', 'orc_routed_layer_shared'):
            getattr(_lib, name).restype = C.c_int
    return _lib


def set_threads(n):
    return lib().orc_set_threads(int(n))


def _c(a, dtype):
    a = np.ascontiguousarray(a)
    if a.dtype != dtype:
        raise TypeError(f'expected {dtype}, got {a.dtype}')
    return a


def _banks(gate_codes, gate_meta, down_codes, down_meta):
    return [_c(gate_codes, np.uint32), _c(gate_meta, np.uint32), _c(down_codes, np.uint32), _c(down_meta, np.uint32)]


def routed_layer(x_bits, weights, ids, gate_codes, gate_meta, down_codes, down_meta, a8=True):
    """Routed layer; x_bits uint16 bf16 bits [T,2048].  Returns (out bf16 bits, out fp32, flags)."""
    x_bits = _c(x_bits, np.uint16)
    weights = _c(weights, np.float32)
    ids = _c(ids, np.int32)
    T = x_bits.shape[0]
    banks = _banks(gate_codes, gate_meta, down_codes, down_meta)
    out = np.zeros((T, H), np.uint16)
    out_f32 = np.zeros((T, H), np.float32)
    flags = np.zeros(1, np.uint32)
    rc = lib().orc_routed_layer(_p(x_bits), _p(weights), _p(ids), C.c_int(T), *[_p(b) for b in banks],
                                C.c_int(1 if a8 else 0), _p(out), _p(out_f32), _p(flags))
    if rc:
        raise MemoryError('oracle allocation failed')
    return out, out_f32, int(flags[0])


def routed_layer_shared(x_bits, weights, ids, gate_codes, gate_meta, down_codes, down_meta,
                        sgate_codes, sgate_meta, sdown_codes, sdown_meta, logit_bits, silu_table, sigmoid_bits):
    """Routed layer + fused shared slot (A8).  Returns (out, shared_out, out_f32, flags)."""
    x_bits = _c(x_bits, np.uint16)
    T = x_bits.shape[0]
    args = [x_bits, _c(weights, np.float32), _c(ids, np.int32)]
    banks = _banks(gate_codes, gate_meta, down_codes, down_meta) + _banks(sgate_codes, sgate_meta, sdown_codes, sdown_meta)
    tables = [_c(logit_bits, np.uint16), _c(silu_table, np.float32), _c(sigmoid_bits, np.uint16)]
    out = np.zeros((T, H), np.uint16)
    shared = np.zeros((T, H), np.uint16)
    out_f32 = np.zeros((T, H), np.float32)
    flags = np.zeros(1, np.uint32)
    rc = lib().orc_routed_layer_shared(_p(args[0]), _p(args[1]), _p(args[2]), C.c_int(T),
                                       *[_p(b) for b in banks], *[_p(t) for t in tables],
                                       _p(out), _p(shared), _p(out_f32), _p(flags))
    if rc:
        raise MemoryError('oracle allocation failed')
    return out, shared, out_f32, int(flags[0])


def route_topk(logits):
    logits = _c(logits, np.float32)
    T = logits.shape[0]
    w = np.zeros((T, TOP), np.float32)
    ids = np.zeros((T, TOP), np.int32)
    lib().orc_route_topk(_p(logits), C.c_int(T), _p(w), _p(ids))
    return w, ids


def router_logits(x_bits, w_bits):
    x_bits, w_bits = _c(x_bits, np.uint16), _c(w_bits, np.uint16)
    out = np.zeros((x_bits.shape[0], E), np.float32)
    lib().orc_router_logits(_p(x_bits), _p(w_bits), C.c_int(x_bits.shape[0]), _p(out))
    return out


def transform_tokens(x_bits, ids=None):
    x_bits = _c(x_bits, np.uint16)
    T = x_bits.shape[0]
    y = np.zeros((T, H), np.float32)
    flags = np.zeros(1, np.uint32)
    lib().orc_transform_tokens(_p(x_bits), None if ids is None else _p(_c(ids, np.int32)), C.c_int(T), _p(y), _p(flags))
    return y, int(flags[0])


def quantize_rows(y, a8=True):
    y = _c(y, np.float32)
    rows, K = y.shape
    q = np.zeros((rows, K), np.int8)
    scales = np.zeros((rows, K // G), np.uint16)
    sums = np.zeros((rows, K // G), np.int32)
    flags = np.zeros(1, np.uint32)
    lib().orc_quantize_rows(_p(y), C.c_int(rows), C.c_int(K), C.c_int(1 if a8 else 0), _p(q), _p(scales), _p(sums), _p(flags))
    return q, scales, sums, int(flags[0])


def wht128(v):
    v = _c(v, np.float32)
    out = np.zeros(128, np.float32)
    lib().orc_wht128(_p(v), _p(out))
    return out


def fp32_reference_layer(x_bits, weights, ids, gate_codes, gate_meta, down_codes, down_meta):
    x_bits = _c(x_bits, np.uint16)
    T = x_bits.shape[0]
    out = np.zeros((T, H), np.float32)
    banks = _banks(gate_codes, gate_meta, down_codes, down_meta)
    lib().orc_fp32_reference_layer(_p(x_bits), _p(_c(weights, np.float32)), _p(_c(ids, np.int32)), C.c_int(T),
                                   *[_p(b) for b in banks], _p(out))
    return out


def repack_n16_to_n32(codes16, meta16, N, K):
    codes16, meta16 = _c(codes16, np.uint32), _c(meta16, np.uint32)
    Ex = codes16.shape[0]
    codes32 = np.zeros((Ex, N // 32, K // G, 32, 32), np.uint32)
    meta32 = np.zeros((Ex, N // 32, K // G, 32), np.uint32)
    lib().orc_repack_n16_to_n32(_p(codes16), _p(meta16), C.c_int(Ex), C.c_int(N), C.c_int(K), _p(codes32), _p(meta32))
    return codes32, meta32


# ---------------------------------------------------------------------------
# The reference's own source, compiled for the CPU (oracle/_ref).
# ---------------------------------------------------------------------------

class RoutedLayout(C.Structure):
    """OrnithRoutedDirectLayout, kernels/routed_storage/routed_direct_api.h:11-14."""
    _fields_ = [(n, C.c_size_t) for n in
                ('workspace_bytes', 'gate_x', 'gate_low', 'gate_high', 'gate_scales',
                 'gate_sums', 'gate_y', 'middle', 'down_x', 'down_low', 'down_high',
                 'down_scales', 'down_sums', 'route_out', 'final_f32')]


def reference_available(name='routed_storage_n32'):
    return (REF_DIR / f'libref_{name}.so').exists()


def ref_lib(name='routed_storage_n32'):
    if name not in _refs:
        path = REF_DIR / f'libref_{name}.so'
        if not path.exists():
            raise FileNotFoundError(f'{path} not built (python oracle/build_ref.py in the build container)')
        _refs[name] = C.CDLL(str(path))
    return _refs[name]


def ref_routed(x_bits, weights, ids, gate_codes, gate_meta, down_codes, down_meta, entry='ornith_routed_direct_launch',
               Tcap=None, library='routed_storage_n32'):
    """Run the compiled reference entry point.  Returns (out bf16 bits, final fp32 diagnostic, flags, status)."""
    L = ref_lib(library)
    x_bits = _c(x_bits, np.uint16)
    T = x_bits.shape[0]
    Tcap = T if Tcap is None else Tcap
    layout = RoutedLayout()
    L.ornith_routed_direct_get_layout.restype = C.c_int
    st = L.ornith_routed_direct_get_layout(C.c_int(Tcap), C.byref(layout))
    if st:
        return None, None, None, st
    ws = np.zeros(max(layout.workspace_bytes, 1), np.uint8)
    out = np.zeros((max(T, 1), H), np.uint16)
    flags = np.zeros(1, np.uint32)
    banks = _banks(gate_codes, gate_meta, down_codes, down_meta)
    fn = getattr(L, entry)
    fn.restype = C.c_int
    st = fn(_p(x_bits), _p(_c(weights, np.float32)), _p(_c(ids, np.int32)), *[_p(b) for b in banks],
            _p(ws), C.c_size_t(ws.size), _p(out), _p(flags), C.c_int(T), C.c_int(Tcap), None)
    final = ws[layout.final_f32:layout.final_f32 + T * H * 4].view(np.float32).reshape(T, H).copy() if T else None
    return out[:T], final, int(flags[0]), st


def ref_routed_shared(x_bits, weights, ids, gate_codes, gate_meta, down_codes, down_meta,
                      sgate_codes, sgate_meta, sdown_codes, sdown_meta, logit_bits, silu_table, sigmoid_bits, Tcap=16):
    """ornith_routed_direct_launch_shared_tables of the compiled reference."""
    L = ref_lib('routed_storage_n32')
    x_bits = _c(x_bits, np.uint16)
    T = x_bits.shape[0]
    layout = RoutedLayout()
    L.ornith_routed_shared_get_layout.restype = C.c_int
    st = L.ornith_routed_shared_get_layout(C.c_int(Tcap), C.byref(layout))
    if st:
        return None, None, None, st
    ws = np.zeros(layout.workspace_bytes, np.uint8)
    out = np.zeros((T, H), np.uint16)
    shared = np.zeros((T, H), np.uint16)
    flags = np.zeros(1, np.uint32)
    banks = _banks(gate_codes, gate_meta, down_codes, down_meta) + _banks(sgate_codes, sgate_meta, sdown_codes, sdown_meta)
    tables = [_c(logit_bits, np.uint16), _c(silu_table, np.float32), _c(sigmoid_bits, np.uint16)]
    fn = L.ornith_routed_direct_launch_shared_tables
    fn.restype = C.c_int
    st = fn(_p(x_bits), _p(_c(weights, np.float32)), _p(_c(ids, np.int32)), *[_p(b) for b in banks],
            *[_p(t) for t in tables], _p(ws), C.c_size_t(ws.size), _p(out), _p(shared), _p(flags),
            C.c_int(T), C.c_int(Tcap), None)
    return out, shared, int(flags[0]), st


# ---------------------------------------------------------------------------
# Dense G256 projection (kernels/dense_n32/, dense_g256_api.h:20-38)
# ---------------------------------------------------------------------------

def dense_project(x_bits, codes, meta, N, K, width=16):
    """A8 dense projection of bf16 rows x [M,K] by a bank stored `width` (16 or 32)
    columns per tile.  Returns (out bf16 bits [M,N], fp32 values [M,N], flags)."""
    x_bits = _c(x_bits, np.uint16).reshape(-1, K)
    M = x_bits.shape[0]
    out = np.zeros((M, N), np.uint16)
    diag = np.zeros((M, N), np.float32)
    flags = np.zeros(1, np.uint32)
    lib().orc_dense_project(_p(x_bits), C.c_int(M), C.c_int(N), C.c_int(K), C.c_int(width),
                            _p(_c(codes, np.uint32)), _p(_c(meta, np.uint32)), _p(out), _p(diag), _p(flags))
    return out, diag, int(flags[0])


def dense_prepare_bf16(x_bits, codes16, meta16, N, K):
    """Prefill preparation: (bf16 H128(x) [M,K], bf16 dequantised W [N,K], flags)."""
    x_bits = _c(x_bits, np.uint16).reshape(-1, K)
    M = x_bits.shape[0]
    xt = np.zeros((M, K), np.uint16)
    w = np.zeros((N, K), np.uint16)
    flags = np.zeros(1, np.uint32)
    lib().orc_dense_prepare_bf16(_p(x_bits), C.c_int(M), C.c_int(N), C.c_int(K),
                                 _p(_c(codes16, np.uint32)), _p(_c(meta16, np.uint32)), _p(xt), _p(w), _p(flags))
    return xt, w, int(flags[0])


def _aligned_bytes(n, alignment=256):
    """Zeroed uint8 buffer of n bytes starting on an `alignment`-byte boundary."""
    raw = np.zeros(n + alignment, np.uint8)
    skip = (-raw.ctypes.data) % alignment
    return raw[skip:skip + n]


class DenseLayout(C.Structure):
    """OrnithDenseG256Layout, kernels/dense_n32/dense_g256_api.h:11-13."""
    _fields_ = [(n, C.c_size_t) for n in
                ('workspace_bytes', 'transformed', 'low', 'high', 'scales', 'sums', 'projection')]


def ref_dense(x_bits, codes, meta, N, K, entry='ornith_dense_g256_launch', geometry=2, Mcap=None):
    """A dense launch of the compiled reference (N16 bank for ornith_dense_g256_launch,
    N32 bank for ornith_dense_g256_launch_n32).  Returns (out, fp32 projection, flags, status)."""
    L = ref_lib('dense_n32')
    x_bits = _c(x_bits, np.uint16).reshape(-1, K)
    M = x_bits.shape[0]
    Mcap = M if Mcap is None else Mcap
    layout = DenseLayout()
    L.ornith_dense_g256_get_layout.restype = C.c_int
    st = L.ornith_dense_g256_get_layout(C.c_int(Mcap), C.c_int(N), C.c_int(K), C.c_int(8), C.byref(layout))
    if st:
        return None, None, None, st
    ws = _aligned_bytes(max(layout.workspace_bytes, 256))
    out = np.zeros((max(M, 1), N), np.uint16)
    flags = np.zeros(1, np.uint32)
    fn = getattr(L, entry)
    fn.restype = C.c_int
    st = fn(_p(x_bits), _p(_c(codes, np.uint32)), _p(_c(meta, np.uint32)), _p(ws), C.c_size_t(ws.size),
            _p(out), _p(flags), C.c_int(M), C.c_int(Mcap), C.c_int(N), C.c_int(K), C.c_int(8), C.c_int(128),
            C.c_int(geometry), None)
    if st:
        return None, None, int(flags[0]), st
    proj = ws[layout.projection:layout.projection + M * N * 4].view(np.float32).reshape(M, N).copy()
    return out[:M], proj, int(flags[0]), st


def ref_dense_prepare_bf16(x_bits, codes16, meta16, N, K):
    L = ref_lib('dense_n32')
    x_bits = _c(x_bits, np.uint16).reshape(-1, K)
    M = x_bits.shape[0]
    xt = np.zeros((M, K), np.uint16)
    w = np.zeros((N, K), np.uint16)
    flags = np.zeros(1, np.uint32)
    fn = L.ornith_dense_g256_prepare_bf16
    fn.restype = C.c_int
    st = fn(_p(x_bits), _p(_c(codes16, np.uint32)), _p(_c(meta16, np.uint32)), _p(xt), _p(w), _p(flags),
            C.c_int(M), C.c_int(N), C.c_int(K), None)
    return xt, w, int(flags[0]), st


# ---------------------------------------------------------------------------
# W8 LM head (kernels/head/, head_i8_tile_api.h:21-41)
# ---------------------------------------------------------------------------

HEAD_K, HEAD_GROUPS = 2048, 16


def head_project(x_bits, words, scales_bits, N, group_dots=False):
    """x bf16 bits [M,2048] by the int8 head bank (words uint32 [N/16,128,4,16],
    scales fp16 bits [N,16]).  Returns (out bf16 bits, fp32 values, flags[, dots])."""
    x_bits = _c(x_bits, np.uint16).reshape(-1, HEAD_K)
    M = x_bits.shape[0]
    out = np.zeros((M, N), np.uint16)
    diag = np.zeros((M, N), np.float32)
    dots = np.zeros((M, N, HEAD_GROUPS), np.int32) if group_dots else None
    flags = np.zeros(1, np.uint32)
    lib().orc_head_project(_p(x_bits), C.c_int(M), C.c_int(N), _p(_c(words, np.uint32)),
                           _p(_c(scales_bits, np.uint16)), _p(out), _p(diag), _p(dots) if dots is not None else None,
                           _p(flags))
    res = (out, diag, int(flags[0]))
    return res + (dots,) if group_dots else res


class HeadLayout(C.Structure):
    """OrnithHeadI8Layout, kernels/head/head_i8_tile_api.h:13-15."""
    _fields_ = [(n, C.c_size_t) for n in
                ('workspace_bytes', 'transformed', 'activation_words', 'activation_scales', 'projection')]


def ref_head(x_bits, words, scales_bits, N, geometry=2, Mcap=None, group_dots=False):
    """ornith_head_i8_tile_launch of the compiled reference.
    Returns (out, fp32 projection, flags, status[, dots])."""
    L = ref_lib('head_i8')
    x_bits = _c(x_bits, np.uint16).reshape(-1, HEAD_K)
    M = x_bits.shape[0]
    Mcap = M if Mcap is None else Mcap
    layout = HeadLayout()
    L.ornith_head_i8_tile_get_layout.restype = C.c_int
    st = L.ornith_head_i8_tile_get_layout(C.c_int(Mcap), C.c_int(N), C.byref(layout))
    if st:
        return (None, None, None, st) + ((None,) if group_dots else ())
    ws = _aligned_bytes(max(layout.workspace_bytes, 256))
    out = np.zeros((max(M, 1), N), np.uint16)
    dots = np.zeros((max(M, 1), N, HEAD_GROUPS), np.int32) if group_dots else None
    flags = np.zeros(1, np.uint32)
    fn = L.ornith_head_i8_tile_launch
    fn.restype = C.c_int
    st = fn(_p(x_bits), _p(_c(words, np.uint32)), _p(_c(scales_bits, np.uint16)), _p(ws), C.c_size_t(ws.size),
            _p(out), _p(dots) if group_dots else None, C.c_size_t(dots.nbytes if group_dots else 0), _p(flags),
            C.c_int(M), C.c_int(Mcap), C.c_int(N), C.c_int(geometry), None)
    proj = None
    if st == 0:
        proj = ws[layout.projection:layout.projection + M * N * 4].view(np.float32).reshape(M, N).copy()
    res = (out[:M], proj, int(flags[0]), st)
    return res + (dots[:M] if group_dots else None,) if group_dots else res


def _bf16_bits(a):
    b = np.ascontiguousarray(a, dtype=np.float32).view(np.uint32)
    nan = (b & 0x7FFFFFFF) > 0x7F800000
    r = ((b + 0x7FFF + ((b >> 16) & 1)) >> 16).astype(np.uint16)
    return np.where(nan, ((b >> 16) | 0x40).astype(np.uint16), r)


def _bf16_f32(bits):
    return (np.ascontiguousarray(bits, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def shared_dense(x_bits, sgate_codes, sgate_meta, sdown_codes, sdown_meta, gate_w_bits):
    """The shared expert in the reference's dense decode form
    (plugin-site/ornith_g256/iu4_correctness/shared_kernel.py:33-62): the two
    dense A8 projections restated above (dense_g256_consumer.cpp), vLLM's
    silu_and_mul (silu in fp32 rounded to bf16, times up rounded to bf16) and
    bf16(sigmoid(bf16(fp32 sum x*w))) * down.  The elementwise functions and the
    logit sum are not pinned by the reference (third-party code, unspecified
    order): numpy's float32 exp and a double sum stand in for them, so callers
    compare within a tolerance.  Banks in N32 storage with one expert.
    Returns (out bf16 bits [M, 2048], gate/up flags, down flags)."""
    x_bits = _c(x_bits, np.uint16).reshape(-1, H)
    gu, _, gate_flags = dense_project(x_bits, np.asarray(sgate_codes).reshape(-1), np.asarray(sgate_meta).reshape(-1),
                                      2 * I, H, 32)
    g, u = _bf16_f32(gu[:, :I]), _bf16_f32(gu[:, I:])
    with np.errstate(over='ignore'):
        silu = _bf16_bits(g / (np.float32(1) + np.exp(-g)))
    act = _bf16_bits(_bf16_f32(silu) * u)
    down, _, down_flags = dense_project(act, np.asarray(sdown_codes).reshape(-1), np.asarray(sdown_meta).reshape(-1),
                                        H, I, 32)
    logit = _bf16_bits((_bf16_f32(x_bits).astype(np.float64) @ _bf16_f32(gate_w_bits).astype(np.float64))
                       .astype(np.float32))
    with np.errstate(over='ignore'):
        sig = _bf16_bits(np.float32(1) / (np.float32(1) + np.exp(-_bf16_f32(logit))))
    out = _bf16_bits(_bf16_f32(sig)[:, None] * _bf16_f32(down))
    return out, gate_flags, down_flags
