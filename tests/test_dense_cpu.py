"""CPU: the dense G256 oracle against the reference's dense library (golden
vectors made by the compiled reference, and live calls where it is built),
plus the dense C-ABI's host-side argument validation."""
import ctypes as C

import numpy as np
import pytest

INVALID = 1  # cudaErrorInvalidValue


def _case_inputs(S, O, make_golden, name, seed, M, N, K, entry, special):
    x, codes, meta = make_golden.make_dense_case(S, seed, M, N, K, special)
    sha = make_golden.digest(x, codes, meta)
    if entry == 'n32':
        codes, meta = O.repack_n16_to_n32(codes[None], meta[None], N, K)
        codes, meta = codes[0], meta[0]
    return x, codes, meta, sha


def test_dense_oracle_matches_golden(dense_golden, make_golden, S, O):
    """Every dense golden case: the C restatement reproduces the compiled
    reference bit for bit (outputs, fp32 projections, flags)."""
    for name, seed, M, N, K, entry, geometry, special in make_golden.DENSE_CASES:
        x, codes, meta, sha = _case_inputs(S, O, make_golden, name, seed, M, N, K, entry, special)
        assert sha == str(dense_golden[f'{name}/inputs_sha256']), name
        if entry == 'prepare':
            xt, w, flags = O.dense_prepare_bf16(x, codes, meta, N, K)
            np.testing.assert_array_equal(xt, dense_golden[f'{name}/transformed'], err_msg=name)
            np.testing.assert_array_equal(w, dense_golden[f'{name}/weights'], err_msg=name)
        else:
            out, diag, flags = O.dense_project(x, codes, meta, N, K, 32 if entry == 'n32' else 16)
            np.testing.assert_array_equal(out, dense_golden[f'{name}/out'], err_msg=name)
            np.testing.assert_array_equal(diag.view(np.uint32), dense_golden[f'{name}/projection'].view(np.uint32),
                                          err_msg=name)
        assert flags == int(dense_golden[f'{name}/flags']), name


def test_dense_edge_flags_cover_every_bit(dense_golden):
    assert int(dense_golden['d_m5_edges/flags']) == 1 | 2 | 4 | 8
    assert int(dense_golden['d_prep_m5/flags']) == 1 | 8


@pytest.mark.parametrize('M,N,K,geometry', [(2, 32, 256, 0), (9, 80, 1024, 1), (4, 64, 512, 2)])
def test_dense_oracle_matches_live_reference(S, O, M, N, K, geometry):
    if not O.reference_available('dense_n32'):
        pytest.skip('oracle/_ref/libref_dense_n32.so not built')
    rng = np.random.default_rng(100 + M)
    codes, meta = S.make_dense_bank(rng, N, K)
    x = S.make_rows(rng, M, K)
    ro, rp, rf, st = O.ref_dense(x, codes, meta, N, K, geometry=geometry)
    assert st == 0
    oo, od, of = O.dense_project(x, codes, meta, N, K, 16)
    np.testing.assert_array_equal(oo, ro)
    np.testing.assert_array_equal(od.view(np.uint32), rp.view(np.uint32))
    assert of == rf


def test_dense_reference_status_codes_match_ours(S, O, native):
    """Where the compiled reference rejects a scalar argument, so does this
    library (both return before any device work)."""
    if not O.reference_available('dense_n32'):
        pytest.skip('oracle/_ref/libref_dense_n32.so not built')
    ref = O.ref_lib('dense_n32')
    ours = native.lib()
    for args in [(-1, 64, 256, 8), (8193, 64, 256, 8), (4, 0, 256, 8), (4, 40, 256, 8), (4, 12304, 256, 8),
                 (4, 248320, 2048, 8), (4, 64, 0, 8), (4, 64, 300, 8), (4, 64, 8448, 8), (4, 64, 256, 4)]:
        a = O.DenseLayout()
        b = native.DenseLayout()
        ref.ornith_dense_g256_get_layout.restype = C.c_int
        assert (ref.ornith_dense_g256_get_layout(*args, C.byref(a)) == 0) == \
            (ours.ornith_dense_g256_get_layout(*args, C.byref(b)) == 0), args


def test_dense_layout(native):
    lib = native.lib()
    layout = native.DenseLayout()
    assert lib.ornith_dense_g256_get_layout(16, 12288, 2048, 8, None) == INVALID
    assert lib.ornith_dense_g256_get_layout(16, 12288, 2048, 8, C.byref(layout)) == 0
    assert layout.transformed == layout.high == 2 ** 64 - 1
    for f in ('low', 'scales', 'sums', 'projection'):
        off = getattr(layout, f)
        assert off % 256 == 0 and off < layout.workspace_bytes
    assert layout.workspace_bytes >= 16 * 2048 + 16 * 12288 * 4
    assert lib.ornith_dense_g256_abi_version() == 1
    assert lib.ornith_dense_g256_n32_rows() == 16


@pytest.mark.parametrize('symbol', ['ornith_dense_g256_launch', 'ornith_dense_g256_launch_n32'])
def test_dense_launch_validation_without_device_work(native, symbol):
    lib = native.lib()
    fn = getattr(lib, symbol)
    N, K = 64, 512
    nb = native.dense_get_layout(8, N, K).workspace_bytes
    base = 1 << 30
    # disjoint fake buffers: input, codes, metadata, workspace, output, flags
    x, codes, meta = C.c_void_p(base), C.c_void_p(base + (1 << 24)), C.c_void_p(base + (2 << 24))
    ws, out, flags = C.c_void_p(base + (3 << 24)), C.c_void_p(base + (4 << 24)), C.c_void_p(base + (5 << 24))
    ok = [x, codes, meta, ws, nb, out, flags]
    if symbol == 'ornith_dense_g256_launch':
        # M == 0: success without touching pointers (even null ones)
        assert fn(None, None, None, None, 0, None, None, 0, 8, N, K, 8, 128, 2, None) == 0
    else:
        assert fn(*ok, 0, 8, N, K, 8, 128, 2, None) == INVALID          # the N32 entry needs M >= 1
        assert fn(*ok, 17, 32, N, K, 8, 128, 2, None) == INVALID        # at most 16 rows
        assert fn(*ok, 1, 8, 48, K, 8, 128, 2, None) == INVALID         # N a multiple of 32
        assert fn(*ok, 1, 8, N, K, 8, 128, 0, None) == INVALID          # geometry 2 only
    assert fn(*ok, 9, 8, N, K, 8, 128, 2, None) == INVALID              # M > Mcap
    assert fn(*ok, 1, 8, N, K, 4, 128, 2, None) == INVALID              # bits 8 only
    assert fn(*ok, 1, 8, N, K, 8, 64, 2, None) == INVALID               # transform 128 only
    assert fn(*ok, 1, 8, N, K, 8, 128, 3, None) == INVALID              # geometry 0..2
    assert fn(x, codes, meta, ws, nb - 1, out, flags, 1, 8, N, K, 8, 128, 2, None) == INVALID
    assert fn(None, codes, meta, ws, nb, out, flags, 1, 8, N, K, 8, 128, 2, None) == INVALID
    assert fn(C.c_void_p(base + 2), codes, meta, ws, nb, out, flags, 1, 8, N, K, 8, 128, 2, None) == INVALID
    assert fn(x, codes, meta, C.c_void_p(base + (3 << 24) + 16), nb, out, flags, 1, 8, N, K, 8, 128, 2,
              None) == INVALID                                          # workspace 256-aligned
    assert fn(x, codes, meta, ws, nb, C.c_void_p(base + (3 << 24) + 256), flags, 1, 8, N, K, 8, 128, 2,
              None) == INVALID                                          # output inside the workspace
    assert fn(x, codes, meta, ws, nb, out, C.c_void_p(base + 64), 1, 8, N, K, 8, 128, 2,
              None) == INVALID                                          # flags inside the input


def test_dense_prepare_validation_without_device_work(native):
    lib = native.lib()
    base = 1 << 30
    p = [C.c_void_p(base + (i << 24)) for i in range(6)]
    assert lib.ornith_dense_g256_prepare_bf16(*([None] * 6), 0, 64, 512, None) == 0
    assert lib.ornith_dense_g256_prepare_bf16(*p, 8193, 64, 512, None) == INVALID
    assert lib.ornith_dense_g256_prepare_bf16(*p, 4, 40, 512, None) == INVALID
    assert lib.ornith_dense_g256_prepare_bf16(*p[:3], p[0], *p[4:], 4, 64, 512, None) == INVALID  # aliasing


def test_dense_workspace_bytes_cover_both_paths(native):
    shapes = [(12288, 2048), (2048, 4096)]
    n = native.dense_workspace_bytes(64, shapes)
    for N, K in shapes:
        assert n >= native.dense_get_layout(64, N, K).workspace_bytes
        assert n >= (64 * K + N * K) * 2


def test_shared_dense_oracle_uses_the_reference_projections(layer1, S, O):
    """The shared expert's dense decode form (shared_kernel.py:33-62): with
    both projections taken from the reference's dense N32 launch compiled for
    the CPU, the oracle composition gives the same output bit for bit."""
    if not O.reference_available('dense_n32'):
        pytest.skip('oracle/_ref/libref_dense_n32.so not built')
    x = S.make_tokens(np.random.default_rng(61), 9)
    out, gf, df = O.shared_dense(x, layer1.sgate_codes, layer1.sgate_meta, layer1.sdown_codes, layer1.sdown_meta,
                                 layer1.shared_gate_w)
    entry = 'ornith_dense_g256_launch_n32'
    gu, _, rgf, st = O.ref_dense(x, layer1.sgate_codes[0], layer1.sgate_meta[0], 1024, 2048, entry=entry)
    assert st == 0
    g, u = S.bf16_bits_to_f32(gu[:, :512]), S.bf16_bits_to_f32(gu[:, 512:])
    with np.errstate(over='ignore'):
        silu = S.f32_to_bf16_bits(g / (np.float32(1) + np.exp(-g)))
    act = S.f32_to_bf16_bits(S.bf16_bits_to_f32(silu) * u)
    down, _, rdf, st = O.ref_dense(act, layer1.sdown_codes[0], layer1.sdown_meta[0], 2048, 512, entry=entry)
    assert st == 0
    logit = S.f32_to_bf16_bits((S.bf16_bits_to_f32(x).astype(np.float64)
                                @ S.bf16_bits_to_f32(layer1.shared_gate_w).astype(np.float64)).astype(np.float32))
    with np.errstate(over='ignore'):
        sig = S.f32_to_bf16_bits(np.float32(1) / (np.float32(1) + np.exp(-S.bf16_bits_to_f32(logit))))
    want = S.f32_to_bf16_bits(S.bf16_bits_to_f32(sig)[:, None] * S.bf16_bits_to_f32(down))
    np.testing.assert_array_equal(out, want)
    assert (gf, df) == (rgf, rdf) == (0, 0)
