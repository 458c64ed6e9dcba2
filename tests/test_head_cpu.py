"""CPU: the W8 head oracle against the reference's head library (golden
vectors made by the compiled reference, live calls where it is built), and
the head C-ABI's host-side argument validation."""
import ctypes as C

import numpy as np
import pytest

INVALID = 1  # cudaErrorInvalidValue


def test_head_oracle_matches_golden(head_golden, make_golden, S, O):
    for name, seed, M, N, geometry, special in make_golden.HEAD_CASES:
        x, words, scales = make_golden.make_head_case(S, seed, M, N, special)
        assert make_golden.digest(x, words, scales) == str(head_golden[f'{name}/inputs_sha256']), name
        out, diag, flags, dots = O.head_project(x, words, scales, N, group_dots=True)
        np.testing.assert_array_equal(out, head_golden[f'{name}/out'], err_msg=name)
        np.testing.assert_array_equal(diag.view(np.uint32), head_golden[f'{name}/projection'].view(np.uint32))
        if f'{name}/group_dots' in head_golden:
            np.testing.assert_array_equal(dots, head_golden[f'{name}/group_dots'], err_msg=name)
        assert flags == int(head_golden[f'{name}/flags']), name
    assert int(head_golden['h_m5_edges/flags']) == 1 | 2 | 4 | 8


@pytest.mark.parametrize('M,N,geometry', [(2, 256, 2), (7, 1024, 0), (40, 256, 0)])
def test_head_oracle_matches_live_reference(S, O, M, N, geometry):
    if not O.reference_available('head_i8'):
        pytest.skip('oracle/_ref/libref_head_i8.so not built')
    rng = np.random.default_rng(200 + M)
    words, scales = S.make_head_bank(rng, N)
    x = S.make_rows(rng, M, 2048)
    ro, rp, rf, st, rd = O.ref_head(x, words, scales, N, geometry=geometry, group_dots=True)
    assert st == 0
    oo, od, of, dd = O.head_project(x, words, scales, N, group_dots=True)
    np.testing.assert_array_equal(oo, ro)
    np.testing.assert_array_equal(od.view(np.uint32), rp.view(np.uint32))
    np.testing.assert_array_equal(dd, rd)
    assert of == rf


def test_head_layout_and_markers(native, O):
    lib = native.lib()
    layout = native.HeadLayout()
    for args in [(-1, 256), (65, 256), (4, 512), (4, 248321)]:
        assert lib.ornith_head_i8_tile_get_layout(*args, C.byref(layout)) == INVALID, args
    assert lib.ornith_head_i8_tile_get_layout(64, 248320, None) == INVALID
    assert lib.ornith_head_i8_tile_get_layout(64, 248320, C.byref(layout)) == 0
    assert layout.transformed == 2 ** 64 - 1
    assert layout.workspace_bytes >= 64 * 2048 + 64 * 248320 * 4
    for f in ('activation_words', 'activation_scales', 'projection'):
        assert getattr(layout, f) % 256 == 0
    assert lib.ornith_head_i8_tile_abi_version() == 1 and lib.ornith_head_i8_tile_shortlist() == 1
    if O.reference_available('head_i8'):
        ref = O.ref_lib('head_i8')
        ref.ornith_head_i8_tile_get_layout.restype = C.c_int
        for args in [(-1, 256), (65, 256), (4, 512), (0, 1024), (64, 65536)]:
            a = O.HeadLayout()
            assert (ref.ornith_head_i8_tile_get_layout(*args, C.byref(a)) == 0) == \
                (lib.ornith_head_i8_tile_get_layout(*args, C.byref(layout)) == 0), args


def test_head_launch_validation_without_device_work(native):
    lib = native.lib()
    fn = lib.ornith_head_i8_tile_launch
    N = 256
    nb = native.head_get_layout(8, N).workspace_bytes
    base = 1 << 30
    x, w, sc, ws, out, dots, fl = (C.c_void_p(base + (i << 24)) for i in range(7))
    dbytes = 8 * N * 16 * 4
    # M == 0: success without touching pointers (after the optional-buffer contract)
    assert fn(None, None, None, None, 0, None, None, 0, None, 0, 8, N, 2, None) == 0
    assert fn(x, w, sc, ws, nb, out, None, 0, fl, 9, 8, N, 2, None) == INVALID          # M > Mcap
    assert fn(x, w, sc, ws, nb, out, None, 0, fl, 1, 8, 512, 2, None) == INVALID        # unsupported N
    assert fn(x, w, sc, ws, nb, out, None, 0, fl, 1, 8, N, 3, None) == INVALID          # geometry
    assert fn(x, w, sc, ws, nb, out, dots, 0, fl, 1, 8, N, 2, None) == INVALID          # dots without bytes
    assert fn(x, w, sc, ws, nb, out, None, 64, fl, 1, 8, N, 2, None) == INVALID         # bytes without dots
    assert fn(x, w, sc, ws, nb, out, dots, 16, fl, 1, 8, N, 2, None) == INVALID         # dots too small
    assert fn(None, None, None, None, 0, None, dots, 0, None, 0, 8, N, 2, None) == INVALID  # checked even at M 0
    assert fn(x, w, sc, ws, nb - 1, out, None, 0, fl, 1, 8, N, 2, None) == INVALID      # workspace too small
    assert fn(C.c_void_p(base + 2), w, sc, ws, nb, out, None, 0, fl, 1, 8, N, 2, None) == INVALID
    assert fn(x, w, sc, ws, nb, C.c_void_p(base + (3 << 24) + 512), None, 0, fl, 1, 8, N, 2, None) == INVALID
    assert fn(x, w, sc, ws, nb, out, C.c_void_p(base + (4 << 24)), dbytes, fl, 1, 8, N, 2, None) == INVALID
