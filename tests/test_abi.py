"""CPU: the C-ABI library loads, exports every declared symbol, and validates
arguments on the host (these calls return before any CUDA work)."""
import ctypes as C
import re
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
INVALID = 1  # cudaErrorInvalidValue


def declared_symbols():
    names = []
    for h in (ROOT / 'include').glob('*.h'):
        names += re.findall(r'ORNITH_MOE_B200_EXPORT\s+[\w\s\*]+?\b(\w+)\s*\(', h.read_text())
    return names


def test_exports_every_declared_symbol(native):
    lib = native.lib()
    names = declared_symbols()
    assert len(names) >= 12
    for n in names:
        assert hasattr(lib, n), n
    assert set(native.SIGNATURES) >= set(names)


def test_markers(native):
    lib = native.lib()
    assert lib.ornith_routed_storage_n32() == 32
    assert lib.ornith_routed_prefill_output_tile() == 32
    assert lib.ornith_moe_b200_abi_version() == 1


def test_layout_bounds(native):
    lib = native.lib()
    layout = native.RoutedLayout()
    assert lib.ornith_routed_direct_get_layout(-1, C.byref(layout)) == INVALID
    assert lib.ornith_routed_direct_get_layout(8193, C.byref(layout)) == INVALID
    assert lib.ornith_routed_direct_get_layout(8192, None) == INVALID
    assert lib.ornith_routed_direct_get_layout(8192, C.byref(layout)) == 0
    big = layout.workspace_bytes
    assert lib.ornith_routed_direct_get_layout(16, C.byref(layout)) == 0
    assert 0 < layout.workspace_bytes < big
    for f in ('gate_low', 'gate_scales', 'gate_sums', 'middle', 'down_low', 'route_out', 'final_f32'):
        off = getattr(layout, f)
        assert off % 256 == 0 and off < layout.workspace_bytes
    for f in ('gate_x', 'gate_high', 'gate_y', 'down_x', 'down_high'):
        assert getattr(layout, f) == 2 ** 64 - 1
    assert lib.ornith_routed_shared_get_layout(17, C.byref(layout)) == INVALID
    assert lib.ornith_routed_shared_get_layout(16, C.byref(layout)) == 0
    n = C.c_size_t()
    assert lib.ornith_moe_b200_get_layout(8193, C.byref(n)) == INVALID
    assert lib.ornith_moe_b200_get_layout(4, C.byref(n)) == 0 and n.value > 0


@pytest.mark.parametrize('symbol', ['ornith_routed_direct_launch', 'ornith_routed_direct_launch_a4',
                                    'ornith_routed_direct_launch_a4_prefill'])
def test_launch_validation_without_device_work(native, symbol):
    lib = native.lib()
    fn = getattr(lib, symbol)
    nb = native.get_layout(4).workspace_bytes
    fake = C.c_void_p(1 << 20)  # never dereferenced: every case returns before any CUDA call
    args = [fake] * 8
    # T == 0: success without touching pointers (even null ones)
    assert fn(*([None] * 8), nb, None, None, 0, 4, None) == 0
    assert fn(*args, nb, fake, fake, 5, 4, None) == INVALID      # T > Tcap
    assert fn(*args, nb, fake, fake, -1, 4, None) == INVALID     # T < 0
    assert fn(*args, nb, fake, fake, 1, 8193, None) == INVALID   # Tcap too large
    assert fn(*args, nb - 1, fake, fake, 1, 4, None) == INVALID  # workspace too small
    nulls = [fake] * 8
    nulls[3] = None                                              # null gate codes
    assert fn(*nulls, nb, fake, fake, 1, 4, None) == INVALID
    odd = [C.c_void_p((1 << 20) + 4)] + [fake] * 7               # misaligned input
    assert fn(*odd, nb, fake, fake, 1, 4, None) == INVALID


def test_shared_and_logits_validation(native):
    lib = native.lib()
    fake = C.c_void_p(1 << 20)
    nb = native.get_layout(16).workspace_bytes
    assert lib.ornith_routed_direct_launch_shared_tables(*([fake] * 15), nb, fake, fake, fake, 17, 17, None) == INVALID
    assert lib.ornith_routed_direct_launch_shared_tables(*([None] * 15), nb, None, None, None, 0, 16, None) == 0
    n = C.c_size_t()
    lib.ornith_moe_b200_get_layout(128, C.byref(n))
    # act_bits must be 0, 4 or 8
    assert lib.ornith_moe_b200_launch_from_logits(*([fake] * 14), n.value, fake, fake, fake, 1, 128, 5, None) == INVALID
    # shared expert with A4 is rejected
    assert lib.ornith_moe_b200_launch_from_logits(*([fake] * 14), n.value, fake, fake, fake, 100, 128, 0, None) == INVALID
    assert lib.ornith_moe_b200_route_topk(fake, 8193, fake, fake, fake, None) == INVALID
    assert lib.ornith_moe_b200_route_topk(None, 0, None, None, None, None) == 0
    assert lib.ornith_moe_b200_repack_n16_to_n32(fake, fake, fake, fake, 1, 48, 256, None) == INVALID
    assert lib.ornith_moe_b200_repack_n16_to_n32(fake, fake, fake, fake, 1, 64, 256, None) == INVALID  # overlap


def test_operators_fail_loudly_without_library(native, monkeypatch, tmp_path):
    monkeypatch.setattr(native, '_lib', None)
    monkeypatch.setattr(native, 'LIB_PATH', tmp_path / 'missing.so')
    with pytest.raises(RuntimeError, match='no CPU fallback'):
        native.lib()


def test_variant_library_is_selected_by_environment(tmp_path):
    """ORNITH_MOE_B200_LIB points the binding at another build; a missing one
    fails loudly instead of falling back."""
    import subprocess
    import sys
    code = ('import sys; sys.path.insert(0, %r); import __graft_entry__ as g; g.load_package(); '
            'from ornith_b200 import native; print(native.LIB_PATH); native.lib()') % str(ROOT)
    env = dict(__import__('os').environ, ORNITH_MOE_B200_LIB=str(tmp_path / 'variant.so'))
    out = subprocess.run([sys.executable, '-c', code], env=env, capture_output=True, text=True, timeout=120)
    assert out.returncode != 0 and 'no CPU fallback' in out.stderr
    assert str(tmp_path / 'variant.so') in out.stdout


def test_phase_plan_of_mixed_batches(native):
    """Mixed prefill/decode batches (the plugin's phase dispatch): the
    configured segments, then any rows past them as prefill; an unsegmented
    batch when no segments are set or the batch is shorter than they cover."""
    try:
        native.set_phase_segments(())
        assert native._phase_plan(40) is None
        native.set_phase_segments([(0, 8, False), (8, 24, True)])
        assert native._phase_plan(20) is None
        assert native._phase_plan(24) == [(0, 8, False), (8, 24, True)]
        assert native._phase_plan(30) == [(0, 8, False), (8, 24, True), (24, 30, True)]
    finally:
        native.set_phase_segments(())


def _routed_fn(lib, name, n_ptrs):
    fn = getattr(lib, name)
    fn.restype = C.c_int
    fn.argtypes = [C.c_void_p] * n_ptrs + [C.c_size_t] + [C.c_void_p] * (3 if n_ptrs == 15 else 2) + \
        [C.c_int, C.c_int, C.c_void_p]
    return fn


def test_routed_reference_status_codes_match_ours(native, O):
    """Where the compiled reference (routed_storage_n32_consumer.cpp:309-324,
    :383-386) answers without device work, this library gives the same
    status: layout capacities, T outside [0, Tcap], a short workspace, T == 0
    with null pointers, and each of the ten pointers null."""
    if not O.reference_available('routed_storage_n32'):
        pytest.skip('oracle/_ref/libref_routed_storage_n32.so not built')
    ref = C.CDLL(str(O.REF_DIR / 'libref_routed_storage_n32.so'))   # own handle: own argtypes
    ours = native.lib()
    for get in ('ornith_routed_direct_get_layout', 'ornith_routed_shared_get_layout'):
        f_ref, f_ours = getattr(ref, get), getattr(ours, get)
        f_ref.restype = C.c_int
        for tcap in (-1, 0, 1, 8, 9, 16, 17, 64, 8192, 8193):
            a, b = native.RoutedLayout(), native.RoutedLayout()
            assert f_ref(tcap, C.byref(a)) == f_ours(tcap, C.byref(b)), (get, tcap)
        assert f_ref(4, None) == f_ours(4, None) == INVALID
    big = 1 << 40                      # a size only; never dereferenced
    fake = 1 << 20
    for name in ('ornith_routed_direct_launch', 'ornith_routed_direct_launch_a4',
                 'ornith_routed_direct_launch_a4_prefill'):
        f_ref, f_ours = _routed_fn(ref, name, 8), _routed_fn(ours, name, 8)
        need = native.get_layout(64).workspace_bytes
        cases = [([None] * 8, big, None, None, 0, 64),          # T == 0: success before any pointer check
                 ([fake] * 8, big, fake, fake, 65, 64),          # T > Tcap
                 ([fake] * 8, big, fake, fake, -1, 64),          # T < 0
                 ([fake] * 8, big, fake, fake, 1, 8193),         # Tcap too large
                 ([fake] * 8, big, fake, fake, 1, -1)]           # Tcap negative
        for i in range(10):                                      # each pointer null in turn
            ptrs, out, flags = [fake] * 8, fake, fake
            if i < 8:
                ptrs[i] = None
            elif i == 8:
                out = None
            else:
                flags = None
            cases.append((ptrs, big, out, flags, 3, 64))
        for ptrs, nbytes, out, flags, T, tcap in cases:
            want = f_ref(*ptrs, nbytes, out, flags, T, tcap, None)
            assert want in (0, INVALID), (name, T, tcap, want)
            assert f_ours(*ptrs, nbytes, out, flags, T, tcap, None) == want, (name, T, tcap)
        # a workspace one byte short of each library's own layout
        ref_need = native.RoutedLayout()
        getattr(ref, 'ornith_routed_direct_get_layout')(64, C.byref(ref_need))
        assert f_ref(*[fake] * 8, ref_need.workspace_bytes - 1, fake, fake, 1, 64, None) == INVALID
        assert f_ours(*[fake] * 8, need - 1, fake, fake, 1, 64, None) == INVALID
    f_ref = _routed_fn(ref, 'ornith_routed_direct_launch_shared_tables', 15)
    f_ours = _routed_fn(ours, 'ornith_routed_direct_launch_shared_tables', 15)
    # the reference's shared entry checks no pointer, so only the scalar cases
    for T, tcap in ((0, 16), (17, 16), (-1, 16), (1, 17), (1, -1)):
        ptrs = [None] * 15 if T == 0 else [fake] * 15
        want = f_ref(*ptrs, big, fake, fake, fake, T, tcap, None)
        assert f_ours(*ptrs, big, fake, fake, fake, T, tcap, None) == want, (T, tcap)


def test_debug_bounds_library_exports_every_declared_symbol(native):
    """The debug-bounds build (-DORNITH_DEBUG_BOUNDS=1) is a drop-in copy of the
    library: same symbols, same signatures, loadable through native.load."""
    path = native.HERE / 'libornith_moe_b200_debug.so'
    if not path.exists():
        pytest.skip(f'{path} not built (__graft_entry__.build() makes it)')
    dbg = native.load(path)
    for n in declared_symbols():
        assert hasattr(dbg, n), n
    assert dbg.ornith_moe_b200_abi_version() == native.lib().ornith_moe_b200_abi_version()
