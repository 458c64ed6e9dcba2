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
