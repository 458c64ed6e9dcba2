"""GPU: the debug-bounds build (-DORNITH_DEBUG_BOUNDS=1, built next to the
default library by __graft_entry__.build()) gives the default build's
outputs and flags bit for bit, and its bounds checks never fire (flag 128),
on every layer path: decode latency and throughput modes, the tensor-core
prefill and the multi-kernel path, A8 and A4, with padding and invalid ids.
The checks stand in for a device sanitizer: an index outside its buffer
would raise flag 128 and be redirected instead of faulting."""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu
DEV = torch.device('cuda:0')
DEBUG_BOUNDS = 128


def _run(handle, native, symbol, x, w, ids, bank, T):
    ws = torch.empty(native.get_layout(T).workspace_bytes, dtype=torch.uint8, device=DEV)
    out = torch.empty((T, 2048), dtype=torch.bfloat16, device=DEV)
    flags = torch.zeros(1, dtype=torch.int32, device=DEV)
    native.check(getattr(handle, symbol)(*[native.ptr(t) for t in (x, w, ids, *bank, ws)], ws.numel(),
                                         native.ptr(out), native.ptr(flags), T, T, native.stream(x)), symbol)
    torch.cuda.synchronize()
    return out.view(torch.int16).cpu(), int(flags.item())


@pytest.mark.parametrize('path', ['default', 'generic'])
@pytest.mark.parametrize('T', [1, 5, 32, 33, 200])
def test_debug_bounds_build_matches_default(native, layer1, S, T, path, monkeypatch):
    debug_lib = native.HERE / 'libornith_moe_b200_debug.so'
    if not debug_lib.exists():
        pytest.fail(f'{debug_lib} was not built (__graft_entry__.build() makes it)')
    if path == 'generic':
        monkeypatch.setenv('ORNITH_MOE_B200_PATH', 'generic')   # read by both libraries at each call
    dbg = native.load(debug_lib)
    rng = np.random.default_rng(900 + T)
    x_np = S.make_tokens(rng, T)
    w_np, ids_np = S.random_routes(rng, T, pad_fraction=0.2)
    ids_np[0, 3] = 300                      # invalid id (flag 4 in both builds)
    x = torch.from_numpy(x_np.view(np.int16)).to(DEV).view(torch.bfloat16)
    w = torch.from_numpy(w_np).to(DEV)
    ids = torch.from_numpy(ids_np).to(DEV)
    bank = [torch.from_numpy(np.ascontiguousarray(b).view(np.int32)).to(DEV)
            for b in (layer1.gate_codes, layer1.gate_meta, layer1.down_codes, layer1.down_meta)]
    for symbol in ('ornith_routed_direct_launch', 'ornith_routed_direct_launch_a4'):
        ref, ref_flags = _run(native.lib(), native, symbol, x, w, ids, bank, T)
        got, got_flags = _run(dbg, native, symbol, x, w, ids, bank, T)
        assert not got_flags & DEBUG_BOUNDS, (symbol, got_flags)
        assert got_flags == ref_flags, (symbol, got_flags, ref_flags)
        assert torch.equal(got, ref), symbol
