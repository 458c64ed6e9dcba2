"""GPU: a routed layer loaded the way the reference plugin loads it (N16
checkpoint banks through the strict loader, one N32 reorder on the device)
and run through G256MoEMethod.apply, bit for bit against the oracle."""
import importlib

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def n32_to_n16(codes32, meta32):
    """Checkpoint (N16) form of N32 banks: N16 tile 2t+h, lane l is column
    16h+l of N32 tile t (the inverse of method.py:142-147)."""
    e, t, g = codes32.shape[:3]
    codes16 = codes32.reshape(e, t, g, 32, 2, 16).transpose(0, 1, 4, 2, 3, 5).reshape(e, 2 * t, g, 32, 16)
    meta16 = meta32.reshape(e, t, g, 2, 16).transpose(0, 1, 3, 2, 4).reshape(e, 2 * t, g, 16)
    return np.ascontiguousarray(codes16), np.ascontiguousarray(meta16)


def _u32(a):
    return torch.from_numpy(np.ascontiguousarray(a).view(np.int32)).view(torch.uint32)


@pytest.mark.parametrize('replace', [True, False])
def test_loaded_layer_matches_oracle(S, O, replace):
    M = importlib.import_module('ornith_b200.method')
    runtime_mod = importlib.import_module('ornith_b200.runtime')
    rng = np.random.default_rng(2)
    lw = S.make_layer(rng)
    g16, gm16 = n32_to_n16(lw.gate_codes, lw.gate_meta)
    d16, dm16 = n32_to_n16(lw.down_codes, lw.down_meta)
    # the inverse permutation is the oracle's repack read backwards
    rc, rm = O.repack_n16_to_n32(g16, gm16, 1024, 2048)
    assert np.array_equal(rc, lw.gate_codes) and np.array_equal(rm, lw.gate_meta)

    layer = torch.nn.Module()
    method = M.G256MoEMethod()
    method.create_weights(layer, 256, 2048, 512, torch.bfloat16, device='cuda')
    ckpt = [('routed_experts.w13_tilebank_codes', _u32(g16)), ('routed_experts.w13_tilebank_metadata', _u32(gm16)),
            ('routed_experts.w2_tilebank_codes', _u32(d16)), ('routed_experts.w2_tilebank_metadata', _u32(dm16))]
    assert len(list(layer.load_weights(iter(ckpt)))) == 4
    method.process_weights_after_loading(layer)
    size = method.prepare_n32_weights(layer, replace=replace)
    assert size == (256 * 1024 * 2048 // 2 + 256 * 1024 * 8 * 4 + 256 * 2048 * 512 // 2 + 256 * 2048 * 2 * 4)
    with pytest.raises(RuntimeError, match='prepared once'):
        method.prepare_n32_weights(layer, replace=replace)

    T = 6
    runtime = runtime_mod.Runtime(['model.layers.0.mlp.experts'], T, 'cuda')
    method.bind(runtime, 0)
    x = S.make_tokens(rng, T)
    w, ids = S.random_routes(rng, T, pad_fraction=0.15)
    dev = torch.device('cuda')
    out = method.apply(layer, torch.from_numpy(x.view(np.int16)).to(dev).view(torch.bfloat16),
                       torch.from_numpy(w).to(dev), torch.from_numpy(ids).to(dev))
    torch.cuda.synchronize()
    ref, _, ref_flags = O.routed_layer(x, w, ids, lw.gate_codes, lw.gate_meta, lw.down_codes, lw.down_meta)
    np.testing.assert_array_equal(out.view(torch.int16).cpu().numpy().view(np.uint16), ref)
    assert runtime.check_error_flags() == [ref_flags] == [0]
