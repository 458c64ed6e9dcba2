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
    with pytest.raises(RuntimeError, match='already prepared'):
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


def _fp32_reduced_gemm(fn):
    """Run fn with cuBLAS told to keep split-K reductions in fp32: by default
    torch lets bf16 GEMMs reduce partial sums in bf16, whose error the fp32
    summation bound of these checks does not cover."""
    flag = torch.backends.cuda.matmul.allow_bf16_reduced_precision_reduction
    torch.backends.cuda.matmul.allow_bf16_reduced_precision_reduction = False
    try:
        result = fn()
        torch.cuda.synchronize()
        return result
    finally:
        torch.backends.cuda.matmul.allow_bf16_reduced_precision_reduction = flag


def test_dense_linear_method_apply(S, O):
    """G256LinearMethod: packed loads, seal, apply on [..., K] rows through
    dense_out (A8 up to dense_a8_max_rows rows, bit for bit; the bf16 prefill
    path beyond, within one bf16 ulp plus an fp32 summation error bound of the
    exact product of its operands, and relative L2 <= 1e-3)."""
    M = importlib.import_module('ornith_b200.method')
    runtime_mod = importlib.import_module('ornith_b200.runtime')
    N, K = 1024, 2048
    rng = np.random.default_rng(17)
    codes, meta = S.make_dense_bank(rng, N, K)
    layer = torch.nn.Module()
    method = M.G256LinearMethod('model.layers.3.mlp.gate_up_proj')
    method.create_weights(layer, K, [N], K, N, torch.bfloat16, device='cuda')
    layer.g256_codes.weight_loader(layer.g256_codes, _u32(codes))
    layer.g256_metadata.weight_loader(layer.g256_metadata, _u32(meta))
    method.process_weights_after_loading(layer)
    runtime = runtime_mod.Runtime(['model.layers.3.mlp.gate_up_proj'], 64, 'cuda', dense_shapes=[(N, K)])
    method.bind(runtime, 0)
    dev = torch.device('cuda')
    x = S.make_rows(rng, 6, K)
    out = method.apply(layer, torch.from_numpy(x.view(np.int16)).to(dev).view(torch.bfloat16).view(2, 3, K))
    torch.cuda.synchronize()
    assert out.shape == (2, 3, N)
    ref, _, ref_flags = O.dense_project(x, codes, meta, N, K, 16)
    np.testing.assert_array_equal(out.reshape(6, N).view(torch.int16).cpu().numpy().view(np.uint16), ref)
    x = S.make_rows(rng, 40, K)   # above dense_a8_max_rows = 32: the bf16 prefill path
    out = _fp32_reduced_gemm(lambda: method.apply(layer, torch.from_numpy(x.view(np.int16)).to(dev)
                                                  .view(torch.bfloat16)))
    xt, w, _ = O.dense_prepare_bf16(x, codes, meta, N, K)
    xa, wa = S.bf16_bits_to_f32(xt).astype(np.float64), S.bf16_bits_to_f32(w).astype(np.float64)
    exact = xa @ wa.T
    magnitude = np.abs(xa) @ np.abs(wa).T   # sum of |products|: scale of the fp32 summation error
    want = S.bf16_bits_to_f32(S.f32_to_bf16_bits(exact.astype(np.float32)))
    got = S.bf16_bits_to_f32(out.view(torch.int16).cpu().numpy().view(np.uint16))
    # one bf16 ulp of the result plus an fp32 summation error bound over K terms
    assert np.all(np.abs(got - want) <= np.abs(want) * 2.0 ** -7 + magnitude * 2.0 ** -16)
    assert np.linalg.norm(got - want) <= 1e-3 * np.linalg.norm(want)
    assert runtime.check_error_flags() == [ref_flags] == [0]


def test_w8_head_method_apply_in_64_row_slices(S, O):
    """W8HeadMethod over the full vocabulary with 70 rows (slices of 64 and 6),
    sampled tiles bit for bit against the oracle."""
    M = importlib.import_module('ornith_b200.method')
    runtime_mod = importlib.import_module('ornith_b200.runtime')
    native = importlib.import_module('ornith_b200.native')
    N = native.HEAD_VOCAB
    dev = torch.device('cuda')
    layer = torch.nn.Module()
    method = M.W8HeadMethod('lm_head')
    method.create_weights(layer, 2048, [N], 2048, N, torch.bfloat16, device='cuda')
    gen = torch.Generator(device=dev).manual_seed(21)
    codes = torch.randint(-127, 128, (N // 16, 128, 4, 16, 4), dtype=torch.int8, device=dev, generator=gen)
    words = codes.view(torch.int32).view(N // 16, 128, 4, 16).view(torch.uint32)
    scales = (0.01 * torch.randn((N, 16), device=dev, generator=gen).abs()).to(torch.float16).clamp_min(2 ** -14)
    layer.head_tilebank_codes.weight_loader(layer.head_tilebank_codes, words)
    layer.head_scales.weight_loader(layer.head_scales, scales)
    method.process_weights_after_loading(layer)
    del codes, words
    runtime = runtime_mod.Runtime(['lm_head'], 64, 'cuda', head=True)
    method.bind(runtime, 0)
    x = S.make_rows(np.random.default_rng(22), 70, 2048)
    out = method.apply(layer, torch.from_numpy(x.view(np.int16)).to(dev).view(torch.bfloat16))
    torch.cuda.synchronize()
    got = out.view(torch.int16).cpu().numpy().view(np.uint16)
    w_np = layer.head_tilebank_codes.view(torch.int32).cpu().numpy().view(np.uint32)
    s_np = layer.head_scales.view(torch.int16).cpu().numpy().view(np.uint16)
    for t in (0, 9999, N // 16 - 1):
        ref, _, _ = O.head_project(x, w_np[t:t + 1], s_np[16 * t:16 * t + 16], 16)
        np.testing.assert_array_equal(got[:, 16 * t:16 * t + 16], ref)
    assert runtime.check_error_flags() == [0]
