"""CPU: the oracle against the golden vectors and known-answer checks."""
import math
from pathlib import Path

import numpy as np


def test_shared_tables_match_reference_receipt(tables):
    # sha256 of native/shared_math_reference.safetensors as recorded in
    # native/shared_math_reference.json:2 of the reference.
    assert str(tables['source_sha256']) == '11552ec53b62b229d0ab42b4e865d0175724cd51c4eef01c05e66e930f27d2eb'
    assert tables['silu_fp32'].shape == (65536,) and tables['silu_fp32'].dtype == np.float32
    assert tables['sigmoid_bf16'].shape == (65536,) and tables['sigmoid_bf16'].dtype == np.uint16


def test_golden_layer_regenerates(golden, layer1, make_golden):
    banks = (layer1.gate_codes, layer1.gate_meta, layer1.down_codes, layer1.down_meta,
             layer1.sgate_codes, layer1.sgate_meta, layer1.sdown_codes, layer1.sdown_meta, layer1.shared_gate_w)
    assert make_golden.digest(*banks) == str(golden['layer_sha256'])



def test_oracle_matches_reference_outputs(golden, layer1, make_golden, S, O):
    """Every golden case: the C restatement reproduces the compiled reference bit for bit."""
    banks = (layer1.gate_codes, layer1.gate_meta, layer1.down_codes, layer1.down_meta)
    for name, _, seed, T, pad, hot, entry, special in make_golden.CASES:
        x, w, ids = make_golden.make_case(S, layer1, seed, T, pad, hot, special)
        assert make_golden.digest(x, w, ids) == str(golden[f'{name}/inputs_sha256']), name
        a8 = entry == 'ornith_routed_direct_launch' or (entry.endswith('_a4_prefill') and T <= 64)
        out, f32, flags = O.routed_layer(x, w, ids, *banks, a8=a8)
        np.testing.assert_array_equal(out, golden[f'{name}/out'], err_msg=name)
        assert flags == int(golden[f'{name}/flags']), name
        if f'{name}/final_f32' in golden:
            np.testing.assert_array_equal(f32.view(np.uint32), golden[f'{name}/final_f32'].view(np.uint32))


def test_oracle_shared_slot_matches_reference(golden, layer1, make_golden, S, O, tables):
    banks = (layer1.gate_codes, layer1.gate_meta, layer1.down_codes, layer1.down_meta)
    sbanks = (layer1.sgate_codes, layer1.sgate_meta, layer1.sdown_codes, layer1.sdown_meta)
    for name, seed, T in (('shared_t1', 21, 1), ('shared_t7', 22, 7), ('shared_t16', 23, 16)):
        x, w, ids = make_golden.make_case(S, layer1, seed, T, 0.1, 0, '')
        logit = S.f32_to_bf16_bits(np.random.default_rng(seed + 100).standard_normal(T).astype(np.float32))
        out, shared, _, flags = O.routed_layer_shared(x, w, ids, *banks, *sbanks, logit,
                                                      tables['silu_fp32'], tables['sigmoid_bf16'])
        np.testing.assert_array_equal(out, golden[f'{name}/out'])
        np.testing.assert_array_equal(shared, golden[f'{name}/shared_out'])
        assert flags == int(golden[f'{name}/flags'])


def test_config1_golden(golden, S, O, make_golden):
    x, router, l1 = S.config1(0)
    banks = (l1.gate_codes, l1.gate_meta, l1.down_codes, l1.down_meta)
    assert make_golden.digest(*banks, l1.sgate_codes, l1.sgate_meta, l1.sdown_codes, l1.sdown_meta,
                              l1.shared_gate_w) == str(golden['config1/layer_sha256'])
    logits = O.router_logits(x, router)
    np.testing.assert_array_equal(logits, golden['config1/logits'])
    w, ids = O.route_topk(logits)
    np.testing.assert_array_equal(ids, golden['config1/ids'])
    np.testing.assert_array_equal(w, golden['config1/weights'])
    for key, a8 in (('a8', True), ('a4', False)):
        out, _, flags = O.routed_layer(x, w, ids, *banks, a8=a8)
        np.testing.assert_array_equal(out, golden[f'config1/out_{key}'])
        assert flags == int(golden[f'config1/flags_{key}'])


def test_bf16_rne_known_answers(O):
    L = O.lib()
    assert L.orc_bf16_rne(1.0) == 0x3F80
    assert L.orc_bf16_rne(float(np.float32(1.0) + np.float32(2 ** -8))) == 0x3F80   # tie -> even
    assert L.orc_bf16_rne(float(np.float32(1.0) + np.float32(3 * 2 ** -8))) == 0x3F82  # tie -> even (up)
    assert L.orc_bf16_rne(float('inf')) == 0x7F80
    assert L.orc_bf16_rne(float('nan')) & 0x7FC0 == 0x7FC0


def test_half_conversion_matches_numpy(O):
    L = O.lib()
    rng = np.random.default_rng(5)
    vals = np.concatenate([rng.standard_normal(2000).astype(np.float32) * 10 ** rng.uniform(-9, 5, 2000).astype(np.float32),
                           np.array([0.0, -0.0, 65504.0, 65519.9, 65520.0, 2 ** -24, 2 ** -25, 3 * 2 ** -26, 6.1e-5], np.float32)])
    for v in vals:
        assert L.orc_f32_to_half_rne(float(v)) == np.float32(v).astype(np.float16).view(np.uint16), v
    for h in range(0, 65536, 7):
        f = np.uint16(h).view(np.float16).astype(np.float32)
        got = L.orc_half_to_f32(h)
        assert (math.isnan(got) and np.isnan(f)) or np.float32(got) == f


def test_portable_exp_accuracy(O):
    L = O.lib()
    for x in np.linspace(-80, 80, 4001, dtype=np.float32):
        got = L.orc_portable_exp(float(x))
        assert abs(got - math.exp(float(x))) <= 4e-7 * math.exp(float(x)), x
    assert L.orc_portable_exp(-104.0) == 0.0 and math.isinf(L.orc_portable_exp(89.0))


def test_wht128_is_scaled_hadamard(O):
    rng = np.random.default_rng(6)
    v = rng.standard_normal(128).astype(np.float32)
    H = np.array([[1.0]])
    for _ in range(7):
        H = np.block([[H, H], [H, -H]])
    expect = (H @ v.astype(np.float64)) / math.sqrt(128)
    np.testing.assert_allclose(O.wht128(v), expect, rtol=1e-5, atol=1e-5)


def test_quantize_known_answer(O):
    # one group: absmax 127 -> scale fp16(1.0); values round half to even.
    y = np.zeros((1, 256), np.float32)
    y[0, :6] = [127.0, -127.0, 2.5, 3.5, -0.5, 300.0 / 300.0]
    q, scales, sums, flags = O.quantize_rows(y, a8=True)
    assert scales[0, 0] == np.float16(1.0).view(np.uint16)
    assert list(q[0, :6]) == [127, -127, 2, 4, 0, 1] and sums[0, 0] == 7 and flags == 0
    z = np.zeros((1, 256), np.float32)
    q, scales, sums, flags = O.quantize_rows(z, a8=True)
    assert scales[0, 0] == np.float16(1.0).view(np.uint16) and not q.any() and flags == 0
    bad = np.zeros((1, 256), np.float32)
    bad[0, 3] = np.inf
    q, scales, sums, flags = O.quantize_rows(bad, a8=False)
    assert flags == 2 and not q.any()


def test_tiny_projection_hand_checked(O, S):
    """One expert, one route, hand-computable weights: code 1 everywhere, scale 1, offset -8."""
    E = S.E
    gc = np.zeros((E, 32, 8, 32, 32), np.uint32)
    gm = np.zeros((E, 32, 8, 32), np.uint32)
    dc = np.zeros((E, 64, 2, 32, 32), np.uint32)
    dm = np.zeros((E, 64, 2, 32), np.uint32)
    one = np.float16(1.0).view(np.uint16).astype(np.uint32)
    neg8 = np.float16(-8.0).view(np.uint16).astype(np.uint32)
    gc[3] = 0x11111111
    gm[3] = one | (neg8 << 16)
    dc[3] = 0x11111111
    dm[3] = one | (neg8 << 16)
    x = np.zeros((1, 2048), np.uint16)     # zero input -> every projection is 0
    w = np.zeros((1, 8), np.float32); w[0, 0] = 1.0
    ids = -np.ones((1, 8), np.int32); ids[0, 0] = 3
    out, f32, flags = O.routed_layer(x, w, ids, gc, gm, dc, dm)
    assert flags == 0 and not f32.any()
    # weight = 1*1 - 8 = -7 for every element; x = e_0 (bf16 1.0 at k=0) -> H128 spreads 1/sqrt(128).
    x[0, 0] = 0x3F80
    out, f32, flags = O.routed_layer(x, w, ids, gc, gm, dc, dm)
    ref = O.fp32_reference_layer(x, w, ids, gc, gm, dc, dm)
    assert flags == 0
    np.testing.assert_allclose(f32, ref, rtol=2e-2, atol=1e-3)


def test_route_topk_semantics(O):
    rng = np.random.default_rng(7)
    logits = rng.standard_normal((64, 256)).astype(np.float32)
    logits[0, 10] = logits[0, 20] = 9.0   # tie: lower index first
    logits[1, :] = -np.inf
    logits[1, 5] = 1.0                    # one finite logit
    w, ids = O.route_topk(logits)
    assert ids[0, 0] == 10 and ids[0, 1] == 20
    assert ids[1, 0] == 5 and (ids[1, 1:] == -1).all() and w[1, 0] == 1.0 and not w[1, 1:].any()
    for t in range(2, 64):
        order = np.argsort(-logits[t], kind='stable')[:8]
        np.testing.assert_array_equal(ids[t], order)
        top = logits[t, order].astype(np.float64)
        p = np.exp(top - top[0]); p /= p.sum()
        np.testing.assert_allclose(w[t], p, rtol=2e-6)


def test_repack_n16_roundtrip(O):
    rng = np.random.default_rng(8)
    N, K = 64, 512
    c32 = rng.integers(0, 2 ** 32, (2, N // 32, K // 256, 32, 32), dtype=np.uint32)
    m32 = rng.integers(0, 2 ** 32, (2, N // 32, K // 256, 32), dtype=np.uint32)
    # inverse of method.py:142-147
    c16 = c32.reshape(2, N // 32, K // 256, 32, 2, 16).transpose(0, 1, 4, 2, 3, 5).reshape(2, N // 16, K // 256, 32, 16)
    m16 = m32.reshape(2, N // 32, K // 256, 2, 16).transpose(0, 1, 3, 2, 4).reshape(2, N // 16, K // 256, 16)
    r_c, r_m = O.repack_n16_to_n32(np.ascontiguousarray(c16), np.ascontiguousarray(m16), N, K)
    np.testing.assert_array_equal(r_c, c32)
    np.testing.assert_array_equal(r_m, m32)


def test_oracle_matches_reference_digests_at_larger_batches(layer1, make_golden, S, O):
    """T = 32 (A8), 64 (A4) and 1120 (A4 prefill): the oracle's outputs hash to
    the digests of the compiled reference's outputs (tests/golden/
    routed_reference_digests.npz; the outputs themselves are too big to keep)."""
    digests = np.load(Path(__file__).resolve().parent / 'golden' / 'routed_reference_digests.npz')
    banks = (layer1.gate_codes, layer1.gate_meta, layer1.down_codes, layer1.down_meta)
    for name, seed, T, pad, entry in make_golden.DIGEST_CASES:
        x, w, ids = make_golden.make_case(S, layer1, seed, T, pad, 0, '')
        assert make_golden.digest(x, w, ids) == str(digests[f'{name}/inputs_sha256']), name
        a8 = entry == 'ornith_routed_direct_launch' or (entry.endswith('_a4_prefill') and T <= 64)
        out, _, flags = O.routed_layer(x, w, ids, *banks, a8=a8)
        assert make_golden.digest(out) == str(digests[f'{name}/out_sha256']), name
        assert flags == int(digests[f'{name}/flags']), name


def test_oracle_matches_reference_digests_with_hot_experts(layer1, make_golden, S, O):
    """T = 300 with experts that hold 127, 128, 129, 256, 257 and 1,100 routes
    (the reference's grouped projection splits them into 16-row jobs): the
    oracle's outputs hash to the compiled reference's, A8 and A4."""
    digests = np.load(Path(__file__).resolve().parent / 'golden' / 'routed_reference_digests.npz')
    banks = (layer1.gate_codes, layer1.gate_meta, layer1.down_codes, layer1.down_meta)
    for name, seed, T, pad, entry, counts in make_golden.HOT_DIGEST_CASES:
        x, w, ids = make_golden.make_hot_case(S, seed, T, pad, counts)
        assert make_golden.digest(x, w, ids) == str(digests[f'{name}/inputs_sha256']), name
        for e, c in counts.items():
            assert int((ids == e).sum()) == c
        out, _, flags = O.routed_layer(x, w, ids, *banks, a8=entry == 'ornith_routed_direct_launch')
        assert make_golden.digest(out) == str(digests[f'{name}/out_sha256']), name
        assert flags == int(digests[f'{name}/flags']), name
