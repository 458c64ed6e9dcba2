"""GPU parity: the CUDA path through the C ABI against the golden vectors
(outputs of the reference's own routed source) and the CPU oracle.
Bit-exact for outputs, fp32 diagnostics, ids, routing weights and flags."""

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu
DEV = torch.device('cuda:0')


def dev(a):
    a = np.ascontiguousarray(a)
    if a.dtype == np.uint16:
        return torch.from_numpy(a.view(np.int16)).to(DEV).view(torch.bfloat16)
    if a.dtype == np.uint32:
        return torch.from_numpy(a.view(np.int32)).to(DEV).view(torch.uint32)
    return torch.from_numpy(a).to(DEV)


def host_bits(t):
    return t.view(torch.int16).cpu().numpy().view(np.uint16)


class Bank:
    def __init__(self, layer):
        self.routed = [dev(b) for b in (layer.gate_codes, layer.gate_meta, layer.down_codes, layer.down_meta)]
        self.shared = [dev(b) for b in (layer.sgate_codes, layer.sgate_meta, layer.sdown_codes, layer.sdown_meta)]
        self.np_routed = (layer.gate_codes, layer.gate_meta, layer.down_codes, layer.down_meta)
        self.np_shared = (layer.sgate_codes, layer.sgate_meta, layer.sdown_codes, layer.sdown_meta)
        self.gate_w = layer.shared_gate_w


@pytest.fixture(scope='module')
def bank1(layer1):
    return Bank(layer1)


def run_entry(native, symbol, x, w, ids, bank, Tcap=None):
    T = x.shape[0]
    Tcap = T if Tcap is None else Tcap
    ws = torch.empty(native.get_layout(Tcap).workspace_bytes, dtype=torch.uint8, device=DEV)
    out = torch.full((max(T, 1), 2048), -1, dtype=torch.int16, device=DEV).view(torch.bfloat16)
    flags = torch.zeros(1, dtype=torch.int32, device=DEV)
    fn = getattr(native.lib(), symbol)
    st = fn(*[native.ptr(t) for t in (dev(x), dev(w), dev(ids), *bank.routed, ws)], ws.numel(),
            native.ptr(out), native.ptr(flags), T, Tcap, native.stream(out))
    torch.cuda.synchronize()
    assert st == 0
    layout = native.get_layout(Tcap)
    final = ws[layout.final_f32:layout.final_f32 + T * 2048 * 4].view(torch.float32).view(T, 2048).cpu().numpy()
    return host_bits(out)[:T], final, int(flags.item())


def test_golden_cases_bit_exact(native, golden, layer1, bank1, make_golden, S):
    for name, _, seed, T, pad, hot, entry, special in make_golden.CASES:
        x, w, ids = make_golden.make_case(S, layer1, seed, T, pad, hot, special)
        out, final, flags = run_entry(native, entry, x, w, ids, bank1)
        np.testing.assert_array_equal(out, golden[f'{name}/out'], err_msg=name)
        assert flags == int(golden[f'{name}/flags']), name
        if f'{name}/final_f32' in golden:
            np.testing.assert_array_equal(final.view(np.uint32), golden[f'{name}/final_f32'].view(np.uint32))


@pytest.mark.parametrize('T', [1, 2, 4, 5, 8, 13, 16, 17, 24, 31, 32, 33, 48, 64, 65, 100, 256])
@pytest.mark.parametrize('a8', [True, False])
def test_random_batches_vs_oracle(native, layer1, bank1, S, O, T, a8):
    rng = np.random.default_rng(1000 + T + (7 if a8 else 0))
    x = S.make_tokens(rng, T)
    bias = np.zeros(256, np.float32)
    bias[rng.integers(0, 256, 6)] = 3.0
    w, ids = S.random_routes(rng, T, pad_fraction=0.08, bias=bias)
    ref, ref_f32, ref_flags = O.routed_layer(x, w, ids, *bank1.np_routed, a8=a8)
    symbol = 'ornith_routed_direct_launch' if a8 else 'ornith_routed_direct_launch_a4'
    out, final, flags = run_entry(native, symbol, x, w, ids, bank1, Tcap=T + 3)
    np.testing.assert_array_equal(out, ref)
    np.testing.assert_array_equal(final.view(np.uint32), ref_f32.view(np.uint32))
    assert flags == ref_flags


def test_a4_prefill_switches_at_64(native, layer1, bank1, S, O):
    for T, a8 in ((64, True), (65, False)):
        rng = np.random.default_rng(T)
        x = S.make_tokens(rng, T)
        w, ids = S.random_routes(rng, T)
        ref, _, _ = O.routed_layer(x, w, ids, *bank1.np_routed, a8=a8)
        out, _, _ = run_entry(native, 'ornith_routed_direct_launch_a4_prefill', x, w, ids, bank1)
        np.testing.assert_array_equal(out, ref)


def test_shared_slot_golden(native, golden, layer1, bank1, make_golden, S, tables):
    silu, sigmoid = dev(tables['silu_fp32']), dev(tables['sigmoid_bf16'])
    for name, seed, T in (('shared_t1', 21, 1), ('shared_t7', 22, 7), ('shared_t16', 23, 16)):
        x, w, ids = make_golden.make_case(S, layer1, seed, T, 0.1, 0, '')
        logit = S.f32_to_bf16_bits(np.random.default_rng(seed + 100).standard_normal(T).astype(np.float32))
        ws = torch.empty(native.get_layout(16).workspace_bytes, dtype=torch.uint8, device=DEV)
        out = torch.empty((T, 2048), dtype=torch.bfloat16, device=DEV)
        shared = torch.empty((T, 2048), dtype=torch.bfloat16, device=DEV)
        flags = torch.zeros(1, dtype=torch.int32, device=DEV)
        native.routed_shared_out(dev(x), dev(w), dev(ids), *bank1.routed, *bank1.shared, dev(logit), silu,
                                 sigmoid, ws, out, shared, flags, 16)
        torch.cuda.synchronize()
        np.testing.assert_array_equal(host_bits(out), golden[f'{name}/out'])
        np.testing.assert_array_equal(host_bits(shared), golden[f'{name}/shared_out'])
        assert int(flags.item()) == int(golden[f'{name}/flags'])


def test_route_topk_bit_exact(native, O):
    rng = np.random.default_rng(3)
    logits = rng.standard_normal((777, 256)).astype(np.float32)
    logits[0, 10] = logits[0, 20] = 9.0
    logits[1, :] = -np.inf
    logits[1, 5] = 1.0
    logits[2, 7] = np.nan
    logits[3, :] = 0.0          # +0 / -0 ties: equal logits, lower index first
    logits[3, 1::3] = -0.0
    logits[4, :] = np.nan       # no finite logit: ids -1, weights 0
    logits[5, :] = -np.inf      # three finite logits
    logits[5, [200, 3, 77]] = [-1.0, -0.0, 0.0]
    w_ref, ids_ref = O.route_topk(logits)
    w = torch.empty((777, 8), dtype=torch.float32, device=DEV)
    ids = torch.empty((777, 8), dtype=torch.int32, device=DEV)
    flags = torch.zeros(1, dtype=torch.int32, device=DEV)
    native.route_topk(dev(logits), w, ids, flags)
    torch.cuda.synchronize()
    np.testing.assert_array_equal(ids.cpu().numpy(), ids_ref)
    np.testing.assert_array_equal(w.cpu().numpy().view(np.uint32), w_ref.view(np.uint32))
    assert int(flags.item()) == 1


def test_config1_from_logits(native, golden, S):
    x, router, l1 = S.config1(0)
    bank = Bank(l1)
    logits = golden['config1/logits']
    T = 4
    for key, bits in (('a8', 8), ('a4', 4)):
        ws = torch.empty(native.workspace_bytes(T), dtype=torch.uint8, device=DEV)
        out = torch.empty((T, 2048), dtype=torch.bfloat16, device=DEV)
        flags = torch.zeros(1, dtype=torch.int32, device=DEV)
        native.routed_from_logits(dev(x), dev(logits), *bank.routed, None, None, None, None, None, None, None,
                                  ws, out, None, flags, T, bits)
        torch.cuda.synchronize()
        np.testing.assert_array_equal(host_bits(out), golden[f'config1/out_{key}'])
        assert int(flags.item()) == int(golden[f'config1/flags_{key}'])


def edge_logits(rng, T):
    logits = rng.standard_normal((T, 256)).astype(np.float32)
    logits[0, 10] = logits[0, 20] = logits[0, 30] = 9.0
    logits[1, :] = 0.0
    logits[1, ::2] = -0.0
    logits[2, :] = -np.inf
    logits[2, [5, 250, 17]] = [0.5, 0.5, -3.0]
    logits[3, 7] = np.nan
    logits[3, 8] = np.inf
    return logits


@pytest.mark.parametrize('T', [1, 4, 8, 16, 27, 32])
def test_fused_routing_edges(native, layer1, bank1, S, O, T):
    """The decode kernel's own top-8 (from-logits entry, T <= 32) on ties,
    signed zeros, non-finite logits and tokens with fewer than 8 finite ones."""
    rng = np.random.default_rng(900 + T)
    x = S.make_tokens(rng, T)
    logits = edge_logits(rng, max(T, 4))[:T]
    w, ids = O.route_topk(logits)
    ref, _, ref_flags = O.routed_layer(x, w, ids, *bank1.np_routed, a8=True)
    ws = torch.empty(native.workspace_bytes(T), dtype=torch.uint8, device=DEV)
    out = torch.empty((T, 2048), dtype=torch.bfloat16, device=DEV)
    flags = torch.zeros(1, dtype=torch.int32, device=DEV)
    native.routed_from_logits(dev(x), dev(logits), *bank1.routed, None, None, None, None, None, None, None,
                              ws, out, None, flags, T, 8)
    torch.cuda.synchronize()
    np.testing.assert_array_equal(host_bits(out), ref)
    want = ref_flags | (1 if not np.isfinite(logits).all() else 0)
    assert int(flags.item()) == want


def shared_logit_like_device(x_bits, w_bits):
    """The device's fixed-order fp32 logit: lane partial sums over k = lane + 32i,
    then an xor tree over the 32 lanes, rounded to bf16."""
    from ornith_b200.synthetic import bf16_bits_to_f32, f32_to_bf16_bits
    x = bf16_bits_to_f32(x_bits).reshape(-1, 2048)
    w = bf16_bits_to_f32(w_bits)
    out = []
    for row in x:
        lanes = np.zeros(32, np.float32)
        for i in range(64):
            k = np.arange(32) + 32 * i
            lanes = (lanes + (row[k] * w[k]).astype(np.float32)).astype(np.float32)
        d = 16
        while d:
            lanes = (lanes + lanes[np.arange(32) ^ d]).astype(np.float32)
            d >>= 1
        out.append(lanes[0])
    return f32_to_bf16_bits(np.array(out, np.float32))


@pytest.mark.parametrize('T', [1, 6, 16, 40])
def test_from_logits_with_shared_expert(native, layer1, bank1, S, O, tables, T):
    rng = np.random.default_rng(50 + T)
    x = S.make_tokens(rng, T)
    logits = rng.standard_normal((T, 256)).astype(np.float32)
    w, ids = O.route_topk(logits)
    logit = shared_logit_like_device(x, bank1.gate_w)
    ref, ref_sh, _, ref_flags = O.routed_layer_shared(x, w, ids, *bank1.np_routed, *bank1.np_shared, logit,
                                                      tables['silu_fp32'], tables['sigmoid_bf16'])
    ws = torch.empty(native.workspace_bytes(T), dtype=torch.uint8, device=DEV)
    out = torch.empty((T, 2048), dtype=torch.bfloat16, device=DEV)
    shared = torch.empty((T, 2048), dtype=torch.bfloat16, device=DEV)
    flags = torch.zeros(1, dtype=torch.int32, device=DEV)
    native.routed_from_logits(dev(x), dev(logits), *bank1.routed, *bank1.shared, dev(bank1.gate_w),
                              dev(tables['silu_fp32']), dev(tables['sigmoid_bf16']), ws, out, shared, flags, T, 0)
    torch.cuda.synchronize()
    np.testing.assert_array_equal(host_bits(out), ref)
    np.testing.assert_array_equal(host_bits(shared), ref_sh)
    assert int(flags.item()) == ref_flags


def test_flags_and_edges_vs_oracle(native, layer1, bank1, S, O):
    rng = np.random.default_rng(77)
    T = 6
    x = S.make_tokens(rng, T)
    w, ids = S.random_routes(rng, T)
    x[0, 5] = 0x7F80            # +inf input
    x[1, :] = 0                 # zero row
    ids[2, :] = -1              # dead token
    ids[3, 1] = 256             # invalid id (flag 4)
    x[4, :256] = 0x7F00         # huge values: bf16 1.7e38 -> invalid activation scale (flag 2)
    for a8, symbol in ((True, 'ornith_routed_direct_launch'), (False, 'ornith_routed_direct_launch_a4')):
        ref, ref_f32, ref_flags = O.routed_layer(x, w, ids, *bank1.np_routed, a8=a8)
        out, final, flags = run_entry(native, symbol, x, w, ids, bank1)
        np.testing.assert_array_equal(out, ref)
        assert flags == ref_flags and flags & 4 and flags & 1


def test_latency_mode_edges_vs_oracle(native, layer1, bank1, S, O):
    """Two tokens (the fused kernel's tile-local mode): non-finite and huge
    inputs, a duplicate expert, padded slots and an invalid id."""
    rng = np.random.default_rng(78)
    T = 2
    x = S.make_tokens(rng, T)
    w, ids = S.random_routes(rng, T)
    x[0, 5] = 0x7F80            # +inf input
    ids[0, 3] = ids[0, 0]       # duplicate expert in one token
    x[1, :256] = 0x7F00         # huge values: invalid activation scale (flag 2)
    ids[1, 1] = 256             # invalid id (flag 4)
    ids[1, 5:] = -1             # padded slots
    for a8, symbol in ((True, 'ornith_routed_direct_launch'), (False, 'ornith_routed_direct_launch_a4')):
        ref, ref_f32, ref_flags = O.routed_layer(x, w, ids, *bank1.np_routed, a8=a8)
        out, final, flags = run_entry(native, symbol, x, w, ids, bank1)
        np.testing.assert_array_equal(out, ref)
        np.testing.assert_array_equal(final.view(np.uint32), ref_f32.view(np.uint32))
        assert flags == ref_flags and flags & 4 and flags & 1


def test_prefill_1120_sampled_tokens(native, layer1, bank1, S, O):
    """Chunked-prefill shape: tokens are independent, so 48 sampled tokens of
    the full 1120-row call are checked against the oracle run on just them."""
    rng = np.random.default_rng(1120)
    T = 1120
    x = S.make_tokens(rng, T)
    w, ids = S.random_routes(rng, T)
    out, _, flags = run_entry(native, 'ornith_routed_direct_launch_a4_prefill', x, w, ids, bank1)
    pick = np.sort(rng.choice(T, 48, replace=False))
    ref, _, ref_flags = O.routed_layer(x[pick], w[pick], ids[pick], *bank1.np_routed, a8=False)
    np.testing.assert_array_equal(out[pick], ref)
    assert flags == 0 == ref_flags


def test_repack_on_device(native):
    rng = np.random.default_rng(9)
    N, K = 1024, 2048
    c32 = rng.integers(0, 2 ** 32, (3, N // 32, K // 256, 32, 32), dtype=np.uint32)
    m32 = rng.integers(0, 2 ** 32, (3, N // 32, K // 256, 32), dtype=np.uint32)
    c16 = np.ascontiguousarray(c32.reshape(3, N // 32, K // 256, 32, 2, 16).transpose(0, 1, 4, 2, 3, 5))
    m16 = np.ascontiguousarray(m32.reshape(3, N // 32, K // 256, 2, 16).transpose(0, 1, 3, 2, 4))
    rc, rm = native.repack_n16_to_n32(dev(c16.reshape(3, N // 16, K // 256, 32, 16)),
                                      dev(m16.reshape(3, N // 16, K // 256, 16)), N, K)
    torch.cuda.synchronize()
    np.testing.assert_array_equal(rc.view(torch.int32).cpu().numpy().view(np.uint32), c32)
    np.testing.assert_array_equal(rm.view(torch.int32).cpu().numpy().view(np.uint32), m32)


def test_repeat_calls_deterministic(native, layer1, bank1, S):
    rng = np.random.default_rng(11)
    x = S.make_tokens(rng, 32)
    w, ids = S.random_routes(rng, 32)
    a = run_entry(native, 'ornith_routed_direct_launch', x, w, ids, bank1)
    b = run_entry(native, 'ornith_routed_direct_launch', x, w, ids, bank1)
    np.testing.assert_array_equal(a[0], b[0])


@pytest.mark.parametrize('T', [1, 3, 8, 32, 40, 300])
def test_multi_kernel_path_matches_fused(native, layer1, bank1, S, O, T, monkeypatch):
    """Decode batches run the fused persistent kernel and larger batches the
    tensor-core path; the multi-kernel CUDA-core path (forced through the
    environment) must give the same bits as both."""
    rng = np.random.default_rng(300 + T)
    x = S.make_tokens(rng, T)
    w, ids = S.random_routes(rng, T, pad_fraction=0.1)
    fused = run_entry(native, 'ornith_routed_direct_launch', x, w, ids, bank1)
    monkeypatch.setenv('ORNITH_MOE_B200_PATH', 'generic')
    multi = run_entry(native, 'ornith_routed_direct_launch', x, w, ids, bank1)
    ref, _, ref_flags = O.routed_layer(x, w, ids, *bank1.np_routed, a8=True)
    np.testing.assert_array_equal(fused[0], ref)
    np.testing.assert_array_equal(multi[0], ref)
    assert fused[2] == multi[2] == ref_flags


@pytest.mark.parametrize('T', [1, 2, 5, 32])
def test_duplicate_expert_ids(native, layer1, bank1, S, O, T):
    """Collisions: the same expert several times in one token.  At T=32 one
    expert receives 96 routes, beyond the fused kernel's register budget."""
    rng = np.random.default_rng(400 + T)
    x = S.make_tokens(rng, T)
    w, ids = S.random_routes(rng, T)
    ids[:, 1] = ids[:, 0]
    ids[:, 2:4] = 17
    for a8, symbol in ((True, 'ornith_routed_direct_launch'), (False, 'ornith_routed_direct_launch_a4')):
        ref, ref_f32, ref_flags = O.routed_layer(x, w, ids, *bank1.np_routed, a8=a8)
        out, final, flags = run_entry(native, symbol, x, w, ids, bank1)
        np.testing.assert_array_equal(out, ref)
        np.testing.assert_array_equal(final.view(np.uint32), ref_f32.view(np.uint32))
        assert flags == ref_flags


@pytest.mark.parametrize('T', [1, 4])
def test_all_slots_padded(native, layer1, bank1, S, T):
    rng = np.random.default_rng(5)
    x = S.make_tokens(rng, T)
    w = np.ones((T, 8), np.float32)
    ids = -np.ones((T, 8), np.int32)
    out, final, flags = run_entry(native, 'ornith_routed_direct_launch', x, w, ids, bank1)
    assert not out.any() and not final.any() and flags == 0


@pytest.mark.parametrize('T', [1, 3])
def test_shared_slot_with_all_routed_padded(native, layer1, bank1, S, O, tables, T):
    rng = np.random.default_rng(6)
    x = S.make_tokens(rng, T)
    w = np.ones((T, 8), np.float32)
    ids = -np.ones((T, 8), np.int32)
    logit = S.f32_to_bf16_bits(rng.standard_normal(T).astype(np.float32))
    ref, ref_sh, _, ref_flags = O.routed_layer_shared(x, w, ids, *bank1.np_routed, *bank1.np_shared, logit,
                                                      tables['silu_fp32'], tables['sigmoid_bf16'])
    ws = torch.empty(native.get_layout(16).workspace_bytes, dtype=torch.uint8, device=DEV)
    out = torch.empty((T, 2048), dtype=torch.bfloat16, device=DEV)
    shared = torch.empty((T, 2048), dtype=torch.bfloat16, device=DEV)
    flags = torch.zeros(1, dtype=torch.int32, device=DEV)
    native.routed_shared_out(dev(x), dev(w), dev(ids), *bank1.routed, *bank1.shared, dev(logit),
                             dev(tables['silu_fp32']), dev(tables['sigmoid_bf16']), ws, out, shared, flags, 16)
    torch.cuda.synchronize()
    np.testing.assert_array_equal(host_bits(out), ref)
    np.testing.assert_array_equal(host_bits(shared), ref_sh)
    assert int(flags.item()) == ref_flags


@pytest.mark.parametrize('T', [1, 7, 64])
def test_combine_gathered_matches_dense_combine(native, S, T):
    """The expert-parallel home combine reads returned rows through a (token, slot)
    index; it must give the dense per-route combine's bits, and flag a valid slot
    whose row index is out of range."""
    rng = np.random.default_rng(11 + T)
    ids = rng.integers(0, 128, (T, 8)).astype(np.int32)
    ids[rng.random((T, 8)) < 0.2] = -1
    w = rng.random((T, 8)).astype(np.float32)
    valid = ids >= 0
    n = int(valid.sum())
    order = rng.permutation(n)
    row_index = -np.ones((T, 8), np.int32)
    row_index[valid] = order
    rows = rng.standard_normal((n + 3, 2048)).astype(np.float32)
    dense = np.zeros((T * 8, 2048), np.float32)
    dense[valid.reshape(-1)] = rows[order]
    ref = np.zeros((T, 2048), np.float32)
    for s in range(8):
        ref = np.where(valid[:, s:s + 1], (ref + dense.reshape(T, 8, 2048)[:, s] * w[:, s:s + 1]).astype(np.float32),
                       ref)
    ref_bits = S.f32_to_bf16_bits(ref)
    wd, idd = dev(w), dev(ids)
    out_g = torch.empty((T, 2048), dtype=torch.bfloat16, device=DEV)
    out_d = torch.empty((T, 2048), dtype=torch.bfloat16, device=DEV)
    flags = torch.zeros(1, dtype=torch.int32, device=DEV)
    native.combine_gathered(dev(rows), dev(row_index), wd, idd, out_g, flags)
    native.combine_rows(dev(dense), wd, idd, out_d, flags)
    torch.cuda.synchronize()
    assert int(flags.item()) == 0
    np.testing.assert_array_equal(host_bits(out_g), ref_bits)
    np.testing.assert_array_equal(host_bits(out_d), ref_bits)
    bad = row_index.copy()
    t, s = np.argwhere(valid)[0]
    bad[t, s] = n + 3
    native.combine_gathered(dev(rows), dev(bad), wd, idd, out_g, flags)
    torch.cuda.synchronize()
    assert int(flags.item()) & 4


@pytest.mark.parametrize('T', [5, 96])
def test_gather_route_rows_across_paths(native, layer1, bank1, S, T, monkeypatch):
    """gather_route_rows and scatter_route_rows return the same per-route rows
    whichever path ran the layer: route order (decode kernel, multi-kernel
    path) or expert-slot order (tensor-core path, read through its route ->
    row map)."""
    rng = np.random.default_rng(900 + T)
    x = S.make_tokens(rng, T)
    w, ids = S.random_routes(rng, T, pad_fraction=0.1)
    sel = torch.from_numpy(np.flatnonzero(ids.reshape(-1) >= 0).astype(np.int32)).to(DEV)

    def rows_after_layer():
        ws = torch.empty(native.get_layout(T).workspace_bytes, dtype=torch.uint8, device=DEV)
        out = torch.empty((T, 2048), dtype=torch.bfloat16, device=DEV)
        flags = torch.zeros(1, dtype=torch.int32, device=DEV)
        native.check(native.lib().ornith_routed_direct_launch(
            *[native.ptr(t) for t in (dev(x), dev(w), dev(ids), *bank1.routed, ws)], ws.numel(), native.ptr(out),
            native.ptr(flags), T, T, native.stream(out)), 'layer')
        rows = torch.empty((sel.numel(), 2048), dtype=torch.float32, device=DEV)
        native.gather_route_rows(ws, T, T, sel, rows, flags)
        dense = torch.zeros((T * 8, 2048), dtype=torch.float32, device=DEV)
        native.scatter_route_rows(ws, T, T, dense)
        torch.cuda.synchronize()
        return rows.cpu().numpy(), dense[sel.long()].cpu().numpy(), int(flags.item())

    fast, fast_dense, f1 = rows_after_layer()
    monkeypatch.setenv('ORNITH_MOE_B200_PATH', 'generic')
    multi, multi_dense, f2 = rows_after_layer()
    assert f1 == f2 == 0
    np.testing.assert_array_equal(fast.view(np.uint32), multi.view(np.uint32))
    np.testing.assert_array_equal(fast_dense.view(np.uint32), fast.view(np.uint32))
    np.testing.assert_array_equal(multi_dense.view(np.uint32), multi.view(np.uint32))


@pytest.mark.parametrize('T', [1, 4, 33, 300])
def test_router_logits_vs_oracle(native, S, O, T):
    """Router linear (gates_projection.py:17-25): fp32 sums whose order the
    reference leaves unspecified, so agreement is to fp32 rounding (relative
    1e-5 of the sum of |x*w|), against the oracle's exact (double) sum."""
    rng = np.random.default_rng(70 + T)
    x = S.make_tokens(rng, T)
    w = S.make_router(rng)
    ref = O.router_logits(x, w)
    logits = torch.empty((T, 256), dtype=torch.float32, device=DEV)
    native.router_logits(dev(x), dev(w), logits)
    torch.cuda.synchronize()
    got = logits.cpu().numpy()
    scale = np.abs(S.bf16_bits_to_f32(x)) @ np.abs(S.bf16_bits_to_f32(w)).T
    assert np.all(np.abs(got - ref) <= 1e-5 * scale + 1e-30)


def test_config1_from_hidden(native, golden, S):
    """Config 1 with the router linear on the GPU: logits within rounding of the
    reference's, the same top-8 ids as the golden case, and the fused entry
    equal bit for bit to the from-logits entry fed the same logits."""
    x, router, l1 = S.config1(0)
    bank = Bank(l1)
    T = 4
    ws = torch.empty(native.workspace_bytes(T), dtype=torch.uint8, device=DEV)
    out_h = torch.empty((T, 2048), dtype=torch.bfloat16, device=DEV)
    out_l = torch.empty((T, 2048), dtype=torch.bfloat16, device=DEV)
    logits = torch.empty((T, 256), dtype=torch.float32, device=DEV)
    flags = torch.zeros(1, dtype=torch.int32, device=DEV)
    native.routed_from_hidden(dev(x), dev(router), logits, *bank.routed, None, None, None, None, None, None, None,
                              ws, out_h, None, flags, T, 8)
    native.routed_from_logits(dev(x), logits.clone(), *bank.routed, None, None, None, None, None, None, None,
                              ws, out_l, None, flags, T, 8)
    torch.cuda.synchronize()
    ref = golden['config1/logits']
    got = logits.cpu().numpy()
    np.testing.assert_allclose(got, ref, rtol=1e-5, atol=1e-5)
    ref_top = np.argsort(-ref, axis=1, kind='stable')[:, :8]
    got_top = np.argsort(-got, axis=1, kind='stable')[:, :8]
    np.testing.assert_array_equal(np.sort(got_top, axis=1), np.sort(ref_top, axis=1))
    np.testing.assert_array_equal(host_bits(out_h), host_bits(out_l))


# Route counts per chosen expert for the multi-tile cases: one short of, at
# and one past a 128-row tile, two tiles and two tiles plus one, more routes
# than tokens at T = 300 (duplicates inside tokens), and at 8192 an expert
# with 16 tiles and one with a single route.
HOT_BY_T = {
    300: None,   # make_golden.HOT_COUNTS, pinned by a reference digest below
    1120: {3: 127, 40: 128, 77: 129, 128: 256, 200: 257, 255: 1100, 9: 1},
    8192: {3: 127, 40: 128, 77: 129, 128: 256, 200: 257, 255: 1100, 17: 2048, 9: 1},
}


def hot_token_sample(rng, ids, counts, per_expert=24, extra=48):
    """Tokens to check against the oracle: for each hot expert its first and
    last token and up to `per_expert` others, plus `extra` random tokens."""
    T = ids.shape[0]
    pick = set(rng.choice(T, min(extra, T), replace=False).tolist())
    for e in counts:
        toks = np.flatnonzero((ids == e).any(axis=1))
        pick.update([int(toks[0]), int(toks[-1])])
        pick.update(rng.choice(toks, min(per_expert, toks.size), replace=False).tolist())
    return np.array(sorted(pick))


@pytest.mark.parametrize('T', [300, 1120, 8192])
@pytest.mark.parametrize('a8', [True, False])
def test_hot_experts_span_several_tiles(native, layer1, bank1, S, O, make_golden, T, a8):
    """Experts whose routes fill several 128-row tiles of the tensor-core path
    (tile tails, the per-expert tile lists and the row positions past the
    first tile): the sampled tokens, every hot expert's first and last token
    among them, equal the oracle bit for bit.  At T = 300 every token is
    checked."""
    counts = HOT_BY_T[T] or make_golden.HOT_COUNTS
    rng = np.random.default_rng(8000 + T + (1 if a8 else 0))
    x = S.make_tokens(rng, T)
    w, ids = S.hot_routes(rng, T, counts, pad_fraction=0.02)
    for e, c in counts.items():
        assert int((ids == e).sum()) == c
    symbol = 'ornith_routed_direct_launch' if a8 else 'ornith_routed_direct_launch_a4'
    out, _, flags = run_entry(native, symbol, x, w, ids, bank1)
    pick = np.arange(T) if T <= 300 else hot_token_sample(rng, ids, counts)
    ref, _, ref_flags = O.routed_layer(x[pick], w[pick], ids[pick], *bank1.np_routed, a8=a8)
    np.testing.assert_array_equal(out[pick], ref)
    assert flags == ref_flags == 0


@pytest.mark.parametrize('entry_name', ['digest', 'hot_digest'])
def test_larger_batches_match_reference_digests(native, layer1, bank1, S, make_golden, entry_name):
    """The CUDA outputs hash to the digests of the compiled reference's own
    outputs: T = 32 (A8), 64 (A4), 1120 (A4 prefill) and the two T = 300
    hot-expert cases whose experts span one to nine 128-row tiles."""
    from pathlib import Path
    digests = np.load(Path(__file__).resolve().parent / 'golden' / 'routed_reference_digests.npz')
    if entry_name == 'digest':
        cases = [(name, make_golden.make_case(S, layer1, seed, T, pad, 0, ''), entry)
                 for name, seed, T, pad, entry in make_golden.DIGEST_CASES]
    else:
        cases = [(name, make_golden.make_hot_case(S, seed, T, pad, counts), entry)
                 for name, seed, T, pad, entry, counts in make_golden.HOT_DIGEST_CASES]
    for name, (x, w, ids), entry in cases:
        assert make_golden.digest(x, w, ids) == str(digests[f'{name}/inputs_sha256']), name
        out, _, flags = run_entry(native, entry, x, w, ids, bank1)
        assert make_golden.digest(out) == str(digests[f'{name}/out_sha256']), name
        assert flags == int(digests[f'{name}/flags']), name


@pytest.mark.parametrize('path', ['a4_prefill', 'from_logits'])
def test_prefill_8192_sampled_tokens(native, layer1, bank1, S, O, path):
    """The headline prefill size: 8192 tokens (about 256 routes per expert, so
    every expert spans two or more 128-row tiles), A4, through the reference's
    A4-prefill entry and through the from-logits operator the benchmark
    calls (device top-8 included); 64 sampled tokens against the oracle."""
    rng = np.random.default_rng(8192)
    T = 8192
    x = S.make_tokens(rng, T)
    logits = rng.standard_normal((T, 256)).astype(np.float32)
    w, ids = O.route_topk(logits)
    if path == 'a4_prefill':
        out, _, flags = run_entry(native, 'ornith_routed_direct_launch_a4_prefill', x, w, ids, bank1)
    else:
        ws = torch.empty(native.workspace_bytes(T), dtype=torch.uint8, device=DEV)
        o = torch.empty((T, 2048), dtype=torch.bfloat16, device=DEV)
        fl = torch.zeros(1, dtype=torch.int32, device=DEV)
        native.routed_from_logits(dev(x), dev(logits), *bank1.routed, None, None, None, None, None, None, None,
                                  ws, o, None, fl, T, 4)
        torch.cuda.synchronize()
        out, flags = host_bits(o), int(fl.item())
        del ws
    assert np.bincount(ids.reshape(-1), minlength=256).min() > 128
    pick = np.sort(rng.choice(T, 64, replace=False))
    ref, _, ref_flags = O.routed_layer(x[pick], w[pick], ids[pick], *bank1.np_routed, a8=False)
    np.testing.assert_array_equal(out[pick], ref)
    assert flags == 0 == ref_flags


def single_token_cases(S, rng, n=10):
    """T = 1 routes: random, padded, duplicated, invalid ids and non-finite
    inputs (one of each kind per case index)."""
    cases = []
    for i in range(n):
        x = S.make_tokens(rng, 1)
        w, ids = S.random_routes(rng, 1, pad_fraction=0.15 if i % 3 == 0 else 0.0)
        if i % 4 == 1:
            ids[0, 5] = ids[0, 2]             # an expert named by two slots
        if i % 5 == 2:
            ids[0, 3] = 300                   # invalid id: flag 4
        if i % 7 == 3:
            x[0, 11] = 0x7F80                 # +inf input: flag 1
        if i == n - 1:
            ids[0, :] = -1                    # every slot padded
        cases.append((x, w, ids))
    return cases


@pytest.mark.parametrize('a8', [True, False])
def test_single_token_kernel_matches_multi_token_kernel(native, layer1, bank1, S, O, a8, monkeypatch):
    """T = 1 runs the single-token kernel; the multi-token kernel (selected
    with ORNITH_MOE_B200_DECODE1=0) and the oracle give the same bits, fp32
    diagnostic and flags on padding, duplicate and invalid ids and non-finite
    inputs."""
    symbol = 'ornith_routed_direct_launch' if a8 else 'ornith_routed_direct_launch_a4'
    for x, w, ids in single_token_cases(S, np.random.default_rng(4242 + a8)):
        monkeypatch.delenv('ORNITH_MOE_B200_DECODE1', raising=False)
        one = run_entry(native, symbol, x, w, ids, bank1)
        monkeypatch.setenv('ORNITH_MOE_B200_DECODE1', '0')
        multi = run_entry(native, symbol, x, w, ids, bank1)
        ref, ref_f32, ref_flags = O.routed_layer(x, w, ids, *bank1.np_routed, a8=a8)
        np.testing.assert_array_equal(one[0], ref)
        np.testing.assert_array_equal(one[1].view(np.uint32), ref_f32.view(np.uint32))
        np.testing.assert_array_equal(multi[0], one[0])
        assert one[2] == multi[2] == ref_flags


def test_single_token_kernel_shared_expert_and_from_logits(native, layer1, bank1, S, O, tables, monkeypatch):
    """The single-token kernel with the shared expert: the caller's logit and
    tables (shared-slot entry) and the from-logits operator (device top-8 and
    shared logit), against the oracle and the multi-token kernel."""
    silu, sigmoid = dev(tables['silu_fp32']), dev(tables['sigmoid_bf16'])
    rng = np.random.default_rng(77)
    for i, (x, w, ids) in enumerate(single_token_cases(S, rng, 6)):
        logit = S.f32_to_bf16_bits(rng.standard_normal(1).astype(np.float32))
        ref, ref_sh, _, ref_flags = O.routed_layer_shared(x, w, ids, *bank1.np_routed, *bank1.np_shared, logit,
                                                          tables['silu_fp32'], tables['sigmoid_bf16'])
        got = []
        for env in (None, '0'):
            if env is None:
                monkeypatch.delenv('ORNITH_MOE_B200_DECODE1', raising=False)
            else:
                monkeypatch.setenv('ORNITH_MOE_B200_DECODE1', env)
            ws = torch.empty(native.get_layout(16).workspace_bytes, dtype=torch.uint8, device=DEV)
            out = torch.empty((1, 2048), dtype=torch.bfloat16, device=DEV)
            shared = torch.empty((1, 2048), dtype=torch.bfloat16, device=DEV)
            flags = torch.zeros(1, dtype=torch.int32, device=DEV)
            native.routed_shared_out(dev(x), dev(w), dev(ids), *bank1.routed, *bank1.shared, dev(logit), silu,
                                     sigmoid, ws, out, shared, flags, 16)
            torch.cuda.synchronize()
            got.append((host_bits(out), host_bits(shared), int(flags.item())))
        for o, sh, fl in got:
            np.testing.assert_array_equal(o, ref)
            np.testing.assert_array_equal(sh, ref_sh)
            assert fl == ref_flags
    monkeypatch.delenv('ORNITH_MOE_B200_DECODE1', raising=False)
    for seed in range(4):
        r2 = np.random.default_rng(600 + seed)
        x = S.make_tokens(r2, 1)
        logits = r2.standard_normal((1, 256)).astype(np.float32)
        if seed == 3:
            logits[0, 40] = np.nan
        w, ids = O.route_topk(logits)
        lg = shared_logit_like_device(x, bank1.gate_w)
        ref, ref_sh, _, ref_flags = O.routed_layer_shared(x, w, ids, *bank1.np_routed, *bank1.np_shared, lg,
                                                          tables['silu_fp32'], tables['sigmoid_bf16'])
        ws = torch.empty(native.workspace_bytes(1), dtype=torch.uint8, device=DEV)
        out = torch.empty((1, 2048), dtype=torch.bfloat16, device=DEV)
        shared = torch.empty((1, 2048), dtype=torch.bfloat16, device=DEV)
        flags = torch.zeros(1, dtype=torch.int32, device=DEV)
        native.routed_from_logits(dev(x), dev(logits), *bank1.routed, *bank1.shared, dev(bank1.gate_w), silu,
                                  sigmoid, ws, out, shared, flags, 1, 0)
        torch.cuda.synchronize()
        np.testing.assert_array_equal(host_bits(out), ref)
        np.testing.assert_array_equal(host_bits(shared), ref_sh)
        assert int(flags.item()) == ref_flags | (1 if seed == 3 else 0)


def test_single_token_kernel_call_numbers(native, layer1, bank1, S, O):
    """The single-token kernel tags its flags with call numbers kept in the
    workspace instead of clearing them: a workspace that starts as all-ones
    bytes, many calls in a row, and calls of the multi-token kernel (T = 3)
    on the same workspace in between all give the oracle's bits."""
    rng = np.random.default_rng(31)
    cases = [(S.make_tokens(rng, T), *S.random_routes(rng, T, pad_fraction=0.1)) for T in (1, 1, 3, 1, 3, 1)]
    refs = [O.routed_layer(x, w, ids, *bank1.np_routed, a8=True) for x, w, ids in cases]
    ws = torch.full((native.get_layout(8).workspace_bytes,), 255, dtype=torch.uint8, device=DEV)
    out = torch.empty((3, 2048), dtype=torch.bfloat16, device=DEV)
    fn = native.lib().ornith_routed_direct_launch
    for rep in range(40):
        i = rep % len(cases)
        x, w, ids = cases[i]
        T = x.shape[0]
        flags = torch.zeros(1, dtype=torch.int32, device=DEV)
        st = fn(*[native.ptr(t) for t in (dev(x), dev(w), dev(ids), *bank1.routed, ws)], ws.numel(),
                native.ptr(out), native.ptr(flags), T, 8, native.stream(out))
        assert st == 0
        torch.cuda.synchronize()
        np.testing.assert_array_equal(host_bits(out)[:T], refs[i][0], err_msg=f'call {rep}')
        assert int(flags.item()) == refs[i][2], f'call {rep}'


def run_from_hidden(native, x, router, bank, shared_args, Tcap, ws=None):
    """One routed_from_hidden call; returns (logits bits, out bits, shared bits, flags)."""
    T = x.shape[0]
    if ws is None:
        ws = torch.empty(native.workspace_bytes(Tcap), dtype=torch.uint8, device=DEV)
    logits = torch.full((T, 256), float('nan'), dtype=torch.float32, device=DEV)
    out = torch.empty((T, 2048), dtype=torch.bfloat16, device=DEV)
    shared = torch.empty((T, 2048), dtype=torch.bfloat16, device=DEV) if shared_args[0] is not None else None
    flags = torch.zeros(1, dtype=torch.int32, device=DEV)
    native.routed_from_hidden(dev(x), router, logits, *bank.routed, *shared_args, ws, out, shared, flags, Tcap, 0)
    torch.cuda.synchronize()
    return (logits.cpu().numpy().view(np.uint32), host_bits(out),
            None if shared is None else host_bits(shared), int(flags.item()))


@pytest.mark.parametrize('with_shared', [False, True])
def test_single_token_from_hidden_router_in_kernel(native, layer1, bank1, S, O, tables, with_shared, monkeypatch):
    """T = 1 from hidden states: the single-token kernel computes the router
    linear itself.  Its logits equal the router launch's bit for bit, and its
    outputs and flags equal the from-logits entry fed those logits, the
    two-launch path (ORNITH_MOE_B200_DECODE1=0) and the oracle routed from
    the same logits; one case has a +inf input (non-finite logits, flag 1)."""
    silu, sigmoid = dev(tables['silu_fp32']), dev(tables['sigmoid_bf16'])
    shared_args = ((*bank1.shared, dev(bank1.gate_w), silu, sigmoid) if with_shared else (None,) * 7)
    rng = np.random.default_rng(900 + with_shared)
    router = dev(S.make_router(rng))
    for case in range(5):
        x = S.make_tokens(rng, 1)
        if case == 4:
            x[0, 100] = 0x7F80
        monkeypatch.delenv('ORNITH_MOE_B200_DECODE1', raising=False)
        lg, out, sh, fl = run_from_hidden(native, x, router, bank1, shared_args, 1)
        sep = torch.empty((1, 256), dtype=torch.float32, device=DEV)
        native.router_logits(dev(x), router, sep)
        torch.cuda.synchronize()
        np.testing.assert_array_equal(lg, sep.cpu().numpy().view(np.uint32))
        monkeypatch.setenv('ORNITH_MOE_B200_DECODE1', '0')
        lg2, out2, sh2, fl2 = run_from_hidden(native, x, router, bank1, shared_args, 1)
        monkeypatch.delenv('ORNITH_MOE_B200_DECODE1', raising=False)
        np.testing.assert_array_equal(lg2, lg)
        np.testing.assert_array_equal(out2, out)
        assert fl2 == fl
        logits = sep.cpu().numpy()
        w, ids = O.route_topk(logits)
        if with_shared:
            lgs = shared_logit_like_device(x, bank1.gate_w)
            ref, ref_sh, _, ref_flags = O.routed_layer_shared(x, w, ids, *bank1.np_routed, *bank1.np_shared, lgs,
                                                              tables['silu_fp32'], tables['sigmoid_bf16'])
            np.testing.assert_array_equal(sh, ref_sh)
            np.testing.assert_array_equal(sh2, sh)
        else:
            ref, _, ref_flags = O.routed_layer(x, w, ids, *bank1.np_routed, a8=True)
        np.testing.assert_array_equal(out, ref)
        nonfinite = 1 if not np.all(np.isfinite(logits)) else 0
        assert fl == ref_flags | nonfinite


def test_single_token_from_hidden_call_numbers(native, layer1, bank1, S):
    """The router words the single-token kernel exchanges carry call numbers:
    one workspace that starts as all-ones bytes, T = 1 and T = 3 calls
    alternating, every T = 1 call equal to its first run."""
    rng = np.random.default_rng(61)
    router = dev(S.make_router(rng))
    xs = [S.make_tokens(rng, T) for T in (1, 3, 1, 1, 3)]
    ws = torch.full((native.workspace_bytes(8),), 255, dtype=torch.uint8, device=DEV)
    none = (None,) * 7
    first = {}
    for rep in range(25):
        i = rep % len(xs)
        got = run_from_hidden(native, xs[i], router, bank1, none, 8, ws)
        if i in first:
            for a, b in zip(got[:2], first[i][:2]):
                np.testing.assert_array_equal(a, b, err_msg=f'call {rep}')
            assert got[3] == first[i][3] == 0
        else:
            first[i] = got
