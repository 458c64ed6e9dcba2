"""CPU: the device dispatch plan of expert parallelism (ornith_moe_b200_ep_plan).

Without a GPU this checks the entry point's argument validation (every case
returns before device work), the kernel's algorithm restated step by step in
Python (per-thread token runs, block scans, second pass) against the torch
form of the plan, and the native planner's use of the kernel's outputs."""
import ctypes as C

import pytest
import torch

E, TOP = 256, 8
THREADS = 1024
INVALID = 1


def _ids(T, seed, world):
    gen = torch.Generator().manual_seed(seed)
    ids = torch.topk(torch.randn((T, E), generator=gen), TOP, dim=1).indices.to(torch.int32)
    if T:
        ids[::7, 2] = -1                      # padding
        ids[0, :] = -1                        # a token with no expert
        ids[T // 2, 5] = 300                  # invalid ids: no rank owns them
        ids[-1, 0] = -9
    return ids


def _placements(world):
    import __graft_entry__ as g
    g.load_package()
    from ornith_b200 import ep
    loads = torch.rand(E, generator=torch.Generator().manual_seed(world)) ** 3
    return ep, [ep.contiguous_placement(world), ep.balanced_placement(loads, world)]


def emulate_kernel(ids, owner, local, world):
    """ep_plan_kernel step by step: thread i owns tokens [i*c, (i+1)*c); the
    per-thread (tokens, slots) counts per destination are scanned in thread
    order; the second pass writes rows.  Buffers are T*world rows, filled with
    a marker beyond the plan."""
    T = ids.shape[0]
    ids_l = ids.tolist()
    owner_l, local_l = owner.tolist(), local.tolist()

    def owners(t):
        out = []
        for v in ids_l[t]:
            d = owner_l[v] if 0 <= v < E else -1
            out.append(d if 0 <= d < world else -1)
        return out

    c = (T + THREADS - 1) // THREADS
    runs = [(min(T, i * c), min(T, min(T, i * c) + c)) for i in range(THREADS)]
    per = []
    for t0, t1 in runs:
        tok, slots = [0] * world, [0] * world
        for t in range(t0, t1):
            own = owners(t)
            for d in range(world):
                tok[d] += d in own
                slots[d] += own.count(d)
        per.append((tok, slots))
    tot_tok = [sum(p[0][d] for p in per) for d in range(world)]
    tot_slot = [sum(p[1][d] for p in per) for d in range(world)]
    n = T * world
    token_index, dest = [-7] * n, [-7] * n
    local_ids, slot_mask = [[-7] * TOP for _ in range(n)], [[False] * TOP for _ in range(n)]
    row_index = [[-7] * TOP for _ in range(T)]
    before_tok, before_slot = [0] * world, [0] * world    # exclusive scan over threads
    for (t0, t1), (tok, slots) in zip(runs, per):
        pos = [sum(tot_tok[:d]) + before_tok[d] for d in range(world)]
        row = [sum(tot_slot[:d]) + before_slot[d] for d in range(world)]
        for t in range(t0, t1):
            own = owners(t)
            ri = [-1] * TOP
            for d in range(world):
                if d not in own:
                    continue
                p = pos[d]
                pos[d] += 1
                token_index[p], dest[p] = t, d
                for s in range(TOP):
                    here = own[s] == d
                    local_ids[p][s] = local_l[ids_l[t][s]] if here else -1
                    slot_mask[p][s] = here
                    if here:
                        ri[s] = row[d]
                        row[d] += 1
            row_index[t] = ri
        for d in range(world):
            before_tok[d] += tok[d]
            before_slot[d] += slots[d]
    counts = torch.tensor([[tot_tok[d], tot_slot[d]] for d in range(world)], dtype=torch.int64).view(world, 2)
    return (counts, torch.tensor(token_index, dtype=torch.int64), torch.tensor(dest, dtype=torch.int64),
            torch.tensor(local_ids, dtype=torch.int32).view(n, TOP), torch.tensor(slot_mask).view(n, TOP),
            torch.tensor(row_index, dtype=torch.int32).view(T, TOP))


def torch_plan(ep, ids, world, placement):
    planner = ep.TorchPlanner(world, placement)
    state, counts = planner.start(ids)
    plan = planner.finish(state, ids, counts[:, 0].tolist(), counts[:, 1].tolist())
    return counts, plan, ep.route_row_index(ids.shape[0], plan, ids.device)


@pytest.mark.parametrize('world', [1, 2, 4, 8])
@pytest.mark.parametrize('T', [0, 1, 37, 1025, 2500])
def test_kernel_algorithm_matches_torch_plan(world, T):
    ep, placements = _placements(world)
    ids = _ids(T, 100 + T + world, world)
    for placement in placements:
        counts, plan, row_index = torch_plan(ep, ids, world, placement)
        k = emulate_kernel(ids, placement.rank.to(torch.int32), placement.local.to(torch.int32), world)
        n = int(counts[:, 0].sum())
        assert torch.equal(k[0], counts)
        assert torch.equal(k[1][:n], plan.token_index)
        assert torch.equal(k[2][:n], plan.dest)
        assert torch.equal(k[3][:n], plan.local_ids)
        assert torch.equal(k[4][:n], plan.slot_mask)
        assert torch.equal(k[5], row_index)


def test_native_planner_uses_the_kernel_outputs(monkeypatch):
    """NativePlanner.finish keeps the first n rows of each buffer and hands the
    kernel's row index to route_row_index (the launch itself is emulated)."""
    world, T = 4, 300
    ep, placements = _placements(world)
    placement = placements[1]
    ids = _ids(T, 7, world)
    from ornith_b200 import native
    monkeypatch.setattr(native, 'ep_plan', lambda i, o, l, w: emulate_kernel(i, o, l, w))
    planner = ep.NativePlanner(world, placement, 'cpu')
    state, counts = planner.start(ids)
    plan = planner.finish(state, ids, counts[:, 0].tolist(), counts[:, 1].tolist())
    ref_counts, ref, ref_rows = torch_plan(ep, ids, world, placement)
    assert torch.equal(counts, ref_counts)
    for field in ('token_index', 'dest', 'local_ids', 'slot_mask'):
        assert torch.equal(getattr(plan, field), getattr(ref, field)), field
    assert plan.send_counts == ref.send_counts and plan.home_counts == ref.home_counts
    assert ep.route_row_index(T, plan, ids.device) is plan.row_index
    assert torch.equal(plan.row_index, ref_rows)


def test_ep_plan_validation_without_device_work(native):
    fn = native.lib().ornith_moe_b200_ep_plan
    base = 1 << 30
    p = [C.c_void_p(base + (i << 24)) for i in range(9)]
    ids, owner, local, counts, tok, dest, lids, mask, rows = p
    ok = dict(ids=ids, owner=owner, local=local, counts=counts, tok=tok, dest=dest, lids=lids, mask=mask, rows=rows)

    def call(T=4, world=2, **kw):
        a = dict(ok, **kw)
        return fn(a['ids'], T, a['owner'], a['local'], world, a['counts'], a['tok'], a['dest'], a['lids'], a['mask'],
                  a['rows'], None)

    assert call(T=-1) == INVALID
    assert call(T=8193) == INVALID
    assert call(world=0) == INVALID
    assert call(world=9) == INVALID
    assert call(owner=None) == INVALID
    assert call(counts=None) == INVALID
    assert call(counts=C.c_void_p(base + (3 << 24) + 4)) == INVALID   # int64 counts 8-byte aligned
    assert call(owner=C.c_void_p(base + (1 << 24) + 2)) == INVALID
    for name in ('ids', 'tok', 'dest', 'lids', 'mask', 'rows'):
        assert call(**{name: None}) == INVALID, name
    assert call(tok=C.c_void_p(base + (4 << 24) + 4)) == INVALID
    assert call(rows=C.c_void_p(base + (8 << 24) + 2)) == INVALID


def test_peer_return_validation_without_device_work(native):
    """The peer-memory return's entry points reject bad arguments before any
    device work; every destination range is checked against the capacity."""
    lib = native.lib()
    p = C.c_void_p()
    assert lib.ornith_moe_b200_ep_buffer_alloc(0, C.byref(p)) == INVALID
    assert lib.ornith_moe_b200_ep_buffer_alloc(256, None) == INVALID
    assert lib.ornith_moe_b200_ep_buffer_free(None) == 0
    assert lib.ornith_moe_b200_ep_ipc_close(None) == 0
    h = (C.c_uint8 * 64)()
    assert lib.ornith_moe_b200_ep_ipc_handle(None, h) == INVALID
    assert lib.ornith_moe_b200_ep_ipc_open(None, C.byref(p)) == INVALID
    sig = C.c_void_p(1 << 30)
    assert lib.ornith_moe_b200_ep_wait_signals(sig, 0, 0, 1, sig, None) == INVALID
    assert lib.ornith_moe_b200_ep_wait_signals(sig, 9, 0, 1, sig, None) == INVALID
    assert lib.ornith_moe_b200_ep_wait_signals(sig, 2, 2, 1, sig, None) == INVALID
    assert lib.ornith_moe_b200_ep_wait_signals(None, 2, 0, 1, sig, None) == INVALID
    assert lib.ornith_moe_b200_ep_wait_signals(sig, 1, 0, 1, sig, None) == 0     # one rank: nothing to wait for

    fn = lib.ornith_moe_b200_ep_return_p2p
    nb = native.get_layout(16).workspace_bytes
    base = 1 << 32
    ws, ri, counter, flags = (C.c_void_p(base + (i << 28)) for i in range(4))
    world = 2
    dst = (C.c_void_p * world)(base + (5 << 28), base + (6 << 28))
    sigs = (C.c_void_p * world)(base + (7 << 28), base + (8 << 28))

    def call(seg=(0, 3, 5), off=(0, 4), cap=8, n=5, me=0, T=16, Tcap=16, nbytes=nb, w=world, d=dst, s=sigs):
        seg_a = (C.c_int32 * len(seg))(*seg)
        off_a = (C.c_int64 * len(off))(*off)
        return fn(ws, nbytes, T, Tcap, ri, n, seg_a, d, off_a, cap, s, w, me, 1, counter, flags, None)

    assert call(T=17) == INVALID
    assert call(nbytes=nb - 1) == INVALID
    assert call(w=0) == INVALID
    assert call(me=2) == INVALID
    assert call(seg=(1, 3, 5)) == INVALID           # segments start at 0
    assert call(seg=(0, 3, 4)) == INVALID           # and end at n
    assert call(seg=(0, 4, 3), n=3) == INVALID      # and never go down
    assert call(off=(6, 0)) == INVALID              # rank 0's 3 rows at 6..8 of an 8-row buffer
    assert call(off=(0, 7)) == INVALID              # rank 1's 2 rows at 7..8
    assert call(off=(-1, 0)) == INVALID
    assert call(cap=-1) == INVALID
    assert call(d=(C.c_void_p * world)(base + (5 << 28), None)) == INVALID
    assert call(d=(C.c_void_p * world)(base + (5 << 28) + 4, base + (6 << 28))) == INVALID   # 16-byte rows
    assert call(s=(C.c_void_p * world)(base + (7 << 28), None)) == INVALID                 # a peer's flags


def test_peer_dispatch_validation_without_device_work(native):
    fn = native.lib().ornith_moe_b200_ep_dispatch_p2p
    base = 1 << 32
    x, tok, lids, counter, flags = (C.c_void_p(base + (i << 28)) for i in range(5))
    world = 2
    dx = (C.c_void_p * world)(base + (5 << 28), base + (6 << 28))
    di = (C.c_void_p * world)(base + (7 << 28), base + (8 << 28))
    sigs = (C.c_void_p * world)(base + (9 << 28), base + (10 << 28))

    def call(seg=(0, 3, 5), off=(0, 4), cap=8, n=5, T=4, me=1, X=x, ids=lids, d=dx, s=sigs):
        seg_a = (C.c_int32 * len(seg))(*seg)
        off_a = (C.c_int64 * len(off))(*off)
        return fn(X, T, tok, ids, n, seg_a, d, di, off_a, cap, s, world, me, 1, counter, flags, None)

    assert call(n=9, seg=(0, 4, 9)) == INVALID         # more rows than T * world
    assert call(T=8193) == INVALID
    assert call(me=2) == INVALID
    assert call(seg=(0, 3, 4)) == INVALID
    assert call(off=(6, 0)) == INVALID                 # 3 rows at 6..8 of an 8-row buffer
    assert call(off=(0, 7)) == INVALID
    assert call(X=C.c_void_p(base + 8)) == INVALID     # 16-byte token rows
    assert call(ids=C.c_void_p(base + (2 << 28) + 4)) == INVALID
    assert call(d=(C.c_void_p * world)(base + (5 << 28), None)) == INVALID
    assert call(s=(C.c_void_p * world)(None, base + (10 << 28))) == INVALID   # rank 0's flags (this is rank 1)


def test_fixed_peer_exchange_validation_without_device_work(native):
    lib = native.lib()
    base = 1 << 32
    x, lids, epoch, counter, flags, ws = (C.c_void_p(base + (i << 28)) for i in range(6))
    world = 2
    sets = (C.c_void_p * (2 * world))(*[base + ((8 + i) << 28) for i in range(2 * world)])
    sigs = (C.c_void_p * world)(base + (14 << 28), base + (15 << 28))
    d = lib.ornith_moe_b200_ep_fixed_dispatch
    cap = 8192
    assert d(x, lids, 0, sets, sets, cap, sigs, world, 0, epoch, counter, flags, None) == INVALID     # T >= 1
    assert d(x, lids, 4097, sets, sets, cap, sigs, world, 0, epoch, counter, flags, None) == INVALID  # world*T <= 8192
    assert d(x, lids, 4, sets, sets, cap, sigs, world, 2, epoch, counter, flags, None) == INVALID     # me < world
    assert d(C.c_void_p(base + 8), lids, 4, sets, sets, cap, sigs, world, 0, epoch, counter, flags,
             None) == INVALID
    bad = (C.c_void_p * (2 * world))(*[base + ((8 + i) << 28) for i in range(2 * world - 1)], None)
    assert d(x, lids, 4, bad, sets, cap, sigs, world, 0, epoch, counter, flags, None) == INVALID  # every set, rank
    assert d(x, lids, 4, sets, sets, 7, sigs, world, 0, epoch, counter, flags, None) == INVALID   # 8 rows, 7 fit
    assert d(x, lids, 4, sets, sets, cap, sigs, world, 0, epoch, counter, None, None) == INVALID  # flags needed
    r = lib.ornith_moe_b200_ep_fixed_return
    nb = native.get_layout(16).workspace_bytes
    assert r(ws, nb, 9, 16, lids, sets, cap, sigs, world, 0, epoch, counter, flags, None) == INVALID  # world*T > Tcap
    assert r(ws, nb - 1, 8, 16, lids, sets, cap, sigs, world, 0, epoch, counter, flags, None) == INVALID
    assert r(ws, nb, 8, 16, lids, bad, cap, sigs, world, 0, epoch, counter, flags, None) == INVALID
    assert r(ws, nb, 8, 16, lids, sets, 63, sigs, world, 0, epoch, counter, flags, None) == INVALID  # 64 slot rows
    assert r(ws, nb, 8, 16, lids, sets, cap, (C.c_void_p * world)(base, None), world, 0, epoch, counter, flags,
             None) == INVALID                                                               # a peer's flags
    w = lib.ornith_moe_b200_ep_wait_epoch
    assert w(sigs[0], 9, 0, epoch, flags, None) == INVALID
    assert w(None, 2, 0, epoch, flags, None) == INVALID
    assert w(sigs[0], 1, 0, epoch, flags, None) == 0          # one rank: nothing to wait for


def test_peer_wait_limit_setting(native):
    """The limit of the waits on other ranks is a library setting: 1 s by
    default, 1 us .. 60 s accepted, anything else refused unchanged."""
    assert native.peer_wait_limit_ns() == 1_000_000_000
    lib = native.lib()
    try:
        assert lib.ornith_moe_b200_set_peer_wait_limit_ns(999) == INVALID
        assert lib.ornith_moe_b200_set_peer_wait_limit_ns(60_000_000_001) == INVALID
        assert native.peer_wait_limit_ns() == 1_000_000_000
        native.set_peer_wait_limit_ns(5_000_000)
        assert native.peer_wait_limit_ns() == 5_000_000
    finally:
        native.set_peer_wait_limit_ns(1_000_000_000)
