"""CPU: expert-parallel host logic on gloo ranks (world sizes 2 and 4).

The expert compute and the combine are deterministic fakes with the same
slot-ordered fp32 semantics as the kernels, so the test checks the dispatch,
both exchanges and the reassembly bit for bit against a single-rank run."""
import os
import socket
import sys
from pathlib import Path

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

ROOT = Path(__file__).resolve().parents[1]
E, TOP, H = 256, 8, 2048


def fake_rows(x, ids_local, table):
    """Deterministic per-slot rows depending on the token row and the global
    expert (table: global expert of each local bank index)."""
    xf = x.float()
    g = table[ids_local.clamp(min=0).long()].float()
    return (xf.unsqueeze(1) * (g.unsqueeze(2) * 0.01 + 1.0) + g.unsqueeze(2) * 0.5).contiguous()


def valid_ids(ids):
    """Slots that name an expert: -1 is padding, ids outside 0..255 are invalid."""
    return (ids >= 0) & (ids < E)


def fake_combine(rows, weights, ids):
    T = ids.shape[0]
    r = rows.view(T, TOP, H)
    out = torch.zeros((T, H), dtype=torch.float32)
    for s in range(TOP):
        valid = valid_ids(ids[:, s]).unsqueeze(1)
        out = torch.where(valid, out + r[:, s] * weights[:, s:s + 1], out)
    return out


def fake_combine_gathered(rows, row_index, weights, ids):
    """The same sum, reading slot s of token t from rows[row_index[t, s]]."""
    T = ids.shape[0]
    dense = torch.zeros((T, TOP, H), dtype=torch.float32)
    have = row_index >= 0
    dense[have] = rows[row_index[have].long()]
    assert bool((valid_ids(ids) <= have).all()), 'a valid slot came back without a row'
    return fake_combine(dense.view(T * TOP, H), weights, ids)


def fake_partial(x, ids_local, w_local, table):
    """Slot-ordered weighted sum of one rank's own slots (padding: -1 ids)."""
    r = fake_rows(x, ids_local, table)
    out = torch.zeros((x.shape[0], H), dtype=torch.float32)
    for s in range(TOP):
        valid = (ids_local[:, s] >= 0).unsqueeze(1)
        out = torch.where(valid, out + r[:, s] * w_local[:, s:s + 1], out)
    return out


def rank_partial_reference(x, ids, weights, placement, world):
    """Sum over ranks, in rank order, of each rank's slot-ordered partial."""
    import __graft_entry__ as g
    g.load_package()
    from ornith_b200 import ep
    owner, lid = ep.map_ids(ids, placement)
    out = torch.zeros((x.shape[0], H), dtype=torch.float32)
    for d in range(world):
        mine = owner == d
        table = torch.tensor(placement.experts_of(d))
        part = fake_partial(x, torch.where(mine, lid, torch.full_like(lid, -1)),
                            torch.where(mine, weights, torch.zeros_like(weights)), table)
        out = torch.where(mine.any(dim=1, keepdim=True), out + part, out)
    return out


def _port():
    with socket.socket() as s:
        s.bind(('127.0.0.1', 0))
        return s.getsockname()[1]


def _inputs(rank, T, seed):
    gen = torch.Generator().manual_seed(seed + rank)
    x = torch.randn((T, H), generator=gen).to(torch.bfloat16)
    logits = torch.randn((T, E), generator=gen)
    ids = torch.topk(logits, TOP, dim=1).indices.to(torch.int32)
    ids[::5, 3] = -1                   # padding slots
    ids[1, :] = -1                     # a token with no expert at all
    ids[4, 2] = 300                    # invalid ids: no rank owns them, the slot is skipped
    ids[6, 7] = -5
    weights = torch.softmax(torch.randn((T, TOP), generator=gen), dim=1)
    return x, ids, weights


def _worker(rank, world, port, T, seed, q, mode, balanced):
    try:
        os.environ['MASTER_ADDR'] = '127.0.0.1'
        os.environ['MASTER_PORT'] = str(port)
        dist.init_process_group('gloo', rank=rank, world_size=world)
        sys.path.insert(0, str(ROOT))
        import __graft_entry__ as g
        g.load_package()
        from ornith_b200 import ep
        x, ids, weights = _inputs(rank, T, seed)
        if balanced:  # a load-balanced placement from (identical) skewed loads
            loads = torch.arange(E, dtype=torch.float64).flip(0) ** 2
            placement = ep.balanced_placement(loads, world)
        else:
            placement = ep.contiguous_placement(world)
        table = torch.tensor(placement.experts_of(rank))

        def compute(xr, ir, n_valid):
            assert n_valid == int((ir >= 0).sum())      # the host count the exchange delivered
            return fake_rows(xr, ir, table)[ir >= 0] if xr.shape[0] else torch.zeros((0, H))

        def compute_block(xa, ia):
            return fake_rows(xa, ia, table)

        def compute_partial(xr, ir, wr):
            return fake_partial(xr, ir, wr, table) if xr.shape[0] else torch.zeros((0, H))

        if mode == 'fixed':
            out = ep.ep_layer_fixed(None, world, x, ids, weights, compute_block, fake_combine_gathered, placement)
        elif mode == 'compact':
            out = ep.ep_layer(None, world, x, ids, weights, compute, fake_combine_gathered, placement)
        elif mode == 'peer':      # the return over peer memory, its stores emulated on the host
            me = dist.get_rank()
            try:                  # too small a capacity: every rank refuses, after the same collective
                ep.dispatch_with_matrix(None, world, me, ids, placement, capacity=1)
                raise AssertionError('capacity 1 was accepted')
            except ValueError:
                pass
            plan, recv_counts, back_counts, offsets, x_offsets = ep.dispatch_with_matrix(None, world, me, ids,
                                                                                        placement)
            plan2, recv2, back2 = ep.dispatch_with_counts(None, world, ids, placement)
            assert (recv_counts, back_counts) == (recv2, back2)
            assert (plan.send_counts, plan.home_counts) == (plan2.send_counts, plan2.home_counts)
            x_recv, ids_recv = ep.exchange_rows(None, world, plan, x, recv_counts)
            # emulated dispatch stores: each home's sent rows at its offset in this rank's token buffer
            sent = [None] * world
            dist.all_gather_object(sent, (x[plan.token_index], plan.local_ids, plan.send_counts, x_offsets))
            x_buf = torch.full((sum(recv_counts), H), float('nan')).to(torch.bfloat16)
            ids_buf = torch.full((sum(recv_counts), TOP), -77, dtype=torch.int32)
            for x_h, ids_h, send_h, off_h in sent:
                lo, k = sum(send_h[:me]), send_h[me]
                assert 0 <= off_h[me] and off_h[me] + k <= x_buf.shape[0]
                x_buf[off_h[me]:off_h[me] + k] = x_h[lo:lo + k]
                ids_buf[off_h[me]:off_h[me] + k] = ids_h[lo:lo + k]
            assert torch.equal(x_buf.view(torch.int16), x_recv.view(torch.int16)) and torch.equal(ids_buf, ids_recv)
            rows = compute(x_recv, ids_recv, sum(back_counts))
            gathered = [None] * world
            dist.all_gather_object(gathered, (rows, back_counts, offsets))
            got = torch.full((sum(plan.home_counts), H), float('nan'))   # an unwritten row would show
            for rows_d, back_d, off_d in gathered:
                lo, k = sum(back_d[:me]), back_d[me]
                assert 0 <= off_d[me] and off_d[me] + k <= got.shape[0]
                got[off_d[me]:off_d[me] + k] = rows_d[lo:lo + k]
            out = fake_combine_gathered(got, ep.route_row_index(T, plan, got.device), weights, ids)
        elif mode == 'fixed_peer':   # the fixed exchange over peer memory, its stores emulated on the host
            me = dist.get_rank()
            owner, lid = ep.map_ids(ids, placement)
            dest = torch.arange(world).view(-1, 1, 1)
            local = torch.where(owner.unsqueeze(0) == dest, lid.unsqueeze(0),
                                torch.full_like(lid, -1).unsqueeze(0)).to(torch.int32)
            sent = [None] * world        # dispatch: rank d's row h*T + t holds token t of rank h
            dist.all_gather_object(sent, (x, local))
            x_all = torch.cat([x_h for x_h, _ in sent])
            ids_all = torch.cat([local_h[me] for _, local_h in sent])
            rows = fake_rows(x_all, ids_all, table)                     # [world*T, 8, H]
            back = [None] * world        # return: home h's row t*8 + s from the slot's owner
            dist.all_gather_object(back, (rows, ids_all))
            res = torch.full((T * TOP, H), float('nan'))
            for rows_d, ids_d in back:
                for t in range(T):
                    for s_ in range(TOP):
                        if ids_d[me * T + t, s_] >= 0:
                            assert bool(torch.isnan(res[t * TOP + s_]).all()), 'two owners stored one slot'
                            res[t * TOP + s_] = rows_d[me * T + t, s_]
            row_index = torch.where((ids >= 0) & (ids < E), torch.arange(T * TOP, dtype=torch.int32).view(T, TOP),
                                    torch.full((T, TOP), -1, dtype=torch.int32))
            out = fake_combine_gathered(res, row_index, weights, ids)
        elif mode == 'chunked':   # pipelined chunks; T + 1 chunks leaves one chunk empty
            chunks = 3 if world == 2 else T + 1
            out = ep.ep_layer_chunked(None, world, x, ids, weights, compute, fake_combine_gathered, placement,
                                      chunks)
        elif mode == 'fixed_partial':
            out = ep.ep_layer_fixed_partial(None, world, x, ids, weights, compute_partial, fake_combine_gathered,
                                            placement)
        else:
            out = ep.ep_layer_partial(None, world, x, ids, weights, compute_partial, fake_combine_gathered,
                                      placement)
        if mode.endswith('partial'):
            ref = rank_partial_reference(x, ids, weights, placement, world)
        else:
            clean = torch.where(valid_ids(ids), ids, torch.full_like(ids, -1))
            ref = fake_combine(fake_rows(x, clean, torch.arange(E)).view(T * TOP, H), weights, ids)
        q.put((rank, bool(torch.equal(out, ref)), ''))
        dist.barrier()
        dist.destroy_process_group()
    except Exception as exc:  # report instead of hanging the parent
        q.put((rank, False, repr(exc)))


@pytest.mark.parametrize('balanced', [False, True])
@pytest.mark.parametrize('mode', ['compact', 'chunked', 'peer', 'fixed', 'fixed_peer', 'compact_partial',
                                  'fixed_partial'])
@pytest.mark.parametrize('world,T', [(2, 16), (4, 9)])
def test_ep_dispatch_combine_matches_single_rank(world, T, mode, balanced):
    ctx = mp.get_context('spawn')
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, T, 1234, q, mode, balanced)) for r in range(world)]
    for p in procs:
        p.start()
    results = [q.get(timeout=180) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
    for rank, equal, err in results:
        assert equal, (rank, err)
    assert all(p.exitcode == 0 for p in procs)


def test_build_dispatch_groups_by_owner():
    sys.path.insert(0, str(ROOT))
    import __graft_entry__ as g
    g.load_package()
    from ornith_b200 import ep
    ids = torch.tensor([[0, 200, 5, -1, 130, 64, 63, 255], [-1] * 8, [129, 128, 127, 1, 2, 3, 4, 6]],
                       dtype=torch.int32)
    plan = ep.build_dispatch(ids, 2)
    assert plan.send_counts == [2, 2]
    assert plan.token_index.tolist() == [0, 2, 0, 2]
    assert plan.local_ids[0].tolist() == [0, -1, 5, -1, -1, 64, 63, -1]
    assert plan.local_ids[2].tolist() == [-1, 72, -1, -1, 2, -1, -1, 127]
    assert plan.local_ids[3].tolist() == [1, 0, -1, -1, -1, -1, -1, -1]
    assert int(plan.slot_mask.sum()) == int((ids >= 0).sum())


def test_balanced_placement_properties():
    import __graft_entry__ as g
    g.load_package()
    from ornith_b200 import ep
    loads = torch.rand(E, generator=torch.Generator().manual_seed(3)) ** 4
    for world in (2, 4, 8):
        pl = ep.balanced_placement(loads, world)
        per = [ep.Placement.experts_of(pl, r) for r in range(world)]
        assert sorted(sum(per, [])) == list(range(E))                   # every expert exactly once
        assert all(len(x) == E // world for x in per)                   # equal banks
        assert all(pl.local[e] == i for x in per for i, e in enumerate(x))
        rank_load = [float(loads[x].sum()) for x in per]
        contiguous = [float(loads[r * E // world:(r + 1) * E // world].sum()) for r in range(world)]
        assert max(rank_load) <= max(contiguous) + 1e-9
        assert max(rank_load) - min(rank_load) <= float(loads.max()) + 1e-9  # greedy bound
