"""Expert parallelism for the routed-MoE layer over torch.distributed.

The reference runs one rank and refuses EP (plugin-site/ornith_g256/moe_base.py:34-39);
this module adds it.  Every rank owns 256/n routed experts: by default rank r
owns [r*256/n, (r+1)*256/n); a Placement can assign them by routed load
instead (balanced_placement).  The shared expert is replicated and runs on
each rank for its own tokens.  One layer call on every rank, for the rank's own
tokens, in one of two exchange modes.

compact (any batch; ranks may hold different token counts):
  1. dispatch plan: for every destination rank d, the local tokens with at
     least one expert on d (deduplicated per (token, rank)), with their eight
     ids rewritten to d's local expert numbers (-1 for slots owned elsewhere);
     on GPUs one launch of ornith_moe_b200_ep_plan (NativePlanner), on any
     device the equivalent torch operations (TorchPlanner);
  2. exchange: one all_to_all of (tokens sent, slots to come back) per rank
     pair and a single host synchronisation for every split size of the
     layer, then token rows (bf16 pairs carried as int32) and local ids
     (all_to_all_single with variable splits; NCCL on GPUs, gloo on CPU);
  3. expert compute on the received rows with the local banks; the fp32
     down projections of the valid slots are gathered in (token, slot) order;
  4. return exchange of those rows, one per (token, slot) owned by d;
  5. home combine: slot-ordered weighted sum into bf16 with the same
     arithmetic as the single-GPU layer, so the result is bit-identical to it.
     It reads the returned rows where they arrived, through a (token, slot)
     -> row index built on the device.

fixed (small batches, the same token count on every rank): no counts and no
host synchronisation.  Every rank gathers every rank's token rows
(all_gather) and receives, per source rank, the eight ids of each of its
tokens in local numbering (-1 where another rank owns the slot).  The expert
compute returns the route-ordered [T, 8, 2048] block of each source rank,
padding slots included, and one all_to_all of equal blocks brings them home;
the row index of slot s of token t is (owner * T + t) * 8 + s.

Both modes also have a rank-partial combine (combine='partial'): the expert
rank weights and sums its own slots of each token in slot order (the layer's
own fp32 combine, before bf16 rounding) and returns one fp32 row per (token,
rank) instead of one per (token, slot); the home rank adds the ranks' partial
rows in rank order and rounds to bf16.  The association differs from the
single-GPU sum, so the result agrees to fp32 rounding (within the north-star
tolerance) rather than bit for bit, for up to 8x less return traffic.

These collectives are the layer's only exchange.  Every rank takes the same
collective steps in the same order, zero-sized messages included.
"""
import ctypes as C
from dataclasses import dataclass

import torch
import torch.distributed as dist

E, TOP, H = 256, 8, 2048


@dataclass
class Placement:
    """Which rank holds each routed expert, and at which index of its banks."""
    rank: torch.Tensor   # int64 [256]
    local: torch.Tensor  # int64 [256]

    def experts_of(self, r):
        """Global expert ids held by rank r, in bank order."""
        mine = (self.rank == r).nonzero().flatten()
        return mine[torch.argsort(self.local[mine])].tolist()


def contiguous_placement(world, device=None):
    e = torch.arange(E, device=device)
    epr = E // world
    return Placement(torch.div(e, epr, rounding_mode='floor'), e % epr)


def balanced_placement(counts, world, device=None):
    """Equal expert counts per rank, routed load balanced greedily: experts in
    decreasing load go to the least-loaded rank that still has room (ties to the
    lower rank, so every rank computes the same placement from the same counts)."""
    counts = [float(c) for c in torch.as_tensor(counts).flatten().tolist()]
    if len(counts) != E or E % world:
        raise ValueError('balanced_placement needs 256 expert loads and a world size dividing 256')
    epr = E // world
    load, fill = [0.0] * world, [0] * world
    rank, local = [0] * E, [0] * E
    for e in sorted(range(E), key=lambda i: (-counts[i], i)):
        r = min((r for r in range(world) if fill[r] < epr), key=lambda r: (load[r], r))
        rank[e], local[e] = r, fill[r]
        load[r] += counts[e]
        fill[r] += 1
    return Placement(torch.tensor(rank, device=device), torch.tensor(local, device=device))


def map_ids(ids, placement):
    """(owning rank, index in the owner's banks) of every slot; -1 for padding
    and for ids outside 0..255, which no rank owns (the home rank's combine
    raises flag 4 for the latter, as the single-GPU layer does)."""
    valid = (ids >= 0) & (ids < E)
    e = torch.where(valid, ids, torch.zeros_like(ids)).long()
    neg = torch.full_like(ids, -1)
    return (torch.where(valid, placement.rank[e].to(ids.dtype), neg),
            torch.where(valid, placement.local[e].to(ids.dtype), neg))


@dataclass
class DispatchPlan:
    send_counts: list          # tokens sent to each rank
    home_counts: list          # (token, slot) rows each rank sends back
    token_index: torch.Tensor  # [sum(send_counts)] local token of each sent row, grouped by rank
    local_ids: torch.Tensor    # [sum(send_counts), 8] ids in the destination's numbering, -1 elsewhere
    slot_mask: torch.Tensor    # [sum(send_counts), 8] True where the slot is owned by the destination
    dest: torch.Tensor = None  # [sum(send_counts)] destination rank of each sent row
    row_index: torch.Tensor = None  # [T, 8] row of each slot among the returned rows, when the planner made it


def _owner_mask(ids, world, placement):
    """Device half of the dispatch plan: (mask [world, T, 8] of the slots each
    rank owns, local ids, int64 [world, 2] = (tokens sent, slots to come back)
    per destination).  No host synchronisation."""
    placement = placement or contiguous_placement(world, ids.device)
    owner, lid = map_ids(ids, placement)
    dest = torch.arange(world, device=ids.device).view(-1, 1, 1)
    mask = owner.unsqueeze(0) == dest                      # [world, T, 8]
    counts = torch.stack([mask.any(dim=2).sum(dim=1), mask.sum(dim=(1, 2))], dim=1).to(torch.int64)
    return mask, lid, counts.contiguous()


def _plan_from_mask(mask, lid, ids, send_counts, home_counts):
    """Host-sized half of the plan: the (destination, token) pairs, grouped by
    destination and ascending in token; nonzero_static with the known total
    needs no host synchronisation."""
    sent = torch.nonzero_static(mask.any(dim=2), size=sum(send_counts))   # (d, t)
    d, tok = sent[:, 0], sent[:, 1]
    slot_mask = mask[d, tok]
    local = torch.where(slot_mask, lid[tok], torch.full_like(slot_mask, -1, dtype=ids.dtype))
    return DispatchPlan(send_counts, home_counts, tok, local.to(torch.int32).contiguous(), slot_mask, d)


def build_dispatch(ids, world, placement=None):
    """Group each token's slots by owning rank (pure tensor logic, any device;
    one host synchronisation for the split sizes)."""
    mask, lid, counts = _owner_mask(ids, world, placement)
    host = counts.tolist()
    return _plan_from_mask(mask, lid, ids, [int(r[0]) for r in host], [int(r[1]) for r in host])


class TorchPlanner:
    """The dispatch plan from torch operations on any device (the CPU ranks
    of the tests use it): start(ids) -> (state, counts int64 [world, 2]) with
    no host synchronisation; finish(state, ids, send_counts, home_counts) ->
    DispatchPlan once the split sizes are known on the host."""

    def __init__(self, world, placement=None):
        self.world, self.placement = world, placement

    def start(self, ids):
        mask, lid, counts = _owner_mask(ids, self.world, self.placement)
        return (mask, lid), counts

    def finish(self, state, ids, send_counts, home_counts):
        mask, lid = state
        return _plan_from_mask(mask, lid, ids, send_counts, home_counts)


class NativePlanner:
    """The same plan from one launch of ornith_moe_b200_ep_plan (CUDA ids),
    row index included; its outputs equal TorchPlanner's."""

    def __init__(self, world, placement, device):
        from . import native
        self.native, self.world = native, world
        self.owner = placement.rank.to(device=device, dtype=torch.int32).contiguous()
        self.local = placement.local.to(device=device, dtype=torch.int32).contiguous()

    def start(self, ids):
        out = self.native.ep_plan(ids.contiguous(), self.owner, self.local, self.world)
        return out, out[0]

    def finish(self, state, ids, send_counts, home_counts):
        _, token_index, dest, local_ids, slot_mask, row_index = state
        n = sum(send_counts)
        return DispatchPlan(send_counts, home_counts, token_index[:n], local_ids[:n], slot_mask[:n], dest[:n],
                            row_index)


def dispatch_with_counts(group, world, ids, placement=None, planner=None):
    """The dispatch plan plus what every peer sends here: one all_to_all of
    the (tokens sent, slots to come back) pairs and the layer's single host
    synchronisation, for all four split lists.  Returns (plan, recv_counts:
    token rows arriving from each rank, back_counts: (token, slot) rows this
    rank returns to each rank)."""
    planner = planner or TorchPlanner(world, placement)
    state, counts = planner.start(ids)
    got = torch.empty_like(counts)
    _a2a(group, got, counts, [1] * world, [1] * world)
    both = torch.cat([counts, got], dim=1).tolist()          # the single host synchronisation
    plan = planner.finish(state, ids, [int(r[0]) for r in both], [int(r[1]) for r in both])
    return plan, [int(r[2]) for r in both], [int(r[3]) for r in both]


def peer_offsets(matrix, me):
    """From the gathered count matrix (matrix[src][d] = (tokens src sends to
    d, (token, slot) rows d returns to src)) the split lists of rank `me` and,
    for the return over peer memory, the first row of its block in every home
    rank's receive buffer: home h holds the blocks of ranks 0, 1, ... in rank
    order, so rank me's block starts after the rows h gets from ranks below me.
    Returns (send_counts, home_counts, recv_counts, back_counts, offsets)."""
    world = len(matrix)
    send = [int(matrix[me][d][0]) for d in range(world)]
    home = [int(matrix[me][d][1]) for d in range(world)]
    recv = [int(matrix[src][me][0]) for src in range(world)]
    back = [int(matrix[src][me][1]) for src in range(world)]
    offsets = [sum(int(matrix[h][d][1]) for d in range(me)) for h in range(world)]
    return send, home, recv, back, offsets


def dispatch_offsets(matrix, me):
    """For the dispatch over peer memory: the first row of this rank's block
    of token rows in every expert rank's receive buffer (after the rows that
    expert rank d gets from lower ranks)."""
    world = len(matrix)
    return [sum(int(matrix[h][d][0]) for h in range(me)) for d in range(world)]


def dispatch_with_matrix(group, world, me, ids, placement=None, planner=None, capacity=None):
    """dispatch_with_counts with an all_gather of every rank's counts instead
    of the all_to_all, so that this rank also learns where its returned rows
    go in each home rank's buffer; still one host synchronisation.  Returns
    (plan, recv_counts, back_counts, return offsets, dispatch offsets).  With
    `capacity`, every rank raises ValueError when any rank would receive more
    token rows than that."""
    planner = planner or TorchPlanner(world, placement)
    state, counts = planner.start(ids)
    parts = [torch.empty_like(counts) for _ in range(world)]
    dist.all_gather(parts, counts.contiguous(), group=group)
    matrix = torch.stack(parts).tolist()                   # the single host synchronisation
    if capacity is not None:
        # every rank sees the same matrix, so all ranks refuse together
        most = max(sum(int(matrix[h][d][0]) for h in range(world)) for d in range(world))
        if most > capacity:
            raise ValueError(f'expert-parallel receive of {most} rows on one rank exceeds capacity {capacity}')
    send, home, recv, back, offsets = peer_offsets(matrix, me)
    return planner.finish(state, ids, send, home), recv, back, offsets, dispatch_offsets(matrix, me)


def _a2a(group, out, inp, out_splits, in_splits):
    dist.all_to_all_single(out, inp, out_splits, in_splits, group=group)


def exchange_rows(group, world, plan, x, recv_counts):
    """Send each rank its token rows and local ids; returns (x_recv, ids_recv)."""
    dev = x.device
    n_in = sum(recv_counts)
    x_words = x.contiguous().view(torch.int32)[plan.token_index].contiguous()   # [n, 1024]
    x_recv = torch.empty((n_in, H // 2), dtype=torch.int32, device=dev)
    _a2a(group, x_recv, x_words, recv_counts, plan.send_counts)
    ids_recv = torch.empty((n_in, TOP), dtype=torch.int32, device=dev)
    _a2a(group, ids_recv, plan.local_ids, recv_counts, plan.send_counts)
    return x_recv.view(x.dtype), ids_recv


def return_rows(group, world, plan, back_counts, out_rows):
    """Send every (token, slot) row computed here back to the token's home rank.

    out_rows: fp32 [n_valid, 2048], one row per received slot with a valid
    local id, in (token, slot) order; back_counts: those rows per source rank.
    Returns the home-side fp32 rows [n_sent_slots, 2048] in the order of
    plan.slot_mask."""
    got = torch.empty((sum(plan.home_counts), H), dtype=torch.float32, device=out_rows.device)
    _a2a(group, got, out_rows, plan.home_counts, back_counts)
    return got


def route_row_index(T, plan, device):
    """int32 [T, 8]: the row of `got` (return_rows) holding slot s of token t,
    -1 for slots no rank returned (padding ids).  No host synchronisation:
    rows arrive in slot_mask order, so the row of a masked entry is the count
    of masked entries before it; each slot has one owner, so the per-token
    maximum over destinations picks it.  A plan that carries its row index
    (NativePlanner) returns that."""
    if plan.row_index is not None:
        return plan.row_index
    flat = plan.slot_mask.reshape(-1).to(torch.int32)
    dense = torch.where(plan.slot_mask, (torch.cumsum(flat, 0, dtype=torch.int32) - 1).view_as(plan.slot_mask),
                        torch.full_like(plan.slot_mask, -1, dtype=torch.int32))
    idx = torch.full((T, TOP), -1, dtype=torch.int32, device=device)
    return idx.scatter_reduce_(0, plan.token_index.view(-1, 1).expand(-1, TOP), dense, 'amax')


def dispatch_chunks(group, world, ids, placement, bounds, planner=None):
    """dispatch_with_counts for the token ranges `bounds` of this rank at
    once: one all_to_all of every chunk's (tokens sent, slots to come back)
    pairs and one host synchronisation.  Returns [(plan, recv_counts,
    back_counts)] per chunk."""
    planner = planner or TorchPlanner(world, placement)
    parts = [planner.start(ids[lo:hi]) for lo, hi in bounds]
    counts = torch.stack([c for _, c in parts], dim=1).contiguous()          # [world, chunks, 2]
    got = torch.empty_like(counts)
    n = len(bounds) * 2
    _a2a(group, got.view(world, n), counts.view(world, n), [1] * world, [1] * world)
    both = torch.cat([counts, got], dim=2).tolist()                         # the single host synchronisation
    out = []
    for c, ((lo, hi), (state, _)) in enumerate(zip(bounds, parts)):
        rows = [both[d][c] for d in range(world)]
        plan = planner.finish(state, ids[lo:hi], [int(r[0]) for r in rows], [int(r[1]) for r in rows])
        out.append((plan, [int(r[2]) for r in rows], [int(r[3]) for r in rows]))
    return out


def ep_layer_chunked(group, world, x, ids, weights, compute, combine, placement=None, chunks=2, planner=None):
    """ep_layer over `chunks` contiguous token ranges, pipelined so that the
    return exchange of chunk c overlaps the expert compute of chunk c + 1:
    per chunk the row exchange of the next chunk is issued before this
    chunk's return, which is asynchronous (collectives of one group run in
    issue order, so the other order would serialise them).  Every rank must
    use the same chunk count.  Tokens are independent, so the output equals
    ep_layer's bit for bit."""
    T = x.shape[0]
    bounds = [(T * c // chunks, T * (c + 1) // chunks) for c in range(chunks)]
    plans = dispatch_chunks(group, world, ids, placement, bounds, planner)

    def send(c):
        lo, hi = bounds[c]
        plan, recv_counts, _ = plans[c]
        return exchange_rows(group, world, plan, x[lo:hi], recv_counts)

    pending = []
    nxt = send(0)
    for c in range(chunks):
        x_recv, ids_recv = nxt
        plan, _, back_counts = plans[c]
        rows = compute(x_recv, ids_recv, sum(back_counts))
        if c + 1 < chunks:
            nxt = send(c + 1)
        got = torch.empty((sum(plan.home_counts), H), dtype=torch.float32, device=rows.device)
        work = dist.all_to_all_single(got, rows, plan.home_counts, back_counts, group=group, async_op=True)
        pending.append((work, got, rows))
    outs = []
    for c, (work, got, _) in enumerate(pending):
        work.wait()
        lo, hi = bounds[c]
        outs.append(combine(got, route_row_index(hi - lo, plans[c][0], got.device), weights[lo:hi], ids[lo:hi]))
    return torch.cat(outs)


def ep_layer(group, world, x, ids, weights, compute, combine, placement=None, planner=None):
    """One expert-parallel layer call, compact exchange.

    compute(x_recv, ids_recv, n_valid) -> fp32 [n_valid, 2048]: the rows of the
    received slots with a valid id, in (token, slot) order (n_valid, known on
    the host, is their count); combine(rows [n, 2048], row_index [T, 8],
    weights, ids) -> output.  Both are injected so that the host logic also
    runs on CPU ranks.  planner: how the dispatch plan is made (TorchPlanner
    by default)."""
    plan, recv_counts, back_counts = dispatch_with_counts(group, world, ids, placement, planner)
    x_recv, ids_recv = exchange_rows(group, world, plan, x, recv_counts)
    out_rows = compute(x_recv, ids_recv, sum(back_counts))
    got = return_rows(group, world, plan, back_counts, out_rows)
    return combine(got, route_row_index(x.shape[0], plan, got.device), weights, ids)


def partial_row_index(T, world, token_index, dest, device):
    """int32 [T, 8] for combine_gathered: column d holds the row of rank d's
    partial for the token (-1 where the token sent nothing to d); columns
    >= world are -1.  token_index / dest: token and rank of each returned row,
    in arrival order."""
    idx = torch.full((T, TOP), -1, dtype=torch.int32, device=device)
    idx[token_index, dest] = torch.arange(token_index.numel(), dtype=torch.int32, device=device)
    return idx


def rank_sum(combine, got, row_index, like_weights):
    """Home-side sum of the ranks' partial rows in rank order, through the
    slot-ordered combine with unit weights (x * 1 is exact) and the ranks as
    slots."""
    ones = torch.ones_like(like_weights)
    ids = torch.where(row_index >= 0, torch.zeros_like(row_index), torch.full_like(row_index, -1))
    return combine(got, row_index, ones, ids)


def ep_layer_partial(group, world, x, ids, weights, compute_partial, combine, placement=None, planner=None):
    """Compact exchange with the rank-partial combine.

    compute_partial(x_recv, ids_recv, w_recv) -> fp32 [n_recv, 2048]: per
    received token, its routing weights times this rank's projections summed
    in slot order."""
    plan, recv_counts, _ = dispatch_with_counts(group, world, ids, placement, planner)
    x_recv, ids_recv = exchange_rows(group, world, plan, x, recv_counts)
    w_send = torch.where(plan.slot_mask, weights[plan.token_index], torch.zeros_like(weights[plan.token_index]))
    w_recv = torch.empty((sum(recv_counts), TOP), dtype=torch.float32, device=x.device)
    _a2a(group, w_recv, w_send.contiguous(), recv_counts, plan.send_counts)
    part = compute_partial(x_recv, ids_recv, w_recv)
    got = torch.empty((plan.token_index.numel(), H), dtype=torch.float32, device=x.device)
    _a2a(group, got, part.contiguous(), plan.send_counts, recv_counts)
    return rank_sum(combine, got, partial_row_index(x.shape[0], world, plan.token_index, plan.dest, x.device),
                    weights)


def ep_layer_fixed(group, world, x, ids, weights, compute_block, combine, placement=None):
    """One expert-parallel layer call, fixed-size exchange (same T on every rank).

    compute_block(x_all [world*T, 2048], ids_all [world*T, 8]) -> fp32
    [world*T, 8, 2048], route-ordered (padding slots unspecified)."""
    T = x.shape[0]
    placement = placement or contiguous_placement(world, ids.device)
    owner, lid = map_ids(ids, placement)
    dest = torch.arange(world, device=ids.device).view(-1, 1, 1)
    local = torch.where(owner.unsqueeze(0) == dest, lid.unsqueeze(0),
                        torch.full_like(owner.unsqueeze(0), -1)).to(torch.int32).contiguous()   # [world, T, 8]
    x_all = torch.empty((world * T, H // 2), dtype=torch.int32, device=x.device)
    dist.all_gather_into_tensor(x_all, x.contiguous().view(torch.int32), group=group)
    ids_all = torch.empty_like(local)
    dist.all_to_all_single(ids_all, local, group=group)
    rows = compute_block(x_all.view(x.dtype), ids_all.view(world * T, TOP))
    got = torch.empty_like(rows)
    dist.all_to_all_single(got, rows, group=group)        # block d: rank d's rows for my tokens
    t = torch.arange(T, device=ids.device, dtype=torch.int32).view(-1, 1)
    s = torch.arange(TOP, device=ids.device, dtype=torch.int32).view(1, -1)
    row_index = torch.where(owner >= 0, (owner.to(torch.int32) * T + t) * TOP + s, torch.full_like(owner, -1))
    return combine(got.view(world * T * TOP, H), row_index.to(torch.int32).contiguous(), weights, ids)


def ep_layer_fixed_partial(group, world, x, ids, weights, compute_partial, combine, placement=None):
    """Fixed-size exchange with the rank-partial combine: one fp32 [T, 2048]
    block per rank comes home (no host synchronisation)."""
    T = x.shape[0]
    placement = placement or contiguous_placement(world, ids.device)
    owner, lid = map_ids(ids, placement)
    dest = torch.arange(world, device=ids.device).view(-1, 1, 1)
    mine = owner.unsqueeze(0) == dest                                                      # [world, T, 8]
    local = torch.where(mine, lid.unsqueeze(0), torch.full_like(owner.unsqueeze(0), -1)).to(torch.int32).contiguous()
    w_local = torch.where(mine, weights.unsqueeze(0), torch.zeros_like(weights).unsqueeze(0)).contiguous()
    x_all = torch.empty((world * T, H // 2), dtype=torch.int32, device=x.device)
    dist.all_gather_into_tensor(x_all, x.contiguous().view(torch.int32), group=group)
    ids_all = torch.empty_like(local)
    dist.all_to_all_single(ids_all, local, group=group)
    w_all = torch.empty_like(w_local)
    dist.all_to_all_single(w_all, w_local, group=group)
    part = compute_partial(x_all.view(x.dtype), ids_all.view(world * T, TOP), w_all.view(world * T, TOP))
    got = torch.empty_like(part)
    dist.all_to_all_single(got, part.contiguous(), group=group)    # block d: rank d's partials for my tokens
    t = torch.arange(T, device=ids.device, dtype=torch.int32).view(-1, 1)
    d = torch.arange(TOP, device=ids.device, dtype=torch.int32).view(1, -1)
    has = (mine.any(dim=2).t() if world == TOP else
           torch.cat([mine.any(dim=2).t(), torch.zeros((T, TOP - world), dtype=torch.bool, device=ids.device)], 1))
    row_index = torch.where(has, d * T + t, torch.full_like(has, -1, dtype=torch.int32))
    return rank_sum(combine, got.view(world * T, H), row_index.contiguous(), weights)


class _DeviceArray:
    """A device range described by __cuda_array_interface__ (v3), so that
    torch.as_tensor can view memory this module allocated itself."""

    def __init__(self, address, shape, typestr, strides=None):
        self.__cuda_array_interface__ = {'shape': tuple(shape), 'typestr': typestr, 'data': (int(address), False),
                                         'strides': None if strides is None else tuple(strides), 'version': 3}


class PeerExchange:
    """This rank's receive buffers for the exchanges over NVLink peer memory,
    shared with the other ranks of the node through CUDA IPC: token rows bf16
    [cap_tokens, 2048] and their local ids int32 [cap_tokens, 8] (dispatch),
    fp32 result rows [cap_rows, 2048] (return), then two flag arrays (return,
    dispatch) of 2*world uint32 words each: the epoch every rank raised, then
    its status word (its flag-64 bit).  Made collectively (every rank at
    once); close() collectively before the process group goes away.

    dispatch() stores this rank's sent token rows into the expert ranks'
    buffers (ornith_moe_b200_ep_dispatch_p2p), ret() stores its computed rows
    into the home ranks' buffers (ornith_moe_b200_ep_return_p2p); each raises
    this rank's flag at the receivers, and wait_*() waits, bounded, for the
    other ranks' flags of the same call (ornith_moe_b200_ep_wait_signals)."""

    def __init__(self, group, world, me, cap_tokens, cap_rows, device):
        from . import native
        if not 1 <= world <= 8:
            raise ValueError('the peer-memory exchange serves 1..8 ranks of one node')
        self.native, self.group, self.world, self.me = native, group, world, me
        self.cap_tokens, self.cap_rows = int(cap_tokens), int(cap_rows)

        def up(n):
            return (n + 255) // 256 * 256
        self.x_offset = 0
        self.ids_offset = up(self.cap_tokens * H * 2)
        self.rows_offset = self.ids_offset + up(self.cap_tokens * TOP * 4)
        self.flag_offset = self.rows_offset + up(self.cap_rows * H * 4)
        self.base = native.ep_buffer_alloc(self.flag_offset + 256)
        self.peers = {}
        try:
            handles = [None] * world
            dist.all_gather_object(handles, native.ep_ipc_handle(self.base), group=group)
            for r in range(world):
                if r != me:
                    self.peers[r] = native.ep_ipc_open(handles[r])
        except BaseException:
            self._release()
            raise
        bases = [self.base if r == me else self.peers[r] for r in range(world)]

        def table(offset):
            return (C.c_void_p * world)(*[b + offset for b in bases])
        self.dst_x, self.dst_ids, self.dst_rows = table(self.x_offset), table(self.ids_offset), table(self.rows_offset)
        self.return_flags, self.dispatch_flags = table(self.flag_offset), table(self.flag_offset + 8 * world)
        self.x = torch.as_tensor(_DeviceArray(self.base + self.x_offset, (self.cap_tokens, H), '<i2'),
                                 device=device).view(torch.bfloat16)
        self.ids = torch.as_tensor(_DeviceArray(self.base + self.ids_offset, (self.cap_tokens, TOP), '<i4'),
                                   device=device)
        self.rows = torch.as_tensor(_DeviceArray(self.base + self.rows_offset, (self.cap_rows, H), '<f4'),
                                    device=device)
        self.counters = torch.zeros(2, dtype=torch.int32, device=device)
        self.epoch = 0

    @staticmethod
    def _segments(counts):
        seg = [0]
        for c in counts:
            seg.append(seg[-1] + int(c))
        return seg

    def dispatch(self, x, plan, offsets, flags):
        """Home side: the plan's sent rows into the expert ranks' token buffers."""
        self.epoch = (self.epoch + 1) & 0xFFFFFFFF
        self.native.ep_dispatch_p2p(x, plan.token_index, plan.local_ids, self._segments(plan.send_counts),
                                    self.dst_x, self.dst_ids, offsets, self.cap_tokens, self.dispatch_flags,
                                    self.world, self.me, self.epoch, self.counters[0:1], flags)

    def wait_dispatch(self, flags):
        self.native.ep_wait_signals(self.base + self.flag_offset + 8 * self.world, self.world, self.me, self.epoch,
                                    flags)

    def ret(self, workspace, T, capacity, route_index, back_counts, offsets, flags):
        """Expert side: the computed rows into the home ranks' result buffers."""
        self.native.ep_return_p2p(workspace, T, capacity, route_index, self._segments(back_counts), self.dst_rows,
                                  offsets, self.cap_rows, self.return_flags, self.world, self.me, self.epoch,
                                  self.counters[1:2], flags)

    def wait_return(self, flags):
        self.native.ep_wait_signals(self.base + self.flag_offset, self.world, self.me, self.epoch, flags)

    def _release(self):
        for ptr in self.peers.values():
            self.native.ep_ipc_close(ptr)
        self.peers = {}
        if self.base:
            self.native.ep_buffer_free(self.base)
            self.base = 0

    def close(self):
        """Collective: no rank unmaps or frees before every rank has finished."""
        if not self.base:
            return
        torch.cuda.synchronize()
        dist.barrier(group=self.group)
        self.x = self.ids = self.rows = None
        for ptr in self.peers.values():
            self.native.ep_ipc_close(ptr)
        self.peers = {}
        dist.barrier(group=self.group)
        self.native.ep_buffer_free(self.base)
        self.base = 0


class PeerFixedExchange:
    """Receive buffers of the fixed-size exchange over NVLink peer memory
    (every rank T tokens), in two sets used by odd and even calls: token rows
    bf16 [2][world*T][2048] and their local ids int32 [2][world*T][8], result
    rows fp32 [2][T*8][2048], then dispatch and return flag arrays (2*world
    uint32 words each: epochs, then status words carrying each sender's
    flag-64 bit).  The call number is an int32 on the device, so a step holds no
    host value that changes between calls and can be captured in a CUDA
    graph.  Made and closed collectively, like PeerExchange."""

    def __init__(self, group, world, me, T, device, partial=False):
        from . import native
        if not 1 <= world <= 8:
            raise ValueError('the peer-memory exchange serves 1..8 ranks of one node')
        self.native, self.group, self.world, self.me, self.T = native, group, world, me, int(T)
        self.partial = bool(partial)
        rows_in = world * self.T
        # result rows: the T*8 slot rows of this rank's tokens, or (rank-partial
        # combine) one fp32 sum per (rank, token): world*T rows
        rows_out = rows_in if self.partial else self.T * TOP
        self.rows_out = rows_out

        def up(n):
            return (n + 255) // 256 * 256
        self.x_offset, self.x_set = 0, up(rows_in * H * 2)
        self.ids_offset, self.ids_set = 2 * self.x_set, up(rows_in * TOP * 4)
        self.w_offset, self.w_set = self.ids_offset + 2 * self.ids_set, (up(rows_in * TOP * 4) if self.partial else 0)
        self.rows_offset, self.rows_set = self.w_offset + 2 * self.w_set, up(rows_out * H * 4)
        self.flag_offset = up(self.rows_offset + 2 * self.rows_set)
        self.base = native.ep_buffer_alloc(self.flag_offset + 256)
        self.peers = {}
        try:
            handles = [None] * world
            dist.all_gather_object(handles, native.ep_ipc_handle(self.base), group=group)
            for r in range(world):
                if r != me:
                    self.peers[r] = native.ep_ipc_open(handles[r])
        except BaseException:
            PeerExchange._release(self)
            raise
        bases = [self.base if r == me else self.peers[r] for r in range(world)]

        def sets(offset, stride):
            return (C.c_void_p * (2 * world))(*[b + offset + k * stride for k in range(2) for b in bases])
        self.dst_x, self.dst_ids = sets(self.x_offset, self.x_set), sets(self.ids_offset, self.ids_set)
        self.dst_w = sets(self.w_offset, self.w_set) if self.partial else None
        self.dst_rows = sets(self.rows_offset, self.rows_set)
        self.dispatch_flags = (C.c_void_p * world)(*[b + self.flag_offset for b in bases])
        self.return_flags = (C.c_void_p * world)(*[b + self.flag_offset + 8 * world for b in bases])
        def view(offset, shape, typestr, strides=None):
            return torch.as_tensor(_DeviceArray(self.base + offset, shape, typestr, strides), device=device)
        # both sets of a buffer as one [2, ...] view (byte strides), so that a
        # device-side index picks a set without touching the other
        self.x2 = view(self.x_offset, (2, rows_in, H), '<i2', (self.x_set, H * 2, 2)).view(torch.bfloat16)
        self.ids2 = view(self.ids_offset, (2, rows_in, TOP), '<i4', (self.ids_set, TOP * 4, 4))
        self.w2 = view(self.w_offset, (2, rows_in, TOP), '<f4', (self.w_set, TOP * 4, 4)) if self.partial else None
        # both result sets as one array of rows (the set stride is whole rows)
        self.rows = view(self.rows_offset, (2 * self.rows_set // (H * 4), H), '<f4')
        self.epoch = torch.zeros(1, dtype=torch.int32, device=device)
        self.counters = torch.zeros(2, dtype=torch.int32, device=device)
        self._slot_rows = torch.arange(self.T * TOP, dtype=torch.int32, device=device).view(self.T, TOP)

    def parity(self):
        """0 or 1: the set of the current call, as a device tensor."""
        return (self.epoch & 1).long()

    def dispatch(self, x, local_ids_per_rank, flags):
        self.native.ep_fixed_dispatch(x, local_ids_per_rank, self.dst_x, self.dst_ids, self.world * self.T,
                                      self.dispatch_flags, self.world, self.me, self.epoch, self.counters[0:1], flags)

    def dispatch_w(self, x, local_ids_per_rank, local_w_per_rank, flags):
        self.native.ep_fixed_dispatch_weights(x, local_ids_per_rank, local_w_per_rank, self.dst_x, self.dst_ids,
                                              self.dst_w, self.world * self.T, self.dispatch_flags, self.world,
                                              self.me, self.epoch, self.counters[0:1], flags)

    def received_w(self):
        """received() plus the slot weights fp32 [world*T, 8] of this call's set."""
        x, ids = self.received()
        w = torch.index_select(self.w2, 0, self.parity())[0]
        return x, ids, w.contiguous()

    def ret_partial(self, workspace, capacity, ids_all, flags):
        self.native.ep_fixed_return_partial(workspace, self.T, capacity, ids_all, self.dst_rows, self.rows_out,
                                            self.return_flags, self.world, self.me, self.epoch,
                                            self.counters[1:2], flags)

    def partial_index(self, mine):
        """int32 [T, 8] for the rank sum: column d holds the row of self.rows
        with rank d's sum for token t in this call's set, -1 where rank d owns
        none of the token's slots (and for columns d >= world).  mine: bool
        [world, T, 8], slot s of token t belongs to rank d."""
        T = self.T
        has = mine.any(dim=2).t()                                                   # [T, world]
        t = torch.arange(T, device=mine.device, dtype=torch.int32).view(-1, 1)
        d = torch.arange(self.world, device=mine.device, dtype=torch.int32).view(1, -1)
        base = (self.parity() * (self.rows_set // (H * 4))).to(torch.int32)
        idx = torch.where(has, base + d * T + t, torch.full_like(t.expand(T, self.world), -1))
        if self.world < TOP:
            idx = torch.cat([idx, torch.full((T, TOP - self.world), -1, dtype=torch.int32, device=mine.device)], 1)
        return idx.contiguous()

    def wait_dispatch(self, flags):
        self.native.ep_wait_epoch(self.base + self.flag_offset, self.world, self.me, self.epoch, flags)

    def received(self):
        """(token rows [world*T, 2048], local ids [world*T, 8]) of this call's
        set, copied out by a device-side choice of the set (index_select reads
        only the chosen one)."""
        k = self.parity()
        x = torch.index_select(self.x2, 0, k)[0]
        ids = torch.index_select(self.ids2, 0, k)[0]
        return x.contiguous(), ids.contiguous()

    def ret(self, workspace, capacity, ids_all, flags):
        self.native.ep_fixed_return(workspace, self.T, capacity, ids_all, self.dst_rows, self.T * TOP,
                                    self.return_flags, self.world, self.me, self.epoch, self.counters[1:2], flags)

    def wait_return(self, flags):
        self.native.ep_wait_epoch(self.base + self.flag_offset + 8 * self.world, self.world, self.me, self.epoch,
                                  flags)

    def result_index(self, ids):
        """int32 [T, 8]: row of self.rows holding slot s of token t in this
        call's set, -1 for padding and invalid ids."""
        valid = (ids >= 0) & (ids < E)
        rows = self._slot_rows + (self.parity() * (self.T * TOP)).to(torch.int32)
        return torch.where(valid, rows, torch.full_like(rows, -1)).contiguous()

    def close(self):
        """Collective, like PeerExchange.close; the views go first."""
        self.x2 = self.ids2 = self.w2 = self.rows = None
        PeerExchange.close(self)


class ExpertParallelMoE:
    """GPU expert-parallel layer over NCCL with this library's kernels.

    banks: (gate_codes, gate_meta, down_codes, down_meta) of the local experts
    only ([256/world, ...] each, in the placement's bank order:
    placement.experts_of(rank)).  capacity: the largest number of token rows
    one rank may receive (world * local tokens at most).  exchange: 'compact'
    (variable splits, any token counts) or 'fixed' (equal blocks, no host
    synchronisation; every rank must call with the same token count).
    combine: 'exact' (per-slot rows, bit-identical to one GPU) or 'partial'
    (per-rank partial sums, fp32-rounding agreement).  placement: the same on
    every rank; contiguous ranges by default.  chunks: compact exchange in
    that many pipelined token ranges (exact combine).  transport: 'nccl'
    (all_to_all) or 'p2p' (token rows and results stored straight into the
    receiving ranks' buffers over NVLink peer memory; compact exchange, exact
    combine, one chunk).  The dispatch plan of the compact exchange comes from
    one device launch (NativePlanner).  close() releases the peer buffers,
    collectively, before the process group is destroyed."""

    def __init__(self, group, world, banks, capacity, act_bits=8, exchange='compact', placement=None,
                 combine='exact', chunks=1, transport='nccl'):
        from . import native
        if exchange not in ('compact', 'fixed'):
            raise ValueError(f'unknown exchange mode {exchange!r}')
        if combine not in ('exact', 'partial'):
            raise ValueError(f'unknown combine mode {combine!r}')
        if combine == 'partial' and world > TOP:
            raise ValueError('the rank-partial combine supports at most 8 ranks')
        if not isinstance(chunks, int) or chunks < 1 or (chunks > 1 and (exchange, combine) != ('compact', 'exact')):
            raise ValueError('chunks > 1 applies to the compact exchange with the exact combine')
        if transport not in ('nccl', 'p2p') or (transport == 'p2p' and (
                chunks != 1 or not 1 <= world <= 8 or (combine == 'partial' and exchange != 'fixed'))):
            raise ValueError("transport 'p2p' applies to one chunk on 1..8 ranks of one node, and with the "
                             "rank-partial combine to the fixed exchange")
        self.transport = transport
        self.chunks = chunks
        self.combine_mode = combine
        self.native = native
        self.group, self.world = group, world
        self.banks = banks
        self.capacity = int(capacity)
        self.exchange = exchange
        self.placement = placement or contiguous_placement(world, banks[0].device)
        self.planner = NativePlanner(world, self.placement, banks[0].device)
        self.me = dist.get_rank(group)
        # an expert rank receives at most `capacity` token rows; a home rank gets
        # back at most one row per (token, slot), 8 per local token
        self.peer = PeerExchange(group, world, self.me, self.capacity, TOP * self.capacity, banks[0].device) \
            if (transport, exchange) == ('p2p', 'compact') else None
        self.peer_fixed = None   # fixed exchange over peer memory: made at the first call (it needs T)
        self.symbol = 'ornith_routed_direct_launch' if act_bits == 8 else 'ornith_routed_direct_launch_a4'
        dev = banks[0].device
        self.layout = native.get_layout(self.capacity)
        self.workspace = torch.empty(self.layout.workspace_bytes, dtype=torch.uint8, device=dev)
        self.flags = torch.zeros(1, dtype=torch.int32, device=dev)
        self._ones = torch.ones((self.capacity, TOP), dtype=torch.float32, device=dev)
        self._scratch_out = torch.empty((self.capacity, H), dtype=torch.bfloat16, device=dev)

    def _layer(self, x_recv, ids_recv, w_recv=None):
        n = x_recv.shape[0]
        if n > self.capacity:
            raise ValueError(f'expert-parallel receive of {n} rows exceeds capacity {self.capacity}')
        if n:
            native = self.native
            fn = getattr(native.lib(), self.symbol)
            w = self._ones[:n] if w_recv is None else w_recv.contiguous()
            native.check(fn(*[native.ptr(t) for t in (x_recv.contiguous(), w, ids_recv, *self.banks,
                                                      self.workspace)],
                            self.workspace.numel(), native.ptr(self._scratch_out), native.ptr(self.flags), n,
                            self.capacity, native.stream(x_recv)), 'expert-parallel compute')
        return n

    def compute(self, x_recv, ids_recv, n_valid=None):
        n = self._layer(x_recv, ids_recv)
        valid = (ids_recv >= 0).view(-1)
        # (token, slot) order; with the count known no host synchronisation
        sel = (valid.nonzero() if n_valid is None else torch.nonzero_static(valid, size=n_valid))
        sel = sel.flatten().to(torch.int32)
        rows = torch.empty((sel.numel(), H), dtype=torch.float32, device=x_recv.device)
        self.native.gather_route_rows(self.workspace, n, self.capacity, sel, rows, self.flags)
        return rows

    def compute_block(self, x_all, ids_all):
        n = self._layer(x_all, ids_all)
        rows = torch.empty((n * TOP, H), dtype=torch.float32, device=x_all.device)
        self.native.scatter_route_rows(self.workspace, n, self.capacity, rows)
        return rows.view(n, TOP, H)

    def compute_partial(self, x_recv, ids_recv, w_recv):
        n = self._layer(x_recv, ids_recv, w_recv)
        off = self.layout.final_f32
        return self.workspace[off:off + n * H * 4].view(torch.float32).view(n, H)

    def combine(self, rows, row_index, weights, ids):
        out = torch.empty((ids.shape[0], H), dtype=torch.bfloat16, device=rows.device)
        self.native.combine_gathered(rows, row_index, weights, ids, out, self.flags)
        return out

    def _layer_p2p(self, x, ids, weights):
        """Compact exchange over NVLink peer memory (PeerExchange): token rows
        go straight into the expert ranks' buffers and results straight into
        the home ranks' buffers; the count all_gather stays on NCCL."""
        plan, recv_counts, back_counts, offsets, x_offsets = dispatch_with_matrix(
            self.group, self.world, self.me, ids, self.placement, self.planner, self.capacity)
        n = sum(recv_counts)
        self.peer.dispatch(x.contiguous(), plan, x_offsets, self.flags)
        self.peer.wait_dispatch(self.flags)
        x_recv, ids_recv = self.peer.x[:n], self.peer.ids[:n]
        self._layer(x_recv, ids_recv)
        valid = (ids_recv >= 0).view(-1)
        sel = torch.nonzero_static(valid, size=sum(back_counts)).flatten().to(torch.int32)
        self.peer.ret(self.workspace, n, self.capacity, sel, back_counts, offsets, self.flags)
        self.peer.wait_return(self.flags)
        got = self.peer.rows[:sum(plan.home_counts)]
        return self.combine(got, route_row_index(x.shape[0], plan, x.device), weights, ids)

    def _layer_fixed_p2p(self, x, ids, weights):
        """Fixed exchange over NVLink peer memory (PeerFixedExchange): every
        rank's token rows go to every rank, the computed slots straight to
        their home ranks; no collective and no host value that changes
        between calls, so the step can be captured in a CUDA graph.  Every
        call must have the token count of the first."""
        T = x.shape[0]
        if self.peer_fixed is None:
            self.peer_fixed = PeerFixedExchange(self.group, self.world, self.me, T, x.device)   # collective
        elif self.peer_fixed.T != T:
            raise ValueError(f'the fixed peer-memory exchange was made for {self.peer_fixed.T} tokens, got {T}')
        if self.world * T > self.capacity:
            raise ValueError(f'expert-parallel receive of {self.world * T} rows exceeds capacity {self.capacity}')
        owner, lid = map_ids(ids, self.placement)
        dest = torch.arange(self.world, device=ids.device, dtype=owner.dtype).view(-1, 1, 1)
        local = torch.where(owner.unsqueeze(0) == dest, lid.unsqueeze(0), torch.full_like(lid, -1).unsqueeze(0))
        pf = self.peer_fixed
        pf.dispatch(x.contiguous(), local.to(torch.int32).contiguous(), self.flags)
        pf.wait_dispatch(self.flags)
        x_all, ids_all = pf.received()
        self._layer(x_all, ids_all)
        pf.ret(self.workspace, self.capacity, ids_all, self.flags)
        pf.wait_return(self.flags)
        return self.combine(pf.rows, pf.result_index(ids), weights, ids)

    def _layer_fixed_p2p_partial(self, x, ids, weights):
        """Fixed exchange over NVLink peer memory with the rank-partial
        combine: every rank's token rows, local ids and slot weights go to
        every rank (one dispatch kernel); each rank's fp32 sums over its own
        slots go straight to the tokens' home ranks (one return kernel, rows of
        tokens with no slot there left out); the home rank adds the ranks'
        sums in rank order.  No collective and no host value that changes
        between calls, so the step can be captured in a CUDA graph.  Every call
        must have the token count of the first."""
        T = x.shape[0]
        if self.peer_fixed is None:
            self.peer_fixed = PeerFixedExchange(self.group, self.world, self.me, T, x.device, partial=True)
        elif self.peer_fixed.T != T:
            raise ValueError(f'the fixed peer-memory exchange was made for {self.peer_fixed.T} tokens, got {T}')
        if self.world * T > self.capacity:
            raise ValueError(f'expert-parallel receive of {self.world * T} rows exceeds capacity {self.capacity}')
        owner, lid = map_ids(ids, self.placement)
        dest = torch.arange(self.world, device=ids.device, dtype=owner.dtype).view(-1, 1, 1)
        mine = owner.unsqueeze(0) == dest                                                  # [world, T, 8]
        local = torch.where(mine, lid.unsqueeze(0), torch.full_like(lid, -1).unsqueeze(0)).to(torch.int32)
        w_local = torch.where(mine, weights.unsqueeze(0), torch.zeros_like(weights).unsqueeze(0))
        pf = self.peer_fixed
        pf.dispatch_w(x.contiguous(), local.contiguous(), w_local.contiguous(), self.flags)
        pf.wait_dispatch(self.flags)
        x_all, ids_all, w_all = pf.received_w()
        self._layer(x_all, ids_all, w_all)
        pf.ret_partial(self.workspace, self.capacity, ids_all, self.flags)
        pf.wait_return(self.flags)
        return rank_sum(self.combine, pf.rows, pf.partial_index(mine), weights)

    def close(self):
        """Release the peer-memory buffers (collective; before the process
        group is destroyed)."""
        for name in ('peer', 'peer_fixed'):
            if getattr(self, name) is not None:
                getattr(self, name).close()
                setattr(self, name, None)

    def _single(self, x, ids, weights):
        """One rank holds every expert: the layer itself, no exchange (the
        single-GPU layer's result, bit for bit)."""
        T = x.shape[0]
        if T > self.capacity:
            raise ValueError(f'{T} tokens exceed capacity {self.capacity}')
        out = torch.empty((T, H), dtype=torch.bfloat16, device=x.device)
        if T:
            native = self.native
            fn = getattr(native.lib(), self.symbol)
            native.check(fn(*[native.ptr(t) for t in (x.contiguous(), weights.contiguous(), ids.contiguous(),
                                                      *self.banks, self.workspace)],
                            self.workspace.numel(), native.ptr(out), native.ptr(self.flags), T, self.capacity,
                            native.stream(x)), 'expert-parallel compute')
        return out

    def __call__(self, x, ids, weights):
        if self.world == 1:
            return self._single(x, ids, weights)
        if self.combine_mode == 'partial':
            # the partial rows reach the combine without the ids: ids outside
            # -1..255 (flag 4 on one GPU) are flagged here, on the device
            self.flags.bitwise_or_(((ids >= E) | (ids < -1)).any().to(self.flags.dtype) * 4)
            if self.exchange == 'fixed' and self.transport == 'p2p':
                return self._layer_fixed_p2p_partial(x, ids, weights)
            if self.exchange == 'fixed':
                return ep_layer_fixed_partial(self.group, self.world, x, ids, weights, self.compute_partial,
                                              self.combine, self.placement)
            return ep_layer_partial(self.group, self.world, x, ids, weights, self.compute_partial, self.combine,
                                    self.placement, self.planner)
        if self.exchange == 'fixed' and self.transport == 'p2p':
            return self._layer_fixed_p2p(x, ids, weights)
        if self.exchange == 'fixed':
            return ep_layer_fixed(self.group, self.world, x, ids, weights, self.compute_block, self.combine,
                                  self.placement)
        if self.peer is not None:
            return self._layer_p2p(x, ids, weights)
        if self.chunks > 1:
            return ep_layer_chunked(self.group, self.world, x, ids, weights, self.compute, self.combine,
                                    self.placement, self.chunks, self.planner)
        return ep_layer(self.group, self.world, x, ids, weights, self.compute, self.combine, self.placement,
                        self.planner)
