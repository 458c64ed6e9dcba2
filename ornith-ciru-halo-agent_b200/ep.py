"""Expert parallelism for the routed-MoE layer over torch.distributed.

The reference runs one rank and refuses EP (plugin-site/ornith_g256/moe_base.py:34-39);
this module adds it.  Rank r of n owns routed experts
[r*256/n, (r+1)*256/n); the shared expert is replicated and runs on each rank
for its own tokens.  One layer call on every rank, for the rank's own tokens:

  1. route: top-8 ids and weights of the local tokens;
  2. dispatch plan: for every destination rank d, the local tokens with at
     least one expert on d (deduplicated per (token, rank)), with their eight
     ids rewritten to d's local expert numbers (-1 for slots owned elsewhere);
  3. exchange: counts, then token rows (bf16 pairs carried as int32) and local
     ids (all_to_all_single; NCCL on GPUs, gloo on CPU);
  4. expert compute on the received rows with the local banks; the fp32
     down projections of the valid slots are gathered in (token, slot) order;
  5. return exchange of those rows, one per (token, slot) owned by d;
  6. home combine: slot-ordered weighted sum into bf16 with the same
     arithmetic as the single-GPU layer, so the result is bit-identical to it;
     it reads the returned rows where they arrived, through a (token, slot)
     -> row index, instead of scattering them into a dense [8T, 2048] buffer.

These collectives are the layer's only exchange.  Every rank takes the same
collective steps in the same order, zero-sized messages included.
"""
from dataclasses import dataclass

import torch
import torch.distributed as dist

E, TOP, H = 256, 8, 2048


@dataclass
class DispatchPlan:
    send_counts: list          # tokens sent to each rank
    token_index: torch.Tensor  # [sum(send_counts)] local token of each sent row, grouped by rank
    local_ids: torch.Tensor    # [sum(send_counts), 8] ids in the destination's numbering, -1 elsewhere
    slot_mask: torch.Tensor    # [sum(send_counts), 8] True where the slot is owned by the destination


def build_dispatch(ids, world, experts_per_rank=None):
    """Group each token's slots by owning rank (pure tensor logic, any device)."""
    epr = experts_per_rank or E // world
    owner = torch.where(ids >= 0, torch.div(ids, epr, rounding_mode='floor'), torch.full_like(ids, -1))
    counts, tokens, lids, masks = [], [], [], []
    for d in range(world):
        m = owner == d
        tok = m.any(dim=1).nonzero().flatten()
        mk = m[tok]
        lid = torch.where(mk, ids[tok] - d * epr, torch.full_like(ids[tok], -1))
        counts.append(int(tok.numel()))
        tokens.append(tok)
        lids.append(lid)
        masks.append(mk)
    return DispatchPlan(counts, torch.cat(tokens), torch.cat(lids).to(torch.int32).contiguous(), torch.cat(masks))


def _a2a(group, out, inp, out_splits, in_splits):
    dist.all_to_all_single(out, inp, out_splits, in_splits, group=group)


def exchange_rows(group, world, plan, x):
    """Send each rank its token rows and local ids; returns (x_recv, ids_recv, recv_counts)."""
    dev = x.device
    send = torch.tensor(plan.send_counts, dtype=torch.int64, device=dev)
    recv = torch.empty_like(send)
    _a2a(group, recv, send, [1] * world, [1] * world)
    recv_counts = [int(v) for v in recv.tolist()]
    n_in = sum(recv_counts)
    x_words = x.contiguous().view(torch.int32)[plan.token_index].contiguous()   # [n, 1024]
    x_recv = torch.empty((n_in, H // 2), dtype=torch.int32, device=dev)
    _a2a(group, x_recv, x_words, recv_counts, plan.send_counts)
    ids_recv = torch.empty((n_in, TOP), dtype=torch.int32, device=dev)
    _a2a(group, ids_recv, plan.local_ids, recv_counts, plan.send_counts)
    return x_recv.view(x.dtype), ids_recv, recv_counts


def return_rows(group, world, plan, ids_recv, recv_counts, out_rows):
    """Send every (token, slot) row computed here back to the token's home rank.

    out_rows: fp32 [n_valid, 2048], one row per received slot with a valid
    local id, in (token, slot) order.  Returns the home-side fp32 rows
    [n_sent_slots, 2048] in the order of plan.slot_mask."""
    valid = ids_recv >= 0
    back_counts = [int(v.sum()) for v in torch.split(valid.sum(dim=1), recv_counts)]
    home_counts = [int(m.sum()) for m in torch.split(plan.slot_mask, plan.send_counts)]
    got = torch.empty((sum(home_counts), H), dtype=torch.float32, device=out_rows.device)
    _a2a(group, got, out_rows, home_counts, back_counts)
    return got


def route_row_index(T, plan, device):
    """int32 [T, 8]: the row of `got` (return_rows) holding slot s of token t,
    -1 for slots no rank returned (padding ids)."""
    idx = torch.full((T, TOP), -1, dtype=torch.int32, device=device)
    k, s = plan.slot_mask.nonzero(as_tuple=True)  # the order of return_rows
    idx[plan.token_index[k], s] = torch.arange(k.numel(), dtype=torch.int32, device=device)
    return idx


def ep_layer(group, world, x, ids, weights, compute, combine):
    """One expert-parallel layer call.

    compute(x_recv, ids_recv) -> fp32 [n_valid, 2048]: the rows of the received
    slots with a valid id, in (token, slot) order; combine(rows [n, 2048],
    row_index [T, 8], weights, ids) -> output.  Both are injected so that the
    host logic also runs on CPU ranks."""
    plan = build_dispatch(ids, world)
    x_recv, ids_recv, recv_counts = exchange_rows(group, world, plan, x)
    out_rows = compute(x_recv, ids_recv)
    got = return_rows(group, world, plan, ids_recv, recv_counts, out_rows)
    return combine(got, route_row_index(x.shape[0], plan, got.device), weights, ids)


class ExpertParallelMoE:
    """GPU expert-parallel layer over NCCL with this library's kernels.

    banks: (gate_codes, gate_meta, down_codes, down_meta) of the local experts
    only ([256/world, ...] each).  capacity: the largest number of token rows
    one rank may receive (world * local tokens at most)."""

    def __init__(self, group, world, banks, capacity, act_bits=8):
        from . import native
        self.native = native
        self.group, self.world = group, world
        self.banks = banks
        self.capacity = int(capacity)
        self.symbol = 'ornith_routed_direct_launch' if act_bits == 8 else 'ornith_routed_direct_launch_a4'
        dev = banks[0].device
        self.layout = native.get_layout(self.capacity)
        self.workspace = torch.empty(self.layout.workspace_bytes, dtype=torch.uint8, device=dev)
        self.flags = torch.zeros(1, dtype=torch.int32, device=dev)
        self._ones = torch.ones((self.capacity, TOP), dtype=torch.float32, device=dev)
        self._scratch_out = torch.empty((self.capacity, H), dtype=torch.bfloat16, device=dev)

    def compute(self, x_recv, ids_recv):
        n = x_recv.shape[0]
        if n > self.capacity:
            raise ValueError(f'expert-parallel receive of {n} rows exceeds capacity {self.capacity}')
        native = self.native
        if n:
            fn = getattr(native.lib(), self.symbol)
            native.check(fn(*[native.ptr(t) for t in (x_recv.contiguous(), self._ones[:n], ids_recv, *self.banks,
                                                      self.workspace)],
                            self.workspace.numel(), native.ptr(self._scratch_out), native.ptr(self.flags), n,
                            self.capacity, native.stream(x_recv)), 'expert-parallel compute')
        sel = (ids_recv >= 0).view(-1).nonzero().flatten().to(torch.int32)  # (token, slot) order
        rows = torch.empty((sel.numel(), H), dtype=torch.float32, device=x_recv.device)
        native.gather_route_rows(self.workspace, n, self.capacity, sel, rows, self.flags)
        return rows

    def combine(self, rows, row_index, weights, ids):
        out = torch.empty((ids.shape[0], H), dtype=torch.bfloat16, device=rows.device)
        self.native.combine_gathered(rows, row_index, weights, ids, out, self.flags)
        return out

    def __call__(self, x, ids, weights):
        return ep_layer(self.group, self.world, x, ids, weights, self.compute, self.combine)
