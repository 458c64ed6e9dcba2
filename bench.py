#!/usr/bin/env python
"""Benchmark of the B200 routed-MoE layer (driver contract: one JSON line on rank 0).

Workload (default): decode B=1 through a stack of 40
Ornith MoE layers (256 routed experts + 1 shared, H2048/I512, affine-u4 G256
weights, A8 activations), fresh seeded weights per layer (16.6 GB resident),
router logits ~N(0,1) per layer and step.  One step = one token through the
40 independent layers (each takes the step's token rows as input), every
layer called through
`ornith_b200::routed_from_logits` (routing, routed experts, shared expert,
combine).  Other workloads: --config decode32 (configs[2], logits + per-expert
bias N(0,0.5)), prefill1120 / prefill8192 (configs[3], A4, 40 weight sets
cycled so that weights never stay in L2).

Timing: W warm-up steps, then K steps between CUDA events on the launching
stream, barrier + synchronize on both sides, max over ranks.  Every step reads
(distinct experts + 1) x 1.62 MB per layer, far more than the 126 MB L2, so no
explicit flush is needed (config.l2 says so).  `e2e` repeats the measurement
through the same public operator with host (pinned) inputs copied in and the
final output copied out inside the timed region.  A decode step is captured
once as a CUDA graph of those operator calls and replayed (as a serving engine
does); --no-graph times the eager launches.

--impl reference times the reference's own routed source compiled for the CPU
(oracle/_ref, built by oracle/build_ref.py) on this host's cores on a bounded
sample of the same workload; rank 0 only.
"""
import argparse
import json
import os
import statistics
import subprocess
import sys
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))
import __graft_entry__ as graft  # noqa: E402

METRIC = 'MoE-layer tokens/s & % of HBM/tensor roofline (decode B=1/32, 8K prefill)'
EXPERT_BYTES = 1_622_016          # w13 codes 1,048,576 + meta 32,768 + w2 codes 524,288 + meta 16,384
# DRAM bytes (read + write) per launch of the dominant kernel, from one ncu
# capture of the same workload (profiles/decode_single_kernel_decode1.md,
# profiles/decode_layer_kernel_decode32.md, profiles/prefill_mma_kernel_prefill8192.md).
NCU_TRAFFIC = {
    'decode1': {'kernel': 'decode_single_kernel<127>', 'bytes': 14_712_832},
    'decode32': {'kernel': 'decode_layer_kernel<127>', 'bytes': 214_940_160 + 5_720_320},
    'prefill8192': {'kernel': 'mma_kernel<8,1> (gate/up)', 'bytes': 448_872_704 + 113_913_600},
    # profiles/dense_fused_kernel_dense_qkvz1.md, profiles/head_project_kernel_head_vocab1.md
    'dense_qkvz1': {'kernel': 'dense_fused_kernel<16>', 'bytes': 13_006_336 + 0},
    'head_vocab1': {'kernel': 'head_project_kernel<0>', 'bytes': 516_537_856 + 3_437_824},
}
# int8 multiply-accumulates per valid route of one layer: gate/up 1024x2048 + down 2048x512
MACS_PER_ROUTE = 3_145_728
# workloads measured in the same process as the default decode B=1 line
SUB_CONFIGS = {'decode1': ['decode32', 'prefill1120', 'prefill8192']}

CONFIGS = {
    'decode1': dict(T=1, layers=40, bias=0.0, act_bits=8, shared=True, name='decode B=1, 40-layer stack (configs[1])'),
    'decode32': dict(T=32, layers=40, bias=0.5, act_bits=8, shared=True, name='decode B=32, 40-layer stack (configs[2])'),
    # decode B=1 through the from-hidden entry: the router linear (bf16 [256, 2048]
    # per layer) inside the operator, a fresh token row per step
    'decode1_hidden': dict(T=1, layers=40, bias=0.0, act_bits=8, shared=True, entry='hidden',
                           name='decode B=1 from hidden states (router linear in the operator), 40-layer stack'),
    'prefill1120': dict(T=1120, layers=40, bias=0.0, act_bits=4, shared=False, name='prefill chunk 1120 (configs[3])'),
    'prefill8192': dict(T=8192, layers=40, bias=0.0, act_bits=4, shared=False, name='prefill chunk 8192 (configs[3])'),
    # expert-parallel sweep: total tokens fixed, experts sharded over the ranks
    'ep_decode256': dict(T=256, layers=40, bias=0.0, act_bits=8, shared=False, ep=True, exchange='fixed',
                         combine='exact', transport='p2p',
                         name='expert-parallel decode B=256, 40 layers, Zipf(1.2) expert skew (configs[4])'),
    # prefill: equal blocks (token rows gathered on every rank, no host
    # synchronisation, one CUDA graph) and per-rank fp32 partial sums coming
    # home (within the north-star tolerance of the single-GPU layer); measured
    # fastest of the exchange modes on 2 B200s
    'ep_prefill8192': dict(T=8192, layers=4, bias=0.0, act_bits=4, shared=False, ep=True, exchange='fixed',
                           combine='partial', transport='nccl',
                           name='expert-parallel prefill 8192 tokens, Zipf(1.2) expert skew (configs[4]); '
                                '4 weight sets cycled'),
    # dense G256 projection (the next row after the MoE layer): QKVZ-shaped
    # 12288 x 2048 banks, 40 of them so that weights stream from HBM
    'dense_qkvz1': dict(T=1, layers=40, N=12288, K=2048, dense=True,
                        name='dense G256 A8 projection N12288 x K2048, 1 row, 40 banks'),
    'dense_qkvz16': dict(T=16, layers=40, N=12288, K=2048, dense=True,
                         name='dense G256 A8 projection N12288 x K2048, 16 rows, 40 banks'),
    # W8 LM head: the 248,320 x 2048 int8 bank (508 MB, four times L2) per decode step
    'head_vocab1': dict(T=1, layers=1, N=248320, K=2048, head=True,
                        name='W8 LM head, vocabulary 248320 x 2048 int8, 1 row'),
    'head_vocab8': dict(T=8, layers=1, N=248320, K=2048, head=True,
                        name='W8 LM head, vocabulary 248320 x 2048 int8, 8 rows'),
}


def parse():
    p = argparse.ArgumentParser()
    p.add_argument('--gpus', type=int, default=1)
    p.add_argument('--steps', type=int, default=20)
    p.add_argument('--warmup', type=int, default=5)
    p.add_argument('--impl', default='b200', choices=['b200', 'reference'])
    p.add_argument('--config', default=None, choices=sorted(CONFIGS),
                   help='workload (default: decode1 as a plain process; ep_prefill8192 under torch.distributed.run, '
                        'any world size)')
    p.add_argument('--no-sub', action='store_true',
                   help='only the named workload (the decode1 line otherwise also measures decode32, prefill1120 '
                        'and prefill8192 as sub_results)')
    p.add_argument('--no-cpu-baseline', action='store_true')
    p.add_argument('--cpu-seconds', type=float, default=12.0)
    p.add_argument('--no-graph', action='store_true', help='time eager launches instead of a captured step')
    p.add_argument('--e2e-overlap', action='store_true',
                   help='e2e with the host copies pipelined: step s+1 copied in and step s-1 copied out on copy '
                        'streams while step s runs (every copy still inside the timed region)')
    p.add_argument('--placement', choices=['balanced', 'contiguous'], default='balanced',
                   help='expert placement of the expert-parallel configs')
    p.add_argument('--combine', choices=['exact', 'partial'], default=None,
                   help='expert-parallel return (default: the config\'s): per-slot rows (bit-exact) or per-rank '
                        'fp32 partial sums')
    p.add_argument('--ep-transport', choices=['nccl', 'p2p'], default=None,
                   help='expert-parallel token dispatch and return: NCCL, or stores into the receiving ranks\' '
                        'buffers over NVLink peer memory (exact combine, one chunk)')
    p.add_argument('--ep-exchange', choices=['compact', 'fixed'], default=None,
                   help='expert-parallel exchange (default: the config\'s): variable-size compact blocks, or '
                        'equal blocks with no host synchronisation')
    p.add_argument('--ep-chunks', type=int, default=1,
                   help='compact expert-parallel exchange in this many pipelined token chunks (exact combine)')
    p.add_argument('--layers', type=int, default=None,
                   help='override the layer count (small cases for profiler captures)')
    p.add_argument('--ep-phases', action='store_true',
                   help='expert-parallel prefill (fixed exchange, partial combine): time each phase of one layer '
                        'call eagerly with CUDA events (max over ranks) instead of the captured step')
    args = p.parse_args()
    if args.config is None:
        args.config = 'ep_prefill8192' if under_torchrun() else 'decode1'
    return args


def under_torchrun():
    """True when torch.distributed.run (torchrun) launched this process."""
    return 'TORCHELASTIC_RUN_ID' in os.environ or 'LOCAL_WORLD_SIZE' in os.environ


# ---------------------------------------------------------------------------
# clocks during the timed region
# ---------------------------------------------------------------------------
class ClockSampler:
    QUERY = ('index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,'
             'clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,'
             'clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap')

    def __init__(self, index):
        self.index = index
        self.proc = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(['nvidia-smi', f'--query-gpu={self.QUERY}', '--format=csv,noheader,nounits',
                                          '-i', str(self.index), '-lms', '100'], stdout=subprocess.PIPE,
                                         stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
        time.sleep(0.3)
        return self

    def __exit__(self, *exc):
        self.lines = []
        if self.proc is not None:
            self.proc.terminate()
            out, _ = self.proc.communicate(timeout=10)
            self.lines = [l for l in out.splitlines() if l.strip()]

    def summary(self):
        sm, mx, reasons = [], None, set()
        names = ['hw_slowdown', 'hw_thermal_slowdown', 'sw_thermal_slowdown', 'sw_power_cap']
        for line in self.lines:
            f = [x.strip() for x in line.split(',')]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx = float(f[2])
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower().startswith('active'):
                    reasons.add(n)
        if not sm:
            return {'sm_mhz': None, 'sm_max_mhz': mx, 'reasons': [], 'samples': 0}
        loaded = sorted(sm)[len(sm) // 4:] or sm
        return {'sm_mhz': statistics.median(loaded), 'sm_max_mhz': mx, 'reasons': sorted(reasons), 'samples': len(sm)}


# ---------------------------------------------------------------------------
# device workload
# ---------------------------------------------------------------------------
def device_bank(torch, gen, dev, experts, N, K):
    codes = torch.randint(-2 ** 31, 2 ** 31 - 1, (experts, N // 32, K // 256, 32, 32), dtype=torch.int32,
                          device=dev, generator=gen).view(torch.uint32)
    z = torch.randn((experts, N // 32, K // 256, 32), device=dev, generator=gen)
    scale = (0.01 * z.abs()).to(torch.float16).clamp_min(2 ** -14)
    offset = (scale.float() * -8.0).to(torch.float16)
    meta = ((scale.view(torch.int16).to(torch.int32) & 0xFFFF) | (offset.view(torch.int16).to(torch.int32) << 16))
    return codes, meta.view(torch.uint32)


class Stack:
    def __init__(self, torch, cfg, dev, seed):
        self.torch = torch
        gen = torch.Generator(device=dev)
        gen.manual_seed(seed)
        self.layers = []
        for _ in range(cfg['layers']):
            g = device_bank(torch, gen, dev, 256, 1024, 2048)
            d = device_bank(torch, gen, dev, 256, 2048, 512)
            sg = device_bank(torch, gen, dev, 1, 1024, 2048)
            sd = device_bank(torch, gen, dev, 1, 2048, 512)
            gw = (0.02 * torch.randn(2048, device=dev, generator=gen)).to(torch.bfloat16)
            self.layers.append((g, d, sg, sd, gw))
        tab = np.load(ROOT / 'tests' / 'golden' / 'shared_math_tables.npz')
        self.silu = torch.from_numpy(tab['silu_fp32']).to(dev)
        self.sigmoid = torch.from_numpy(tab['sigmoid_bf16'].view(np.int16)).to(dev).view(torch.bfloat16)
        self.gen = gen


def ep_phase_times(torch, dist, ep, native, layer, placement, x, logits, w, ids, rflags, world, rank, dev, T, args):
    """The phases of one fixed-exchange, rank-partial layer call (the steps of
    ep.ep_layer_fixed_partial), each between CUDA events on the compute
    stream, eagerly (not captured), averaged over the timed repetitions;
    rank 0 prints the per-phase maximum over ranks as one JSON line."""
    if (layer.exchange, layer.combine_mode) != ('fixed', 'partial'):
        raise SystemExit('--ep-phases times the fixed exchange with the partial combine')
    H, TOP = 2048, 8
    native.route_topk(logits, w, ids, rflags)
    names = ['plan', 'all_gather_tokens', 'all_to_all_ids_weights', 'layer', 'all_to_all_partials', 'rank_sum']
    acc = np.zeros(len(names))
    reps = args.warmup + args.steps
    ids_all = None
    for it in range(reps):
        ev = [torch.cuda.Event(enable_timing=True) for _ in range(len(names) + 1)]
        dist.barrier()
        torch.cuda.synchronize()
        ev[0].record()
        owner, lid = ep.map_ids(ids, placement)
        dest = torch.arange(world, device=dev).view(-1, 1, 1)
        mine = owner.unsqueeze(0) == dest
        local_ids = torch.where(mine, lid.unsqueeze(0), torch.full_like(owner.unsqueeze(0), -1)).to(torch.int32)
        local_ids = local_ids.contiguous()
        w_local = torch.where(mine, w.unsqueeze(0), torch.zeros_like(w).unsqueeze(0)).contiguous()
        ev[1].record()
        x_all = torch.empty((world * T, H // 2), dtype=torch.int32, device=dev)
        dist.all_gather_into_tensor(x_all, x.contiguous().view(torch.int32))
        ev[2].record()
        ids_all = torch.empty_like(local_ids)
        dist.all_to_all_single(ids_all, local_ids)
        w_all = torch.empty_like(w_local)
        dist.all_to_all_single(w_all, w_local)
        ev[3].record()
        part = layer.compute_partial(x_all.view(torch.bfloat16), ids_all.view(world * T, TOP),
                                     w_all.view(world * T, TOP))
        ev[4].record()
        got = torch.empty_like(part)
        dist.all_to_all_single(got, part.contiguous())
        ev[5].record()
        t = torch.arange(T, device=dev, dtype=torch.int32).view(-1, 1)
        d = torch.arange(TOP, device=dev, dtype=torch.int32).view(1, -1)
        has = (mine.any(dim=2).t() if world == TOP else
               torch.cat([mine.any(dim=2).t(), torch.zeros((T, TOP - world), dtype=torch.bool, device=dev)], 1))
        row_index = torch.where(has, d * T + t, torch.full_like(has, -1, dtype=torch.int32))
        ep.rank_sum(layer.combine, got.view(world * T, H), row_index.contiguous(), w)
        ev[6].record()
        torch.cuda.synchronize()
        if it >= args.warmup:
            acc += np.array([ev[i].elapsed_time(ev[i + 1]) for i in range(len(names))])
    acc /= max(1, args.steps)
    tm = torch.tensor(acc, device=dev)
    if world > 1:
        dist.all_reduce(tm, op=dist.ReduceOp.MAX)
    if rank == 0:
        print(json.dumps({'ep_phases_ms': dict(zip(names, [round(v, 4) for v in tm.tolist()])),
                          'world': world, 'tokens_total': T * world, 'layer_calls_timed': args.steps,
                          'how': 'one layer call, eager launches, CUDA events per phase on the compute stream, '
                                 'mean over the timed calls, max over ranks'}), flush=True)


def run_ep(args):
    """Expert-parallel step: the total token count is
    fixed and split over the ranks; every rank routes its tokens (device
    top-8 from its router logits) and runs each layer through ornith_b200.ep
    (dispatch to the expert ranks, local experts, return, slot-ordered
    combine on the home rank).  Under torch.distributed.run this is the
    default workload at every world size, one included."""
    import datetime
    import torch
    import torch.distributed as dist
    cfg = dict(CONFIGS[args.config])
    if args.layers:
        cfg['layers'] = args.layers
    if args.ep_exchange:
        cfg['exchange'] = args.ep_exchange
    args.combine = args.combine or cfg['combine']
    args.ep_transport = args.ep_transport or cfg['transport']
    if args.combine == 'partial' and cfg['exchange'] != 'fixed':
        args.ep_transport = 'nccl'   # the rank-partial sums travel over peer memory in the fixed exchange only
    world = int(os.environ.get('WORLD_SIZE', '1'))
    rank = int(os.environ.get('RANK', '0'))
    local = int(os.environ.get('LOCAL_RANK', '0'))
    torch.cuda.set_device(local)
    dev = torch.device('cuda', local)
    os.environ.setdefault('MASTER_ADDR', '127.0.0.1')
    os.environ.setdefault('MASTER_PORT', '29541')
    dist.init_process_group('nccl' if world > 1 else 'gloo', rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=120))
    graft.load_package()
    import importlib
    native = importlib.import_module('ornith_b200.native')
    ep = importlib.import_module('ornith_b200.ep')
    S = importlib.import_module('ornith_b200.synthetic')
    lib = native.lib()
    T_total, L, bits = cfg['T'], cfg['layers'], cfg['act_bits']
    T = T_total // world
    epr = 256 // world
    gen = torch.Generator(device=dev)
    gen.manual_seed(4321 + rank)
    bias = torch.from_numpy(S.zipf_bias(np.random.default_rng(12), 256, 1.2)).to(dev)  # same on every rank
    # expert placement balanced by routed load, from a calibration batch drawn
    # from the same distribution (identical on every rank); each rank's random
    # banks stand for the experts the placement gives it
    calib = torch.randn((4096, 256), generator=torch.Generator().manual_seed(999)) + bias.cpu()
    loads = torch.bincount(torch.topk(calib, 8, dim=1).indices.flatten(), minlength=256)
    placement = ep.balanced_placement(loads, world, dev) if args.placement == 'balanced' else \
        ep.contiguous_placement(world, dev)
    layers = []
    for _ in range(L):
        g = device_bank(torch, gen, dev, epr, 1024, 2048)
        d = device_bank(torch, gen, dev, epr, 2048, 512)
        layers.append(ep.ExpertParallelMoE(None, world, (g[0], g[1], d[0], d[1]), capacity=min(T * world, 8192),
                                           act_bits=bits, exchange=cfg['exchange'], placement=placement,
                                           combine=args.combine,
                                           chunks=args.ep_chunks if cfg['exchange'] == 'compact' else 1,
                                           transport=args.ep_transport))
    logits = torch.randn((L, T, 256), device=dev, generator=gen) + bias
    x = torch.randn((T, 2048), device=dev, generator=gen).to(torch.bfloat16)
    w = torch.empty((L, T, 8), dtype=torch.float32, device=dev)
    ids = torch.empty((L, T, 8), dtype=torch.int32, device=dev)
    rflags = torch.zeros(1, dtype=torch.int32, device=dev)
    outs = [None]

    def step():
        for l in range(L):
            native.route_topk(logits[l], w[l], ids[l], rflags)   # routing is part of the layer
            outs[0] = layers[l](x, ids[l], w[l])

    if args.ep_phases:
        ep_phase_times(torch, dist, ep, native, layers[0], placement, x, logits[0], w[0], ids[0], rflags, world,
                       rank, dev, T, args)
        dist.destroy_process_group()
        return

    # NVLink bytes this rank sends per step: a token row (4,096 B) per (token,
    # remote expert rank), an fp32 result row (8,192 B) per (token, slot) whose
    # expert lives on another rank; summed over the ranks
    step()
    torch.cuda.synchronize()
    owner = placement.rank[ids.clamp_min(0).long()]
    valid = ids >= 0
    home = torch.full_like(owner, rank)
    remote_slot = valid & (owner != home)
    remote_rank_tok = torch.zeros((L, T, world), dtype=torch.bool, device=dev)
    remote_rank_tok.scatter_(2, owner.masked_fill(~remote_slot, rank), remote_slot)
    remote_rank_tok[:, :, rank] = False
    nv = torch.tensor([float(remote_rank_tok.sum()) * 4096 + float(remote_slot.sum()) * 8192,
                       float(valid.sum())], device=dev, dtype=torch.float64)
    nv_max = nv.clone()
    if world > 1:
        dist.all_reduce(nv, op=dist.ReduceOp.SUM)
        dist.all_reduce(nv_max, op=dist.ReduceOp.MAX)
    nvlink_step, routes_step, nvlink_rank_max = float(nv[0]), float(nv[1]), float(nv_max[0])
    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    # The fixed-block exchange has no host synchronisation, so the whole step
    # (collectives included) is captured once and replayed.
    graph = None
    if cfg['exchange'] == 'fixed' and not args.no_graph:
        side = torch.cuda.Stream()
        side.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(side):
            step()
        torch.cuda.current_stream().wait_stream(side)
        torch.cuda.synchronize()
        dist.barrier()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            step()
        torch.cuda.synchronize()
        dist.barrier()
        for _ in range(max(3, args.warmup)):   # the captured collectives warmed up on every rank
            graph.replay()
        torch.cuda.synchronize()
    run_step = graph.replay if graph is not None else step
    n0 = lib.ornith_moe_b200_kernel_launches()
    dist.barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clk:
        e0.record()
        for _ in range(args.steps):
            run_step()
        e1.record()
        torch.cuda.synchronize()
    launches = lib.ornith_moe_b200_kernel_launches() - n0
    if graph is not None:
        launches = launches_per_step(lib, step) * args.steps
    ms = e0.elapsed_time(e1)

    def max_over_ranks(v):
        t = torch.tensor([v], device=dev, dtype=torch.float64)
        if world > 1:
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    ms = max_over_ranks(ms)
    ms_step = ms / args.steps
    value = T_total * args.steps / (ms / 1e3)
    # end to end: each rank's token rows and router logits copied in from
    # pinned host memory, the last layer's output copied out, every step
    pin_x = x.cpu().pin_memory()
    pin_logits = logits.cpu().pin_memory()
    pin_out = torch.empty((T, 2048), dtype=torch.bfloat16).pin_memory()
    dist.barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(args.steps):
        x.copy_(pin_x, non_blocking=True)
        logits.copy_(pin_logits, non_blocking=True)
        run_step()
        pin_out.copy_(outs[0], non_blocking=True)
    e1.record()
    torch.cuda.synchronize()
    e2e_ms = max_over_ranks(e0.elapsed_time(e1))
    peaks = json.loads((ROOT / 'MEASURED_PEAKS.json').read_text()) if (ROOT / 'MEASURED_PEAKS.json').exists() else {}
    flags_max = int(max_over_ranks(float(max(rflags.item(), max(int(ly.flags.item()) for ly in layers)))))
    ops_step = 2.0 * routes_step * MACS_PER_ROUTE
    bytes_step = L * 256 * EXPERT_BYTES + 2 * L * T_total * 4096
    tops = ops_step / (ms_step * 1e-3) / 1e12
    hbm_gbs = bytes_step / (ms_step * 1e-3) / 1e9
    if cfg['T'] > 64:
        dense = measure_dense_peaks(torch, dev, seconds=1.0) if rank == 0 else {}
        tpeak = max(dense.get('int8_tops', 0.0), dense.get('fp8_tflops', 0.0)) or 2 * peaks.get('bf16_tflops', 1590.0)
        roofline = {'bound': 'tensor', 'achieved': round(tops, 1), 'peak': round(tpeak * world, 1), 'unit': 'TOP/s',
                    'frac': round(tops / (tpeak * world), 4), 'algorithmic_ops_per_step': ops_step,
                    'peak_source': 'world x rank 0 int8/fp8 dense burst, measured in line (of measured)',
                    'dense_tensor_peaks_rank0': dense}
    else:
        hpeak = peaks.get('hbm_gbs', 6650.0)
        roofline = {'bound': 'hbm', 'achieved': round(hbm_gbs, 1), 'peak': round(hpeak * world, 1), 'unit': 'GB/s',
                    'frac': round(hbm_gbs / (hpeak * world), 4), 'algorithmic_bytes_per_step': bytes_step,
                    'peak_source': 'world x MEASURED_PEAKS.json hbm_gbs (of measured)'}
    roofline.update({
        'traffic': None, 'kernel': 'whole expert-parallel step, max over ranks',
        'nvlink': {'bytes_per_layer_all_ranks': round(nvlink_step / L), 'bytes_per_layer_max_rank':
                   round(nvlink_rank_max / L), 'peak_gbs_per_rank': 770.0,
                   'bound_ms_per_step': round(nvlink_rank_max / 770e9 * 1e3, 4),
                   'peak_source': 'measured peer copy 770 GB/s per direction per GPU (profiling recipe)'}})
    result = {
        'metric': METRIC, 'value': round(value, 3), 'unit': 'tokens/s', 'n_gpus': world, 'steps': args.steps,
        'warmup': args.warmup, 'ms_per_step': round(ms_step, 4), 'higher_is_better': True,
        'scaling': 'strong', 'vs_baseline': None, 'dtype': 'int8',
        'data': 'synthetic (seeded random-init weights and logits of the configured shapes)',
        'config': {'workload': cfg['name'], 'tokens_per_step': T_total, 'tokens_per_rank': T, 'layers': L,
                   'experts_per_rank': epr, 'parallelism': f'ep{world}',
                   'placement': ('balanced by routed load of a 4096-token calibration batch'
                                 if args.placement == 'balanced' else 'contiguous ranges'),
                   'combine': ('per-slot fp32 rows, bit-identical to one GPU' if args.combine == 'exact' else
                               'per-rank fp32 partial sums, equal to one GPU within fp32 rounding'),
                   'exchange': 'none: one rank holds all 256 experts' if world == 1 else ({('fixed', 'nccl'): 'NCCL all_gather of token rows + equal-block all_to_all of '
                                                   'fp32 per-slot rows (no host synchronisation)',
                                 ('compact', 'nccl'): 'NCCL all_to_all_single dispatch + fp32 per-slot return '
                                                      '(variable splits)',
                                 ('fixed', 'p2p'): 'token rows to every rank and owned fp32 slots to their home '
                                                   'as NVLink peer stores (double-buffered, no collective)',
                                 ('compact', 'p2p'): 'NCCL count all_gather, then token rows and fp32 per-slot '
                                                     'rows as NVLink peer stores'}[(cfg['exchange'],
                                                                                    args.ep_transport)]),
                   'chunks': args.ep_chunks if cfg['exchange'] == 'compact' else 1,
                   'transport': 'NVLink peer stores' if args.ep_transport == 'p2p' else 'NCCL',
                   'routing': 'device top-8 of each rank\'s router logits inside the step',
                   'single_gpu_line_differs': 'the plain-process line (BASELINE run) is decode B=1; '
                                             'this expert-parallel workload is what torchrun runs at every N'},
        'e2e': {'value': round(T_total * args.steps / (e2e_ms / 1e3), 3), 'unit': 'tokens/s',
                'h2d_bytes_per_step': T * 4096 + L * T * 1024, 'd2h_bytes_per_step': T * 4096,
                'per': 'rank (every rank copies its own rows; time = max over ranks)'},
        'gpu_launches': int(launches), 'roofline': roofline,
        'flags_max': flags_max, 'clocks': clk.summary(), 'cuda_graph': graph is not None,
    }
    dist.barrier()
    step = run_step = None
    graph = None  # a graph holding NCCL calls is released before the process group
    torch.cuda.synchronize()
    for layer in layers:
        layer.close()   # peer-memory buffers, collectively
    dist.destroy_process_group()
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        result['cpu_baseline'] = cpu_baseline(cfg, args.cpu_seconds)
    if rank == 0:
        print(json.dumps(result), flush=True)


def run_dense(args):
    """Dense G256 projections (ornith_dense_g256_launch, N16 banks): one step =
    the step's rows through 40 independent banks, captured as one CUDA graph.
    Roofline: the algorithmic bytes of one call (codes N*K/2, metadata N*K/64,
    bf16 rows in and out, the fp32 diagnostic row out) over its share of the
    step's CUDA-event time."""
    import torch
    cfg = dict(CONFIGS[args.config])
    if args.layers:
        cfg['layers'] = args.layers
    dev = torch.device('cuda', 0)
    torch.cuda.set_device(dev)
    graft.load_package()
    import importlib
    native = importlib.import_module('ornith_b200.native')
    lib = native.lib()
    M, L, N, K = cfg['T'], cfg['layers'], cfg['N'], cfg['K']
    gen = torch.Generator(device=dev)
    gen.manual_seed(777)
    banks = []
    for _ in range(L):
        codes = torch.randint(-2 ** 31, 2 ** 31 - 1, (N // 16, K // 256, 32, 16), dtype=torch.int32, device=dev,
                              generator=gen).view(torch.uint32)
        z = torch.randn((N // 16, K // 256, 16), device=dev, generator=gen)
        scale = (0.01 * z.abs()).to(torch.float16).clamp_min(2 ** -14)
        offset = (scale.float() * -8.0).to(torch.float16)
        meta = ((scale.view(torch.int16).to(torch.int32) & 0xFFFF) |
                (offset.view(torch.int16).to(torch.int32) << 16)).view(torch.uint32)
        banks.append((codes, meta))
    x = torch.randn((M, K), device=dev, generator=gen).to(torch.bfloat16)
    outs = [torch.empty((M, N), dtype=torch.bfloat16, device=dev) for _ in range(2)]
    ws = torch.empty(native.dense_workspace_bytes(M, [(N, K)]), dtype=torch.uint8, device=dev)
    flags = torch.zeros(1, dtype=torch.int32, device=dev)

    def call(l):
        native.dense_out(x, banks[l][0], banks[l][1], ws, outs[l % 2], flags, M, N, K, 2, M)

    def step():
        for l in range(L):
            call(l)

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        step()
    torch.cuda.current_stream().wait_stream(side)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        step()
    for _ in range(args.warmup):
        graph.replay()
    torch.cuda.synchronize()
    launches = launches_per_step(lib, step) * args.steps
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(0) as clk:
        start.record()
        for _ in range(args.steps):
            graph.replay()
        end.record()
        torch.cuda.synchronize()
    ms = start.elapsed_time(end)
    # one launch = one bank's call inside the captured step (the step's device
    # time over its L calls; eager calls would add host launch gaps)
    launch_ms = ms / args.steps / L
    algo = N * K // 2 + N * (K // 256) * 4 + M * K * 2 + M * N * 2 + M * N * 4
    peaks = json.loads((ROOT / 'MEASURED_PEAKS.json').read_text()) if (ROOT / 'MEASURED_PEAKS.json').exists() else {}
    peak = peaks.get('hbm_gbs', 6650.0)
    achieved = algo / (launch_ms * 1e-3) / 1e9
    # end to end through the operator: pinned rows in, last output out
    pin_x = x.cpu().pin_memory()
    pin_out = torch.empty((M, N), dtype=torch.bfloat16).pin_memory()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(args.steps):
        x.copy_(pin_x, non_blocking=True)
        graph.replay()
        pin_out.copy_(outs[(L - 1) % 2], non_blocking=True)
    e1.record()
    torch.cuda.synchronize()
    e2e_ms = e0.elapsed_time(e1)
    line = {
        'metric': 'dense G256 projection rows/s (40-bank step) & % of HBM roofline', 'value': round(
            M * L * args.steps / (ms / 1e3), 3), 'unit': 'row-projections/s', 'n_gpus': 1, 'steps': args.steps,
        'warmup': args.warmup, 'ms_per_step': round(ms / args.steps, 4), 'higher_is_better': True,
        'scaling': 'weak', 'vs_baseline': None, 'dtype': 'int8', 'data': 'synthetic (seeded random banks)',
        'config': {'workload': cfg['name'], 'rows': M, 'N': N, 'K': K, 'banks': L,
                   'l2': f'inputs larger than L2: {L * algo / 1e6:.0f} MB per step'},
        'e2e': {'value': round(M * L * args.steps / (e2e_ms / 1e3), 3), 'unit': 'row-projections/s',
                'h2d_bytes_per_step': M * K * 2, 'd2h_bytes_per_step': M * N * 2},
        'gpu_launches': int(launches),
        'roofline': {'bound': 'hbm', 'achieved': round(achieved, 1), 'peak': peak, 'unit': 'GB/s',
                     'frac': round(achieved / peak, 4),
                     'traffic': NCU_TRAFFIC[args.config]['bytes'] if args.config in NCU_TRAFFIC else None,
                     'kernel': ('one dense call: dense_fused_kernel<16>' if M <= 4 else
                                'one dense call: dense_quant_kernel + dense_project_kernel<16>'),
                     'algorithmic_bytes_per_launch': algo, 'launch_ms': round(launch_ms, 5),
                     'peak_source': 'MEASURED_PEAKS.json hbm_gbs (of measured)' if peaks else 'fallback 6650 GB/s'},
        'flags': int(flags.item()), 'clocks': clk.summary(), 'cuda_graph': True,
    }
    if not args.no_cpu_baseline:
        line['cpu_baseline'] = cpu_baseline_projection(cfg, min(args.cpu_seconds, 5.0))
    print(json.dumps(line), flush=True)


def run_head(args):
    """W8 LM head (ornith_b200::head_out): one step = the step's rows through
    the full-vocabulary bank, captured as a CUDA graph.  Roofline: algorithmic
    bytes of one launch (int8 codes N*K, fp16 scales N*32, bf16 rows in, bf16
    logits and the fp32 diagnostic out) over its CUDA-event time."""
    import torch
    cfg = dict(CONFIGS[args.config])
    dev = torch.device('cuda', 0)
    torch.cuda.set_device(dev)
    graft.load_package()
    import importlib
    native = importlib.import_module('ornith_b200.native')
    lib = native.lib()
    M, N, K = cfg['T'], cfg['N'], cfg['K']
    gen = torch.Generator(device=dev)
    gen.manual_seed(555)
    codes = torch.randint(-127, 128, (N // 16, K // 16, 4, 16, 4), dtype=torch.int8, device=dev, generator=gen)
    words = codes.view(torch.int32).view(N // 16, K // 16, 4, 16).view(torch.uint32)
    scales = (0.01 * torch.randn((N, K // 128), device=dev, generator=gen).abs()).to(torch.float16).clamp_min(2 ** -14)
    x = torch.randn((M, K), device=dev, generator=gen).to(torch.bfloat16)
    out = torch.empty((M, N), dtype=torch.bfloat16, device=dev)
    ws = torch.empty(native.head_get_layout(native.HEAD_ROWS, N).workspace_bytes, dtype=torch.uint8, device=dev)
    flags = torch.zeros(1, dtype=torch.int32, device=dev)

    def step():
        native.head_out(x, words, scales, ws, out, flags, 2)

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        step()
    torch.cuda.current_stream().wait_stream(side)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        step()
    for _ in range(args.warmup):
        graph.replay()
    torch.cuda.synchronize()
    launches = launches_per_step(lib, step) * args.steps
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(0) as clk:
        start.record()
        for _ in range(args.steps):
            graph.replay()
        end.record()
        torch.cuda.synchronize()
    ms = start.elapsed_time(end)
    algo = N * K + N * (K // 128) * 2 + M * K * 2 + M * N * 2 + M * N * 4
    peaks = json.loads((ROOT / 'MEASURED_PEAKS.json').read_text()) if (ROOT / 'MEASURED_PEAKS.json').exists() else {}
    peak = peaks.get('hbm_gbs', 6650.0)
    launch_ms = ms / args.steps
    achieved = algo / (launch_ms * 1e-3) / 1e9
    pin_x = x.cpu().pin_memory()
    pin_out = torch.empty((M, N), dtype=torch.bfloat16).pin_memory()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(args.steps):
        x.copy_(pin_x, non_blocking=True)
        graph.replay()
        pin_out.copy_(out, non_blocking=True)
    e1.record()
    torch.cuda.synchronize()
    e2e_ms = e0.elapsed_time(e1)
    line = {
        'metric': 'W8 LM head rows/s & % of HBM roofline', 'value': round(M * args.steps / (ms / 1e3), 3),
        'unit': 'rows/s', 'n_gpus': 1, 'steps': args.steps, 'warmup': args.warmup,
        'ms_per_step': round(launch_ms, 4), 'higher_is_better': True, 'scaling': 'weak', 'vs_baseline': None,
        'dtype': 'int8', 'data': 'synthetic (seeded random int8 bank)',
        'config': {'workload': cfg['name'], 'rows': M, 'N': N, 'K': K,
                   'l2': f'inputs larger than L2: {algo / 1e6:.0f} MB per step'},
        'e2e': {'value': round(M * args.steps / (e2e_ms / 1e3), 3), 'unit': 'rows/s',
                'h2d_bytes_per_step': M * K * 2, 'd2h_bytes_per_step': M * N * 2},
        'gpu_launches': int(launches),
        'roofline': {'bound': 'hbm', 'achieved': round(achieved, 1), 'peak': peak, 'unit': 'GB/s',
                     'frac': round(achieved / peak, 4),
                     'traffic': NCU_TRAFFIC[args.config]['bytes'] if args.config in NCU_TRAFFIC else None,
                     'kernel': 'one head launch (head_quant_kernel + head_project_kernel)',
                     'algorithmic_bytes_per_launch': algo, 'launch_ms': round(launch_ms, 5),
                     'peak_source': 'MEASURED_PEAKS.json hbm_gbs (of measured)' if peaks else 'fallback 6650 GB/s'},
        'flags': int(flags.item()), 'clocks': clk.summary(), 'cuda_graph': True,
    }
    if not args.no_cpu_baseline:
        line['cpu_baseline'] = cpu_baseline_projection(cfg, min(args.cpu_seconds, 5.0))
    print(json.dumps(line), flush=True)


def launches_per_step(lib, step_fn):
    """Kernels one step enqueues: counted by running the step eagerly once."""
    import torch
    n0 = lib.ornith_moe_b200_kernel_launches()
    step_fn()
    torch.cuda.synchronize()
    return lib.ornith_moe_b200_kernel_launches() - n0


def e2e_pipelined(torch, steps, pin_x, pin_logits, x_static, static_logits, out_dev, pin_out, replay, e0, e1):
    """The e2e steps with their host copies overlapped, as a serving engine
    runs them: step s+1's inputs go from pinned host memory into a device
    staging pair on an upload stream while step s computes; the compute
    stream moves them into the captured step's input buffers (device copies)
    and, after the step, its output into an output staging pair, which a
    download stream copies to pinned host memory while the next step runs.
    Events order every reuse of a staging buffer.  e0/e1 bracket all of it:
    the first upload waits for e0 and e1 waits for the last download."""
    comp = torch.cuda.current_stream()
    up, down = torch.cuda.Stream(), torch.cuda.Stream()
    stage_x = [torch.empty_like(x_static) for _ in range(2)]
    stage_l = [torch.empty_like(static_logits) for _ in range(2)]
    stage_o = [torch.empty_like(out_dev) for _ in range(2)]
    uploaded = [torch.cuda.Event() for _ in range(2)]     # stage k holds step s's inputs
    consumed = [torch.cuda.Event() for _ in range(2)]     # the compute stream has read stage k
    produced = [torch.cuda.Event() for _ in range(2)]     # stage_o k holds step s's output
    downloaded = [torch.cuda.Event() for _ in range(2)]   # stage_o k has reached the host
    n_sets = pin_logits.shape[0]

    def upload(s):
        k = s % 2
        with torch.cuda.stream(up):
            if s >= 2:
                up.wait_event(consumed[k])
            stage_x[k].copy_(pin_x, non_blocking=True)
            stage_l[k].copy_(pin_logits[s % n_sets], non_blocking=True)
            uploaded[k].record(up)

    e0.record(comp)
    up.wait_event(e0)
    upload(0)
    for s in range(steps):
        k = s % 2
        comp.wait_event(uploaded[k])
        x_static.copy_(stage_x[k])
        static_logits.copy_(stage_l[k])
        consumed[k].record(comp)
        if s + 1 < steps:
            upload(s + 1)
        replay()
        if s >= 2:
            comp.wait_event(downloaded[k])
        stage_o[k].copy_(out_dev)
        produced[k].record(comp)
        with torch.cuda.stream(down):
            down.wait_event(produced[k])
            pin_out.copy_(stage_o[k], non_blocking=True)
            downloaded[k].record(down)
    comp.wait_stream(down)
    comp.wait_stream(up)
    e1.record(comp)
    torch.cuda.synchronize()   # the staging buffers are released when this returns


def measure_dense_peaks(torch, dev, seconds=2.0):
    """Dense int8 and fp8 tensor-core rates of this GPU, measured in line:
    torch._int_mm (int8 x int8 -> int32) and torch._scaled_mm (fp8 e4m3 ->
    bf16), both 8192^3 (2 * 8192^3 operations per call), as the best of ten
    calls (burst) and over `seconds` of back-to-back calls (sustained).  The
    prefill roofline uses the higher of the two burst figures as its peak."""
    n = 8192
    out = {}
    gen = torch.Generator(device=dev)
    gen.manual_seed(3)

    def rate(fn):
        for _ in range(3):
            fn()
        torch.cuda.synchronize()
        best = float('inf')
        for _ in range(10):
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            fn()
            e1.record()
            e1.synchronize()
            best = min(best, e0.elapsed_time(e1))
        calls = max(1, int(seconds / (best * 1e-3)))
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(calls):
            fn()
        e1.record()
        e1.synchronize()
        ops = 2.0 * n ** 3
        return round(ops / (best * 1e-3) / 1e12, 1), round(ops * calls / (e0.elapsed_time(e1) * 1e-3) / 1e12, 1)

    try:
        a = torch.randint(-127, 128, (n, n), dtype=torch.int8, device=dev, generator=gen)
        b = torch.randint(-127, 128, (n, n), dtype=torch.int8, device=dev, generator=gen).t()
        out['int8_tops'], out['int8_tops_sustained'] = rate(lambda: torch._int_mm(a, b))
        del a, b
    except Exception as exc:  # no int8 GEMM on this build: the fp8 figure stands alone
        out['int8_error'] = repr(exc)[:120]
    try:
        a = torch.randn((n, n), device=dev, generator=gen).to(torch.float8_e4m3fn)
        b = torch.randn((n, n), device=dev, generator=gen).to(torch.float8_e4m3fn).t()
        one = torch.ones((), device=dev)
        out['fp8_tflops'], out['fp8_tflops_sustained'] = rate(
            lambda: torch._scaled_mm(a, b, scale_a=one, scale_b=one, out_dtype=torch.bfloat16))
        del a, b
    except Exception as exc:
        out['fp8_error'] = repr(exc)[:120]
    torch.cuda.empty_cache()
    out['how'] = ('torch._int_mm int8 and torch._scaled_mm fp8 e4m3, 8192^3: best of 10 calls (burst), '
                  f'{seconds:.0f} s back to back (sustained)')
    return out


def measure_layer_config(torch, native, lib, stack, cfg, args, dev, peaks, dense_peaks):
    """One workload (a CONFIGS entry) on the resident 40-layer stack: W
    warm-up steps, K timed steps of a captured CUDA graph (router logits of
    each step copied in first), then the same steps end to end with pinned
    host inputs copied in and the output copied out inside the timed region.
    Returns the workload's part of the JSON line."""
    T, L, bits = cfg['T'], cfg['layers'], cfg['act_bits']
    steps_total = args.warmup + args.steps
    bias = (cfg['bias'] * torch.randn((L, 256), device=dev, generator=stack.gen)) if cfg['bias'] else None
    n_logit_sets = steps_total if T <= 64 else 1
    logits = torch.randn((n_logit_sets, L, T, 256), device=dev, generator=stack.gen)
    if bias is not None:
        logits += bias[None, :, None, :]
    x0 = torch.randn((T, 2048), device=dev, generator=stack.gen).to(torch.bfloat16)
    hidden = cfg.get('entry') == 'hidden'
    if hidden:
        # the router computes the logits from a fresh token row every step
        routers = [(0.02 * torch.randn((256, 2048), device=dev, generator=stack.gen)).to(torch.bfloat16)
                   for _ in range(L)]
        x_sets = torch.randn((n_logit_sets, T, 2048), device=dev, generator=stack.gen).to(torch.bfloat16)
        logits_out = torch.empty((L, T, 256), device=dev)
        logits = torch.stack([torch.stack([x_sets[s].float() @ routers[l].float().t() for l in range(L)])
                              for s in range(n_logit_sets)])
        x0 = x_sets[0]
    ws = torch.empty(native.workspace_bytes(T), dtype=torch.uint8, device=dev)
    outs = [torch.empty((T, 2048), dtype=torch.bfloat16, device=dev) for _ in range(2)]
    shared_out = torch.empty((T, 2048), dtype=torch.bfloat16, device=dev) if cfg['shared'] else None
    flags = torch.zeros(L, dtype=torch.int32, device=dev)
    L_stack = len(stack.layers)

    def layer_call(l, x, lg, out):
        (gc, gm), (dc, dm), (sgc, sgm), (sdc, sdm), gw = stack.layers[l % L_stack]
        if hidden:
            native.routed_from_hidden(x, routers[l], logits_out[l], gc, gm, dc, dm, sgc, sgm, sdc, sdm, gw,
                                      stack.silu, stack.sigmoid, ws, out, shared_out, flags[l:l + 1], T, bits)
        elif cfg['shared']:
            native.routed_from_logits(x, lg, gc, gm, dc, dm, sgc, sgm, sdc, sdm, gw, stack.silu, stack.sigmoid,
                                      ws, out, shared_out, flags[l:l + 1], T, bits)
        else:
            native.routed_from_logits(x, lg, gc, gm, dc, dm, None, None, None, None, None, None, None,
                                      ws, out, None, flags[l:l + 1], T, bits)

    static_logits = logits[0].clone()
    x_static = x0.clone() if hidden else x0

    def step_static():
        for l in range(L):
            layer_call(l, x_static, static_logits[l], outs[l % 2])

    def stage_inputs(s):
        if hidden:
            x_static.copy_(x_sets[s % n_logit_sets], non_blocking=True)
        else:
            static_logits.copy_(logits[s % n_logit_sets], non_blocking=True)

    # algorithmic bytes per step: (distinct experts + 1) * EXPERT_BYTES per layer + activations
    ids = torch.topk(logits, 8, dim=-1).indices  # [sets, L, T, 8]
    distinct = []
    for s in range(n_logit_sets):
        d = 0
        for l in range(L):
            d += int(torch.unique(ids[s, l]).numel()) + (1 if cfg['shared'] else 0)
        distinct.append(d)
    del ids
    act_bytes = L * (2 * T * 4096 + T * 1024) + (L * 256 * 2048 * 2 if hidden else 0)  # + router weights

    def step_bytes(s):
        return distinct[s % n_logit_sets] * EXPERT_BYTES + act_bytes

    for s in range(args.warmup):
        stage_inputs(s)
        step_static()
    torch.cuda.synchronize()
    graph, graph_error = None, None
    if not args.no_graph:
        try:
            side = torch.cuda.Stream()
            side.wait_stream(torch.cuda.current_stream())
            with torch.cuda.stream(side):
                step_static()
            torch.cuda.current_stream().wait_stream(side)
            torch.cuda.synchronize()
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph):
                step_static()
            torch.cuda.synchronize()
        except Exception as exc:  # capture unsupported: time the eager launches instead
            graph, graph_error = None, repr(exc)[:200]
            torch.cuda.synchronize()

    def run_step(s):
        stage_inputs(s)
        if graph is not None:
            graph.replay()
        else:
            step_static()

    for s in range(args.warmup):
        run_step(s)
    torch.cuda.synchronize()
    launches0 = lib.ornith_moe_b200_kernel_launches()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(dev.index) as clk:
        start.record()
        for s in range(args.warmup, steps_total):
            run_step(s)
        end.record()
        torch.cuda.synchronize()
    per_step_launches = launches_per_step(lib, step_static)
    launches = (lib.ornith_moe_b200_kernel_launches() - launches0) if graph is None else per_step_launches * args.steps
    ms = start.elapsed_time(end)
    ms_step = ms / args.steps
    value = T * args.steps / (ms / 1e3)
    bytes_step = sum(step_bytes(s) for s in range(args.warmup, steps_total)) / args.steps
    hbm_peak = peaks.get('hbm_gbs', 6650.0)
    peak_src = 'MEASURED_PEAKS.json hbm_gbs (of measured)' if peaks else 'fallback 6650 GB/s (of fallback)'
    gbs = bytes_step / (ms_step * 1e-3) / 1e9
    per_layer_launches = per_step_launches / L
    hbm = {'bound': 'hbm', 'achieved': round(gbs, 1), 'peak': hbm_peak, 'unit': 'GB/s',
           'frac': round(gbs / hbm_peak, 4), 'algorithmic_bytes_per_step': int(bytes_step),
           'kernel': ('the layer kernels back to back in one captured step: '
                      f'{per_layer_launches:g} launch(es) per layer, {L} layers; achieved = algorithmic bytes '
                      'of the timed steps over their CUDA-event time'),
           'launch_ms': round(ms_step / L, 5), 'peak_source': peak_src}
    traffic = NCU_TRAFFIC.get(cfg['key'])
    if T > 64:
        ops_step = 2.0 * L * T * 8 * MACS_PER_ROUTE
        tops = ops_step / (ms_step * 1e-3) / 1e12
        tpeak = max(dense_peaks.get('int8_tops', 0.0), dense_peaks.get('fp8_tflops', 0.0))
        src = 'measured in line: max of int8 / fp8 dense burst (of measured)'
        if not tpeak:
            tpeak, src = 2 * peaks.get('bf16_tflops', 1590.0), '2 x bf16 (of measured bf16; no int8/fp8 figure)'
        roofline = {'bound': 'tensor', 'achieved': round(tops, 1), 'peak': tpeak, 'unit': 'TOP/s',
                    'frac': round(tops / tpeak, 4), 'algorithmic_ops_per_step': ops_step,
                    'kernel': hbm['kernel'], 'launch_ms': hbm['launch_ms'], 'peak_source': src,
                    'hbm': hbm}
    else:
        roofline = hbm
    roofline['traffic'] = traffic['bytes'] if traffic else None
    if traffic:
        roofline['traffic_kernel'] = traffic['kernel'] + ' (per launch, ncu)'

    # end to end through the public operator: pinned host inputs copied in, the
    # step (graph of the operator's launches) run, the last output copied out
    pin_x = (x_sets[: min(n_logit_sets, 4)] if hidden else x0).cpu().pin_memory()
    pin_logits = logits[: min(n_logit_sets, 4)].cpu().pin_memory()
    pin_out = torch.empty((T, 2048), dtype=torch.bfloat16).pin_memory()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    replay = graph.replay if graph is not None else step_static
    if args.e2e_overlap and not hidden:
        e2e_pipelined(torch, args.steps, pin_x, pin_logits, x_static, static_logits, outs[(L - 1) % 2], pin_out,
                      replay, e0, e1)
    else:
        e0.record()
        for s in range(args.steps):
            if hidden:
                x_static.copy_(pin_x[s % pin_x.shape[0]], non_blocking=True)
            else:
                x_static.copy_(pin_x, non_blocking=True)
                static_logits.copy_(pin_logits[s % pin_logits.shape[0]], non_blocking=True)
            replay()
            pin_out.copy_(outs[(L - 1) % 2], non_blocking=True)
        e1.record()
    torch.cuda.synchronize()
    e2e_ms = e0.elapsed_time(e1)
    part = {
        'value': round(value, 3), 'unit': 'tokens/s', 'ms_per_step': round(ms_step, 4),
        'config': {'workload': cfg['name'], 'tokens_per_step': T, 'layers': L, 'experts': 256, 'top_k': 8,
                   'hidden': 2048, 'intermediate': 512, 'shared_expert': cfg['shared'],
                   'weights': 'affine-u4 G256 (scale, offset=-8*scale), N32 storage',
                   'activations': f'A{bits} per 256-group after H128', 'arith': 'u4 x s8 -> int32 dot, fp32 epilogue',
                   'l2': f'inputs larger than L2: {bytes_step / 1e6:.0f} MB of weights read per step'},
        'e2e': {'value': round(T * args.steps / (e2e_ms / 1e3), 3), 'unit': 'tokens/s',
                'h2d_bytes_per_step': T * 4096 + (0 if hidden else L * T * 1024), 'd2h_bytes_per_step': T * 4096,
                'copies': ('pipelined on copy streams, inside the timed region' if args.e2e_overlap and not hidden
                           else 'in line with the steps')},
        'gpu_launches': int(launches),
        'roofline': roofline,
        'flags_max': int(flags.max().item()),
        'cuda_graph': graph is not None,
        'clocks': clk.summary(),
    }
    if graph_error:
        part['cuda_graph_error'] = graph_error
    graph = None
    del ws, logits
    torch.cuda.synchronize()
    torch.cuda.empty_cache()
    return part


def run(args):
    """Single-GPU workloads of the routed layer: the named config as the line,
    and (for the default decode B=1 line) decode B=32, prefill 1120 and
    prefill 8192 measured in the same process on the same resident weights
    as `sub_results`, each with its own timing, roofline and clocks."""
    import torch
    cfg = dict(CONFIGS[args.config], key=args.config)
    if args.layers:
        cfg['layers'] = args.layers
    dev = torch.device('cuda', 0)
    torch.cuda.set_device(dev)
    graft.load_package()
    import importlib
    native = importlib.import_module('ornith_b200.native')
    lib = native.lib()
    peaks = json.loads((ROOT / 'MEASURED_PEAKS.json').read_text()) if (ROOT / 'MEASURED_PEAKS.json').exists() else {}
    subs = [] if (args.no_sub or args.layers) else list(SUB_CONFIGS.get(args.config, []))
    need_tensor = cfg['T'] > 64 or any(CONFIGS[k]['T'] > 64 for k in subs)
    dense_peaks = measure_dense_peaks(torch, dev) if need_tensor else {}
    stack = Stack(torch, cfg, dev, seed=1234)
    main = measure_layer_config(torch, native, lib, stack, cfg, args, dev, peaks, dense_peaks)
    result = {
        'metric': METRIC, 'value': main['value'], 'unit': 'tokens/s', 'n_gpus': 1,
        'steps': args.steps, 'warmup': args.warmup, 'ms_per_step': main['ms_per_step'],
        'higher_is_better': True, 'scaling': 'weak', 'vs_baseline': None, 'dtype': 'int8',
        'data': 'synthetic (seeded random-init weights and logits of the configured shapes)',
        'config': dict(main['config'], parallelism='single GPU'),
        'e2e': main['e2e'], 'gpu_launches': main['gpu_launches'], 'roofline': main['roofline'],
        'flags_max': main['flags_max'], 'cuda_graph': main['cuda_graph'], 'clocks': main['clocks'],
    }
    if 'cuda_graph_error' in main:
        result['cuda_graph_error'] = main['cuda_graph_error']
    if subs:
        result['sub_results'] = {}
        for key in subs:
            sub_cfg = dict(CONFIGS[key], key=key)
            result['sub_results'][key] = measure_layer_config(torch, native, lib, stack, sub_cfg, args, dev, peaks,
                                                              dense_peaks)
    if dense_peaks:
        result['dense_tensor_peaks'] = dense_peaks
    if not args.no_cpu_baseline:
        result['cpu_baseline'] = cpu_baseline(cfg, args.cpu_seconds)
    print(json.dumps(result), flush=True)


# ---------------------------------------------------------------------------
# CPU legs (oracle port for cpu_baseline; compiled reference for --impl reference)
# ---------------------------------------------------------------------------
def _cpu_layer(seed=5):
    graft.load_package()
    import importlib
    S = importlib.import_module('ornith_b200.synthetic')
    return S, S.make_layer(np.random.default_rng(seed))


def cpu_baseline(cfg, seconds):
    from oracle import oracle as O
    S, layer = _cpu_layer()
    cores = O.set_threads(os.cpu_count() or 1)
    tab = np.load(ROOT / 'tests' / 'golden' / 'shared_math_tables.npz')
    rng = np.random.default_rng(9)
    T = min(cfg['T'], 64)
    n, t0 = 0, time.perf_counter()
    while time.perf_counter() - t0 < seconds or n < 2:
        x = S.make_tokens(rng, T)
        logits = rng.standard_normal((T, 256)).astype(np.float32)
        w, ids = O.route_topk(logits)
        if cfg['shared']:
            logit = S.f32_to_bf16_bits(rng.standard_normal(T).astype(np.float32))
            O.routed_layer_shared(x, w, ids, layer.gate_codes, layer.gate_meta, layer.down_codes, layer.down_meta,
                                  layer.sgate_codes, layer.sgate_meta, layer.sdown_codes, layer.sdown_meta, logit,
                                  tab['silu_fp32'], tab['sigmoid_bf16'])
        else:
            O.routed_layer(x, w, ids, layer.gate_codes, layer.gate_meta, layer.down_codes, layer.down_meta,
                           a8=cfg['act_bits'] == 8)
        n += 1
    layer_s = (time.perf_counter() - t0) / n
    tokens_per_s = T / (layer_s * cfg['layers'])
    return {'value': round(tokens_per_s, 4), 'unit': 'tokens/s', 'cores': cores, 'kind': 'port',
            'sample': f'{n} single-layer calls of T={T} (oracle C port, OpenMP), scaled to a {cfg["layers"]}-layer step'}


def run_reference(args):
    cfg = CONFIGS[args.config]
    rank = int(os.environ.get('RANK', '0'))
    if rank != 0:
        return
    from oracle import oracle as O
    if not O.reference_available():
        print(json.dumps({'impl': 'reference', 'unavailable': 'oracle/_ref was not built (needs the reference checkout)'}))
        return
    if cfg.get('dense'):
        return run_reference_dense(args, cfg, O)
    if cfg.get('head'):
        return run_reference_head(args, cfg, O)
    S, layer = _cpu_layer()
    tab = np.load(ROOT / 'tests' / 'golden' / 'shared_math_tables.npz')
    rng = np.random.default_rng(10)
    T = min(cfg['T'], 16 if cfg['shared'] else 64)
    layers_per_step = 2
    # inputs drawn before any timing: the timed loop runs only the reference's layer calls
    pool = []
    for _ in range(4 * layers_per_step):
        x = S.make_tokens(rng, T)
        w, ids = O.route_topk(rng.standard_normal((T, 256)).astype(np.float32))
        logit = S.f32_to_bf16_bits(rng.standard_normal(T).astype(np.float32))
        pool.append((x, w, ids, logit))
    entry = 'ornith_routed_direct_launch' if cfg['act_bits'] == 8 else 'ornith_routed_direct_launch_a4'
    calls = [0]

    def one():
        for _ in range(layers_per_step):
            x, w, ids, logit = pool[calls[0] % len(pool)]
            calls[0] += 1
            if cfg['shared']:
                O.ref_routed_shared(x, w, ids, layer.gate_codes, layer.gate_meta, layer.down_codes, layer.down_meta,
                                    layer.sgate_codes, layer.sgate_meta, layer.sdown_codes, layer.sdown_meta, logit,
                                    tab['silu_fp32'], tab['sigmoid_bf16'])
            else:
                O.ref_routed(x, w, ids, layer.gate_codes, layer.gate_meta, layer.down_codes, layer.down_meta,
                             entry=entry)

    for _ in range(args.warmup):
        one()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        one()
    el = time.perf_counter() - t0
    layer_s = el / (args.steps * layers_per_step)
    value = T / (layer_s * cfg['layers'])
    cores = os.cpu_count() or 1
    sample = (f'{layers_per_step} layer calls of T={T} per step (reference routed_storage source compiled for the CPU '
              f'with a SIMT shim), scaled to a {cfg["layers"]}-layer step')
    print(json.dumps({
        'impl': 'reference', 'metric': METRIC, 'value': round(value, 4), 'unit': 'tokens/s', 'n_gpus': 0,
        'steps': args.steps, 'warmup': args.warmup, 'ms_per_step': round(el / args.steps * 1e3, 3),
        'higher_is_better': True, 'scaling': 'weak', 'vs_baseline': None, 'dtype': 'int8',
        'data': 'synthetic', 'config': {'workload': cfg['name'], 'tokens_per_step': T},
        'cpu_baseline': {'value': round(value, 4), 'unit': 'tokens/s', 'cores': cores, 'kind': 'reference',
                         'sample': sample},
        'e2e': {'value': round(value, 4), 'unit': 'tokens/s', 'h2d_bytes_per_step': 0, 'd2h_bytes_per_step': 0},
    }), flush=True)


def run_reference_dense(args, cfg, O):
    """The reference's dense library compiled for the CPU (oracle/_ref), one
    bank per call, scaled to the 40-bank step."""
    import importlib.util
    spec = importlib.util.spec_from_file_location('ornith_synthetic', ROOT / 'ornith-ciru-halo-agent_b200' / 'synthetic.py')
    S = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(S)
    rng = np.random.default_rng(10)
    M, N, K, L = cfg['T'], cfg['N'], cfg['K'], cfg['layers']
    codes, meta = S.make_dense_bank(rng, N, K)
    x = S.make_rows(rng, M, K)
    calls = 4
    for _ in range(args.warmup):
        O.ref_dense(x, codes, meta, N, K)
    t0 = time.perf_counter()
    for _ in range(args.steps * calls):
        O.ref_dense(x, codes, meta, N, K)
    el = time.perf_counter() - t0
    call_s = el / (args.steps * calls)
    value = M / call_s
    sample = f'{calls} calls per step of one {N}x{K} bank, {M} rows (reference dense source compiled for the CPU)'
    print(json.dumps({
        'impl': 'reference', 'metric': 'dense G256 projection rows/s (40-bank step) & % of HBM roofline',
        'value': round(value, 4), 'unit': 'row-projections/s', 'n_gpus': 0, 'steps': args.steps,
        'warmup': args.warmup, 'ms_per_step': round(call_s * L * 1e3, 3), 'higher_is_better': True,
        'scaling': 'weak', 'vs_baseline': None, 'dtype': 'int8', 'data': 'synthetic',
        'config': {'workload': cfg['name'], 'rows': M},
        'cpu_baseline': {'value': round(value, 4), 'unit': 'row-projections/s', 'cores': os.cpu_count() or 1,
                         'kind': 'reference', 'sample': sample},
        'e2e': {'value': round(value, 4), 'unit': 'row-projections/s', 'h2d_bytes_per_step': 0,
                'd2h_bytes_per_step': 0},
    }), flush=True)


def _synthetic_module():
    import importlib.util
    spec = importlib.util.spec_from_file_location('ornith_synthetic', ROOT / 'ornith-ciru-halo-agent_b200' / 'synthetic.py')
    S = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(S)
    return S


def run_reference_head(args, cfg, O):
    """The reference's head library compiled for the CPU (oracle/_ref) on a
    65,536-column slice of the vocabulary (a size it supports), scaled to the
    full 248,320 columns."""
    S = _synthetic_module()
    rng = np.random.default_rng(10)
    M, N, slice_n = cfg['T'], cfg['N'], 65536
    words, scales = S.make_head_bank(rng, slice_n)
    x = S.make_rows(rng, M, 2048)
    for _ in range(args.warmup):
        O.ref_head(x, words, scales, slice_n)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        O.ref_head(x, words, scales, slice_n)
    call_s = (time.perf_counter() - t0) / args.steps * (N / slice_n)
    value = M / call_s
    sample = (f'{args.steps} calls of a {slice_n}-column slice, {M} rows (reference head source compiled for '
              f'the CPU), scaled to {N} columns')
    print(json.dumps({
        'impl': 'reference', 'metric': 'W8 LM head rows/s & % of HBM roofline', 'value': round(value, 4),
        'unit': 'rows/s', 'n_gpus': 0, 'steps': args.steps, 'warmup': args.warmup,
        'ms_per_step': round(call_s * 1e3, 3), 'higher_is_better': True, 'scaling': 'weak', 'vs_baseline': None,
        'dtype': 'int8', 'data': 'synthetic', 'config': {'workload': cfg['name'], 'rows': M},
        'cpu_baseline': {'value': round(value, 4), 'unit': 'rows/s', 'cores': os.cpu_count() or 1,
                         'kind': 'reference', 'sample': sample},
        'e2e': {'value': round(value, 4), 'unit': 'rows/s', 'h2d_bytes_per_step': 0, 'd2h_bytes_per_step': 0},
    }), flush=True)


def cpu_baseline_projection(cfg, seconds):
    """The oracle port (C, OpenMP on every host core) on the dense or head
    workload: repeated single-bank calls for about `seconds`, as rows (or row
    projections) per second."""
    from oracle import oracle as O
    S = _synthetic_module()
    rng = np.random.default_rng(11)
    M, N, K = cfg['T'], cfg['N'], cfg['K']
    if cfg.get('head'):
        words, scales = S.make_head_bank(rng, N)
        call = lambda x: O.head_project(x, words, scales, N)  # noqa: E731
    else:
        codes, meta = S.make_dense_bank(rng, N, K)
        call = lambda x: O.dense_project(x, codes, meta, N, K, 16)  # noqa: E731
    x = S.make_rows(rng, M, K)
    call(x)
    n, t0 = 0, time.perf_counter()
    while time.perf_counter() - t0 < seconds or n == 0:
        call(x)
        n += 1
    per_call = (time.perf_counter() - t0) / n
    return {'value': round(M / per_call, 4), 'unit': 'rows/s' if cfg.get('head') else 'row-projections/s',
            'cores': O.set_threads(0), 'kind': 'port',
            'sample': f'{n} calls of one {N}x{K} bank with {M} rows (oracle C port, OpenMP)'}


if __name__ == '__main__':
    a = parse()
    if a.impl == 'reference':
        run_reference(a)
    elif CONFIGS[a.config].get('ep'):
        run_ep(a)
    elif CONFIGS[a.config].get('dense'):
        run_dense(a)
    elif CONFIGS[a.config].get('head'):
        run_head(a)
    else:
        if int(os.environ.get('WORLD_SIZE', '1')) > 1:
            raise SystemExit(f'--config {a.config} runs on one GPU; the multi-GPU workloads are ep_prefill8192 '
                             'and ep_decode256')
        run(a)
