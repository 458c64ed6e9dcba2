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
# capture of the same workload (profiles/decode_layer_kernel_decode1.md,
# profiles/decode_layer_kernel_decode32.md, profiles/prefill_mma_kernel_prefill8192.md).
NCU_TRAFFIC = {
    'decode1': {'kernel': 'decode_layer_kernel<127>', 'bytes': 14_737_152},
    'decode32': {'kernel': 'decode_layer_kernel<127>', 'bytes': 214_940_160 + 5_720_320},
    'prefill8192': {'kernel': 'mma_kernel<8,1> (gate/up)', 'bytes': 454_199_552 + 119_388_928},
    # profiles/dense_fused_kernel_dense_qkvz1.md, profiles/head_project_kernel_head_vocab1.md
    'dense_qkvz1': {'kernel': 'dense_fused_kernel<16>', 'bytes': 13_006_336 + 0},
    'head_vocab1': {'kernel': 'head_project_kernel<0>', 'bytes': 516_537_856 + 3_437_824},
}
# int8 multiply-accumulates per valid route of one layer: gate/up 1024x2048 + down 2048x512
MACS_PER_ROUTE = 3_145_728

CONFIGS = {
    'decode1': dict(T=1, layers=40, bias=0.0, act_bits=8, shared=True, name='decode B=1, 40-layer stack (configs[1])'),
    'decode32': dict(T=32, layers=40, bias=0.5, act_bits=8, shared=True, name='decode B=32, 40-layer stack (configs[2])'),
    'prefill1120': dict(T=1120, layers=40, bias=0.0, act_bits=4, shared=False, name='prefill chunk 1120 (configs[3])'),
    'prefill8192': dict(T=8192, layers=40, bias=0.0, act_bits=4, shared=False, name='prefill chunk 8192 (configs[3])'),
    # expert-parallel sweep: total tokens fixed, experts sharded over the ranks
    'ep_decode256': dict(T=256, layers=40, bias=0.0, act_bits=8, shared=False, ep=True, exchange='fixed',
                         name='expert-parallel decode B=256, 40 layers, Zipf(1.2) expert skew (configs[4])'),
    'ep_prefill8192': dict(T=8192, layers=4, bias=0.0, act_bits=4, shared=False, ep=True, exchange='compact',
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
    p.add_argument('--config', default='decode1', choices=sorted(CONFIGS))
    p.add_argument('--no-cpu-baseline', action='store_true')
    p.add_argument('--cpu-seconds', type=float, default=12.0)
    p.add_argument('--no-graph', action='store_true', help='time eager launches instead of a captured step')
    p.add_argument('--e2e-overlap', action='store_true',
                   help='e2e with the host copies pipelined: step s+1 copied in and step s-1 copied out on copy '
                        'streams while step s runs (every copy still inside the timed region)')
    p.add_argument('--placement', choices=['balanced', 'contiguous'], default='balanced',
                   help='expert placement of the expert-parallel configs')
    p.add_argument('--combine', choices=['exact', 'partial'], default='exact',
                   help='expert-parallel return: per-slot rows (bit-exact) or per-rank fp32 partial sums')
    p.add_argument('--ep-transport', choices=['nccl', 'p2p'], default='nccl',
                   help='expert-parallel token dispatch and return: NCCL, or stores into the receiving ranks\' '
                        'buffers over NVLink peer memory (exact combine, one chunk)')
    p.add_argument('--ep-chunks', type=int, default=1,
                   help='compact expert-parallel exchange in this many pipelined token chunks (exact combine)')
    p.add_argument('--layers', type=int, default=None,
                   help='override the layer count (small cases for profiler captures)')
    return p.parse_args()


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


def run_ep(args):
    """Expert-parallel step: every rank routes its share of the tokens and runs
    each layer through ornith_b200.ep (NCCL all-to-all dispatch, local experts,
    return of the fp32 per-slot rows, slot-ordered combine)."""
    import datetime
    import torch
    import torch.distributed as dist
    cfg = dict(CONFIGS[args.config])
    if args.layers:
        cfg['layers'] = args.layers
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
    flags = torch.zeros(1, dtype=torch.int32, device=dev)
    for l in range(L):
        native.route_topk(logits[l], w[l], ids[l], flags)

    def step():
        for l in range(L):
            layers[l](x, ids[l], w[l])

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
        graph.replay()
        torch.cuda.synchronize()
        step = graph.replay
    dist.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clk:
        e0.record()
        for _ in range(args.steps):
            step()
        e1.record()
        torch.cuda.synchronize()
    ms = e0.elapsed_time(e1)
    t = torch.tensor([ms], device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX) if world > 1 else None
    ms = float(t.item())
    value = T_total * args.steps / (ms / 1e3)
    result = {
        'metric': METRIC, 'value': round(value, 3), 'unit': 'tokens/s', 'n_gpus': world, 'steps': args.steps,
        'warmup': args.warmup, 'ms_per_step': round(ms / args.steps, 4), 'higher_is_better': True,
        'scaling': 'strong', 'vs_baseline': None, 'dtype': 'int8',
        'data': 'synthetic (seeded random-init weights and logits of the configured shapes)',
        'config': {'workload': cfg['name'], 'tokens_per_step': T_total, 'tokens_per_rank': T, 'layers': L,
                   'experts_per_rank': epr, 'parallelism': f'ep{world}',
                   'placement': ('balanced by routed load of a 4096-token calibration batch'
                                 if args.placement == 'balanced' else 'contiguous ranges'),
                   'combine': ('per-slot fp32 rows, bit-identical to one GPU' if args.combine == 'exact' else
                               'per-rank fp32 partial sums, equal to one GPU within fp32 rounding'),
                   'exchange': ({('fixed', 'nccl'): 'NCCL all_gather of token rows + equal-block all_to_all of '
                                                   'fp32 per-slot rows (no host synchronisation)',
                                 ('compact', 'nccl'): 'NCCL all_to_all_single dispatch + fp32 per-slot return '
                                                      '(variable splits)',
                                 ('fixed', 'p2p'): 'token rows to every rank and owned fp32 slots to their home '
                                                   'as NVLink peer stores (double-buffered, no collective)',
                                 ('compact', 'p2p'): 'NCCL count all_gather, then token rows and fp32 per-slot '
                                                     'rows as NVLink peer stores'}[(cfg['exchange'],
                                                                                    args.ep_transport)]),
                   'chunks': args.ep_chunks if cfg['exchange'] == 'compact' else 1,
                   'transport': 'NVLink peer stores' if args.ep_transport == 'p2p' else 'NCCL'},
        'flags': int(flags.item()), 'clocks': clk.summary(), 'cuda_graph': graph is not None,
    }
    dist.barrier()
    step = None
    graph = None  # a graph holding NCCL calls is released before the process group
    torch.cuda.synchronize()
    for layer in layers:
        layer.close()   # peer-memory buffers, collectively
    dist.destroy_process_group()
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


def run(args):
    import torch
    import torch.distributed as dist
    cfg = dict(CONFIGS[args.config])
    if args.layers:
        cfg['layers'] = args.layers
    world = int(os.environ.get('WORLD_SIZE', '1'))
    rank = int(os.environ.get('RANK', '0'))
    local = int(os.environ.get('LOCAL_RANK', '0'))
    if world > 1:
        torch.cuda.set_device(local)
        dist.init_process_group('nccl', timeout=__import__('datetime').timedelta(seconds=120))
    dev = torch.device('cuda', local)
    torch.cuda.set_device(dev)
    graft.load_package()
    import importlib
    native = importlib.import_module('ornith_b200.native')
    lib = native.lib()
    T, L, bits = cfg['T'], cfg['layers'], cfg['act_bits']
    stack = Stack(torch, cfg, dev, seed=1234 + rank)
    steps_total = args.warmup + args.steps
    # router logits per (step, layer): N(0,1) (+ per-layer per-expert bias)
    bias = (cfg['bias'] * torch.randn((L, 256), device=dev, generator=stack.gen)) if cfg['bias'] else None
    n_logit_sets = steps_total if T <= 64 else 1
    logits = torch.randn((n_logit_sets, L, T, 256), device=dev, generator=stack.gen)
    if bias is not None:
        logits += bias[None, :, None, :]
    x0 = torch.randn((T, 2048), device=dev, generator=stack.gen).to(torch.bfloat16)
    ws = torch.empty(native.workspace_bytes(T), dtype=torch.uint8, device=dev)
    outs = [torch.empty((T, 2048), dtype=torch.bfloat16, device=dev) for _ in range(2)]
    shared_out = torch.empty((T, 2048), dtype=torch.bfloat16, device=dev) if cfg['shared'] else None
    flags = torch.zeros(L, dtype=torch.int32, device=dev)

    def layer_call(l, x, lg, out):
        (gc, gm), (dc, dm), (sgc, sgm), (sdc, sdm), gw = stack.layers[l]
        if cfg['shared']:
            native.routed_from_logits(x, lg, gc, gm, dc, dm, sgc, sgm, sdc, sdm, gw, stack.silu, stack.sigmoid,
                                      ws, out, shared_out, flags[l:l + 1], T, bits)
        else:
            native.routed_from_logits(x, lg, gc, gm, dc, dm, None, None, None, None, None, None, None,
                                      ws, out, None, flags[l:l + 1], T, bits)

    # static inputs: a step reads its token rows and router logits from these
    static_logits = logits[0].clone()
    x_static = x0

    def step_static():
        for l in range(L):
            layer_call(l, x_static, static_logits[l], outs[l % 2])

    def stage_inputs(s):
        static_logits.copy_(logits[s % n_logit_sets], non_blocking=True)

    # algorithmic bytes per step: (distinct experts + 1) * EXPERT_BYTES per layer + activations
    ids = torch.topk(logits, 8, dim=-1).indices  # [sets, L, T, 8]
    distinct = []
    for s in range(n_logit_sets):
        d = 0
        for l in range(L):
            d += int(torch.unique(ids[s, l]).numel()) + (1 if cfg['shared'] else 0)
        distinct.append(d)
    act_bytes = L * (2 * T * 4096 + T * 1024)

    def step_bytes(s):
        return distinct[s % n_logit_sets] * EXPERT_BYTES + act_bytes

    for s in range(args.warmup):
        stage_inputs(s)
        step_static()
    torch.cuda.synchronize()

    # Decode steps are captured once as a CUDA graph and replayed (the way a
    # serving engine runs decode); the layer calls inside are the same C-ABI
    # launches.  Each replay is preceded by a device copy of that step's logits.
    graph, graph_error = None, None
    layer_graphs = []
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
            for l in range(L):
                g1 = torch.cuda.CUDAGraph()
                with torch.cuda.graph(g1):
                    layer_call(l, x_static, static_logits[l], outs[l % 2])
                layer_graphs.append(g1)
            torch.cuda.synchronize()
        except Exception as exc:  # capture unsupported: time the eager launches instead
            graph, layer_graphs, graph_error = None, [], repr(exc)[:200]
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
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    launches0 = lib.ornith_moe_b200_kernel_launches()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clk:
        start.record()
        for s in range(args.warmup, steps_total):
            run_step(s)
        end.record()
        torch.cuda.synchronize()
    # kernels of this library enqueued per step (graph replays re-run the captured launches)
    launches = (lib.ornith_moe_b200_kernel_launches() - launches0) if graph is None else \
        launches_per_step(lib, step_static) * args.steps
    ms = start.elapsed_time(end)
    if world > 1:
        t = torch.tensor([ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    ms_step = ms / args.steps
    value = world * T * args.steps / (ms / 1e3)
    bytes_timed = sum(step_bytes(s) for s in range(args.warmup, steps_total)) / args.steps

    # per-layer timing: each layer call (routing + fused layer kernel) replayed
    # as its own graph between events, layers in sequence so that weights stream
    # from HBM as in a step
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(L)]
    per_layer = []
    for rep in range(3):
        stage_inputs(args.warmup + rep)
        for l in range(L):
            ev[l][0].record()
            if layer_graphs:
                layer_graphs[l].replay()
            else:
                layer_call(l, x_static, static_logits[l], outs[l % 2])
            ev[l][1].record()
        torch.cuda.synchronize()
        per_layer += [a.elapsed_time(b) for a, b in ev]
    layer_ms = statistics.mean(per_layer)
    layer_bytes = bytes_timed / L
    peaks = json.loads((ROOT / 'MEASURED_PEAKS.json').read_text()) if (ROOT / 'MEASURED_PEAKS.json').exists() else {}
    peak = peaks.get('hbm_gbs', 6650.0)
    achieved = layer_bytes / (layer_ms * 1e-3) / 1e9
    traffic = NCU_TRAFFIC.get(args.config)
    hbm_roofline = {'bound': 'hbm', 'achieved': round(achieved, 1), 'peak': peak, 'unit': 'GB/s',
                    'frac': round(achieved / peak, 4), 'traffic': traffic['bytes'] if traffic else None,
                    'kernel': 'one routed_from_logits layer call (all its kernels)',
                    'algorithmic_bytes_per_launch': int(layer_bytes), 'launch_ms': round(layer_ms, 5),
                    'peak_source': 'MEASURED_PEAKS.json hbm_gbs (of measured)' if peaks else 'fallback 6650 GB/s'}
    if T > 64:
        # prefill: the grouped int8 GEMMs bound the layer; int8 dense tensor rate is
        # twice bf16 on B200, and only the bf16 rate is measured on this pool
        ops = 2.0 * T * 8 * MACS_PER_ROUTE
        bf16 = peaks.get('bf16_tflops', 1590.0)
        tops = ops / (layer_ms * 1e-3) / 1e12
        roofline = {'bound': 'tensor', 'achieved': round(tops, 1), 'peak': round(2 * bf16, 1), 'unit': 'TOP/s',
                    'frac': round(tops / (2 * bf16), 4), 'traffic': traffic['bytes'] if traffic else None,
                    'kernel': 'one routed_from_logits layer call (all its kernels)',
                    'algorithmic_ops_per_launch': ops, 'launch_ms': round(layer_ms, 5),
                    'peak_source': ('2 x MEASURED_PEAKS.json bf16_tflops (of measured; int8 = 2 x bf16 dense)'
                                    if peaks else '2 x fallback 1590 TFLOP/s'),
                    'frac_of_bf16_peak': round(tops / bf16, 4),
                    'hbm': hbm_roofline}
    else:
        roofline = hbm_roofline
    if traffic:
        roofline['traffic_kernel'] = traffic['kernel']

    # end to end through the public operator: pinned host inputs copied in, the
    # step (graph of the operator's launches) run, the last output copied out
    pin_x = x0.cpu().pin_memory()
    pin_logits = logits[: min(n_logit_sets, 4)].cpu().pin_memory()
    pin_out = torch.empty((T, 2048), dtype=torch.bfloat16).pin_memory()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    replay = graph.replay if graph is not None else step_static
    if args.e2e_overlap:
        e2e_pipelined(torch, args.steps, pin_x, pin_logits, x_static, static_logits, outs[(L - 1) % 2], pin_out,
                      replay, e0, e1)
    else:
        e0.record()
        for s in range(args.steps):
            x_static.copy_(pin_x, non_blocking=True)
            static_logits.copy_(pin_logits[s % pin_logits.shape[0]], non_blocking=True)
            replay()
            pin_out.copy_(outs[(L - 1) % 2], non_blocking=True)
        e1.record()
    torch.cuda.synchronize()
    e2e_ms = e0.elapsed_time(e1)
    if world > 1:
        t = torch.tensor([e2e_ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_ms = float(t.item())
    e2e_value = world * T * args.steps / (e2e_ms / 1e3)
    flag_any = int(flags.max().item())

    result = {
        'metric': METRIC, 'value': round(value, 3), 'unit': 'tokens/s', 'n_gpus': world,
        'steps': args.steps, 'warmup': args.warmup, 'ms_per_step': round(ms_step, 4),
        'higher_is_better': True, 'scaling': 'weak', 'vs_baseline': None, 'dtype': 'int8',
        'data': 'synthetic (seeded random-init weights and logits of the configured shapes)',
        'config': {'workload': cfg['name'], 'tokens_per_step': T, 'layers': L, 'experts': 256, 'top_k': 8,
                   'hidden': 2048, 'intermediate': 512, 'shared_expert': cfg['shared'],
                   'weights': 'affine-u4 G256 (scale, offset=-8*scale), N32 storage',
                   'activations': f'A{bits} per 256-group after H128', 'arith': 'u4 x s8 -> int32 dot, fp32 epilogue',
                   'parallelism': f'replicas x{world}' if world > 1 else 'single GPU',
                   'l2': f'inputs larger than L2: {bytes_timed / 1e6:.0f} MB of weights read per step'},
        'e2e': {'value': round(e2e_value, 3), 'unit': 'tokens/s', 'h2d_bytes_per_step': T * 4096 + L * T * 1024,
                'd2h_bytes_per_step': T * 4096,
                'copies': ('pipelined on copy streams, inside the timed region' if args.e2e_overlap
                           else 'in line with the steps')},
        'gpu_launches': int(launches),
        'roofline': roofline,
        'step_roofline_frac': round(bytes_timed / (ms_step * 1e-3) / 1e9 / peak, 4),
        'flags_max': flag_any,
        'cuda_graph': graph is not None,
        'clocks': clk.summary(),
    }
    if graph_error:
        result['cuda_graph_error'] = graph_error
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        result['cpu_baseline'] = cpu_baseline(cfg, args.cpu_seconds)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    if rank == 0:
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

    def one():
        for _ in range(layers_per_step):
            x = S.make_tokens(rng, T)
            w, ids = O.route_topk(rng.standard_normal((T, 256)).astype(np.float32))
            if cfg['shared']:
                logit = S.f32_to_bf16_bits(rng.standard_normal(T).astype(np.float32))
                O.ref_routed_shared(x, w, ids, layer.gate_codes, layer.gate_meta, layer.down_codes, layer.down_meta,
                                    layer.sgate_codes, layer.sgate_meta, layer.sdown_codes, layer.sdown_meta, logit,
                                    tab['silu_fp32'], tab['sigmoid_bf16'])
            else:
                entry = 'ornith_routed_direct_launch' if cfg['act_bits'] == 8 else 'ornith_routed_direct_launch_a4'
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
        run(a)
