"""GPU: expert parallelism over NCCL (needs 2+ GPUs; skipped otherwise).

Two ranks each hold half of the experts and their own tokens; the expert-
parallel result must equal the single-GPU layer bit for bit.  NVLS is off as
the pool requires for multi-rank GPU tests."""
import os
import socket
import sys
from pathlib import Path

import pytest
import torch

pytestmark = pytest.mark.gpu
ROOT = Path(__file__).resolve().parents[1]


def _port():
    with socket.socket() as s:
        s.bind(('127.0.0.1', 0))
        return s.getsockname()[1]


def _bank(gen, experts, N, K, dev):
    codes = torch.randint(-2 ** 31, 2 ** 31 - 1, (experts, N // 32, K // 256, 32, 32), dtype=torch.int32,
                          device=dev, generator=gen).view(torch.uint32)
    z = torch.randn((experts, N // 32, K // 256, 32), device=dev, generator=gen)
    scale = (0.01 * z.abs()).to(torch.float16).clamp_min(2 ** -14)
    offset = (scale.float() * -8.0).to(torch.float16)
    meta = (scale.view(torch.int16).to(torch.int32) & 0xFFFF) | (offset.view(torch.int16).to(torch.int32) << 16)
    return codes, meta.view(torch.uint32)


CASES = [  # (exchange, balanced placement, combine, further ExpertParallelMoE options)
    ('compact', False, 'exact', {}), ('compact', True, 'exact', {}), ('fixed', False, 'exact', {}),
    ('fixed', True, 'exact', {}), ('compact', True, 'partial', {}), ('fixed', True, 'partial', {}),
    ('compact', True, 'exact', {'chunks': 3}),
    ('compact', False, 'exact', {'transport': 'p2p'}), ('compact', True, 'exact', {'transport': 'p2p'}),
    ('fixed', False, 'exact', {'transport': 'p2p'}), ('fixed', True, 'exact', {'transport': 'p2p'}),
    ('fixed', True, 'partial', {'transport': 'p2p'}),   # bit-identical to the NCCL form of the same mode
]


def _close(out, ref):
    """Rank-partial combine: a different association of the same fp32 sum, so
    elements with cancellation may differ by more than a bf16 step; the check is
    the north-star bound (relative L2 <= 1e-3, max-abs <= 2e-2)."""
    a = out.float()
    b = ref.float()
    rel_l2 = float((a - b).norm() / b.norm().clamp_min(1e-30))
    return rel_l2 <= 1e-3 and float((a - b).abs().max()) <= 2e-2


def _worker(rank, world, port, T, q):
    try:
        import datetime
        import torch.distributed as dist
        os.environ.update(MASTER_ADDR='127.0.0.1', MASTER_PORT=str(port), NCCL_NVLS_ENABLE='0')
        torch.cuda.set_device(rank)
        dev = torch.device('cuda', rank)
        dist.init_process_group('nccl', rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
        sys.path.insert(0, str(ROOT))
        import __graft_entry__ as g
        g.load_package()
        from ornith_b200 import ep, native
        gen = torch.Generator(device=dev)
        gen.manual_seed(77)                      # identical full banks on every rank
        gc, gm = _bank(gen, 256, 1024, 2048, dev)
        dc, dm = _bank(gen, 256, 2048, 512, dev)
        tok = torch.Generator(device=dev)
        tok.manual_seed(1000 + rank)             # each rank's own tokens
        x = torch.randn((T, 2048), device=dev, generator=tok).to(torch.bfloat16)
        logits = torch.randn((T, 256), device=dev, generator=tok)
        w = torch.empty((T, 8), dtype=torch.float32, device=dev)
        ids = torch.empty((T, 8), dtype=torch.int32, device=dev)
        flags = torch.zeros(1, dtype=torch.int32, device=dev)
        native.route_topk(logits, w, ids, flags)
        # single-GPU reference on this rank
        ws = torch.empty(native.get_layout(T).workspace_bytes, dtype=torch.uint8, device=dev)
        ref = torch.empty((T, 2048), dtype=torch.bfloat16, device=dev)
        native.check(native.lib().ornith_routed_direct_launch(
            *[native.ptr(t) for t in (x, w, ids, gc, gm, dc, dm, ws)], ws.numel(), native.ptr(ref),
            native.ptr(flags), T, T, native.stream(x)), 'reference layer')
        results = []
        partial_outputs = {}   # (mode, balanced) -> output of the NCCL rank-partial form
        for mode, balanced, combine, options in CASES:
            if balanced:  # any placement must give the same result; use a skewed-load one
                placement = ep.balanced_placement(torch.arange(256, dtype=torch.float64).flip(0) ** 2, world, dev)
            else:
                placement = ep.contiguous_placement(world, dev)
            sl = torch.tensor(placement.experts_of(rank), device=dev)

            def pick(bank):  # this rank's experts, in the placement's bank order
                return bank.view(torch.int32)[sl].contiguous().view(torch.uint32)

            layer = ep.ExpertParallelMoE(None, world, (pick(gc), pick(gm), pick(dc), pick(dm)), capacity=T * world,
                                         exchange=mode, placement=placement, combine=combine, **options)
            ok = True
            for _ in range(3):   # three calls: both buffer sets of the fixed peer exchange, then the first again
                out = layer(x, ids, w)
                torch.cuda.synchronize()
                ok = ok and (bool(torch.equal(out.view(torch.int16), ref.view(torch.int16))) if combine == 'exact'
                             else _close(out, ref))
                if combine == 'partial' and mode == 'fixed':
                    if options.get('transport') == 'p2p':   # the same sums, added in the same rank order
                        nccl = partial_outputs.get((mode, balanced))
                        ok = ok and nccl is not None and bool(torch.equal(out.view(torch.int16), nccl.view(torch.int16)))
                    else:
                        partial_outputs[(mode, balanced)] = out.clone()
            results.append(((mode, balanced, combine, tuple(options.items())), ok, int(layer.flags.item())))
            layer.close()
            dist.barrier()
        q.put((rank, results, int(flags.item()), ''))
        dist.barrier()
        dist.destroy_process_group()
    except Exception as exc:
        q.put((rank, None, -1, repr(exc)))


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason='needs 2 GPUs')
@pytest.mark.parametrize('T', [5, 96])
def test_expert_parallel_matches_single_gpu(T):
    """Every exchange mode and placement: bit-identical to the single-GPU layer
    with the exact combine, within fp32 rounding with the rank-partial one."""
    import torch.multiprocessing as mp
    ctx = mp.get_context('spawn')
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, T, q)) for r in range(2)]
    for p in procs:
        p.start()
    results = [q.get(timeout=300) for _ in range(2)]
    for p in procs:
        p.join(timeout=60)
    for rank, cases, flags, err in results:
        assert cases is not None and flags == 0, (rank, flags, err)
        for case, ok, case_flags in cases:
            assert ok and case_flags == 0, (rank, case, case_flags)


def _timeout_worker(rank, world, port, q):
    """Fixed exchange over peer memory with a 50 ms wait limit; rank 1 sleeps
    on the host before its layer call (no kernel of it in flight), so rank 0's
    wait for rank 1's token rows runs out.  Rank 0 carries on and its flag-64
    bit travels with its returned rows, so rank 1 reports flag 64 as well."""
    try:
        import datetime
        import time
        import torch.distributed as dist
        os.environ.update(MASTER_ADDR='127.0.0.1', MASTER_PORT=str(port), NCCL_NVLS_ENABLE='0')
        torch.cuda.set_device(rank)
        dev = torch.device('cuda', rank)
        dist.init_process_group('nccl', rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
        sys.path.insert(0, str(ROOT))
        import __graft_entry__ as g
        g.load_package()
        from ornith_b200 import ep, native
        native.set_peer_wait_limit_ns(50_000_000)
        T = 4
        gen = torch.Generator(device=dev)
        gen.manual_seed(5)
        gc, gm = _bank(gen, 256 // world, 1024, 2048, dev)
        dc, dm = _bank(gen, 256 // world, 2048, 512, dev)
        x = torch.randn((T, 2048), device=dev, generator=gen).to(torch.bfloat16)
        logits = torch.randn((T, 256), device=dev, generator=gen)
        w = torch.empty((T, 8), dtype=torch.float32, device=dev)
        ids = torch.empty((T, 8), dtype=torch.int32, device=dev)
        rflags = torch.zeros(1, dtype=torch.int32, device=dev)
        native.route_topk(logits, w, ids, rflags)
        layer = ep.ExpertParallelMoE(None, world, (gc, gm, dc, dm), capacity=T * world, exchange='fixed',
                                     transport='p2p')
        layer.peer_fixed = ep.PeerFixedExchange(None, world, rank, T, dev)   # made collectively, before the sleep
        torch.cuda.synchronize()
        dist.barrier()
        if rank == 1:
            time.sleep(0.5)
        layer(x, ids, w)
        torch.cuda.synchronize()
        flags = int(layer.flags.item())
        dist.barrier()
        layer.close()
        q.put((rank, flags, ''))
        dist.barrier()
        dist.destroy_process_group()
    except Exception as exc:
        q.put((rank, -1, repr(exc)))


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason='needs 2 GPUs')
def test_fixed_peer_timeout_reaches_every_rank():
    import torch.multiprocessing as mp
    ctx = mp.get_context('spawn')
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_timeout_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    results = dict((rank, (flags, err)) for rank, flags, err in (q.get(timeout=300) for _ in range(2)))
    for p in procs:
        p.join(timeout=60)
    for rank in (0, 1):
        flags, err = results[rank]
        assert flags >= 0, err
        assert flags & 64, (rank, flags)
