"""GPU: the entry point for callers that cannot allocate device memory.

ornith_routed_direct_launch_noalloc takes inputs and outputs only and keeps its
scratch in a fixed array inside the library, for callers such as framework
plugins that are handed tensors but no allocator.  This file is collected
last so that a stop-at-first-failure run has already run every other test,
and it builds its own inputs so that it also passes alone in a fresh process.
"""
import ctypes as C

import pytest
import torch

pytestmark = pytest.mark.gpu
DEV = torch.device('cuda:0')


def _bank(gen, experts, N, K):
    codes = torch.randint(-2 ** 31, 2 ** 31 - 1, (experts, N // 32, K // 256, 32, 32), dtype=torch.int32,
                          device=DEV, generator=gen).view(torch.uint32)
    z = torch.randn((experts, N // 32, K // 256, 32), device=DEV, generator=gen)
    scale = (0.01 * z.abs()).to(torch.float16).clamp_min(2 ** -14)
    offset = (scale.float() * -8.0).to(torch.float16)
    meta = (scale.view(torch.int16).to(torch.int32) & 0xFFFF) | (offset.view(torch.int16).to(torch.int32) << 16)
    return codes, meta.view(torch.uint32)


def _case(gen, T):
    x = torch.randn((T, 2048), device=DEV, generator=gen).to(torch.bfloat16)
    logits = torch.randn((T, 256), device=DEV, generator=gen)
    ids = torch.topk(logits, 8, dim=1).indices.to(torch.int32).contiguous()
    ids[0, 7] = -1
    w = torch.softmax(torch.randn((T, 8), device=DEV, generator=gen), dim=1).contiguous()
    return x, w, ids


def test_noalloc_entry_matches_workspace_entry(native):
    lib = native.lib()
    gen = torch.Generator(device=DEV)
    gen.manual_seed(2024)
    gc, gm = _bank(gen, 256, 1024, 2048)
    dc, dm = _bank(gen, 256, 2048, 512)
    banks = [native.ptr(t) for t in (gc, gm, dc, dm)]
    stream = native.stream(gc)
    for T in (3, 8):  # two calls in a row share the library's scratch array
        x, w, ids = _case(gen, T)
        ws = torch.empty(native.get_layout(T).workspace_bytes, dtype=torch.uint8, device=DEV)
        ref = torch.empty((T, 2048), dtype=torch.bfloat16, device=DEV)
        ref_flags = torch.zeros(1, dtype=torch.int32, device=DEV)
        assert lib.ornith_routed_direct_launch(native.ptr(x), native.ptr(w), native.ptr(ids), *banks,
                                               native.ptr(ws), ws.numel(), native.ptr(ref), native.ptr(ref_flags),
                                               T, T, stream) == 0
        out = torch.full((T, 2048), -1, dtype=torch.int16, device=DEV).view(torch.bfloat16)
        flags = torch.zeros(1, dtype=torch.int32, device=DEV)
        assert lib.ornith_routed_direct_launch_noalloc(native.ptr(x), native.ptr(w), native.ptr(ids), *banks,
                                                       native.ptr(out), native.ptr(flags), T, stream) == 0
        torch.cuda.synchronize()
        # same kernels and arithmetic: exact equality, like every parity test here
        assert torch.equal(out.view(torch.int16), ref.view(torch.int16))
        assert int(flags.item()) == int(ref_flags.item()) == 0


def test_noalloc_entry_rejects_too_many_tokens(native):
    lib = native.lib()
    fake = C.c_void_p(1 << 20)
    assert lib.ornith_routed_direct_launch_noalloc(*([fake] * 9), 9, None) == 1  # cudaErrorInvalidValue
