"""Seeded synthetic inputs for the Ornith routed-MoE layer.

The shapes and value distributions are those of the benchmark configurations
of the reference's MoE layer (Ornith 1.5 35B-A3B: 256 routed experts, top-8,
hidden 2048, intermediate 512, one shared expert):

  * activations x ~ N(0, 1), stored as bf16;
  * router weight ~ N(0, 0.02) bf16 [256, 2048];
  * expert codes uniform over the u4 range [0, 15];
  * per-(column, 256-group) fp16 scale = 0.01*|N(0,1)| floored at 2^-14 (the
    loader's admission floor, plugin-site/ornith_g256/loader.py:35-36) and
    fp16 offset = -8*scale, i.e. symmetric int4 expressed in the reference's
    affine-u4 G256 format (weight = scale*code + offset);
  * shared-expert gate weight ~ N(0, 0.02) bf16 [2048].

Host generation uses numpy's PCG64 `default_rng(seed)` with the fixed draw
order documented on each function.  Device generation (the 40-layer benchmark
stores, 16.6 GB) uses torch's CUDA generator; those weights are parity-checked
by copying a layer back to the host.

Banks use the N32 storage of the reference's production library:
codes uint32 [E, N/32, K/256, 32, 32] and metadata uint32 [E, N/32, K/256, 32].
"""
from dataclasses import dataclass

import numpy as np

E, TOP, H, I, G = 256, 8, 2048, 512, 256
GATE_N, GATE_K = 2 * I, H
DOWN_N, DOWN_K = H, I


def f32_to_bf16_bits(a):
    """Round fp32 to bf16 (nearest even) and return the raw uint16 bits."""
    b = np.ascontiguousarray(a, dtype=np.float32).view(np.uint32)
    nan = (b & 0x7FFFFFFF) > 0x7F800000
    r = ((b + 0x7FFF + ((b >> 16) & 1)) >> 16).astype(np.uint16)
    return np.where(nan, ((b >> 16) | 0x40).astype(np.uint16), r)


def bf16_bits_to_f32(b):
    return (np.ascontiguousarray(b, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def make_bank(rng, experts, N, K):
    """One packed bank.  Draw order: codes (uint32 words), then scales (normals)."""
    codes = rng.integers(0, 2 ** 32, size=(experts, N // 32, K // G, 32, 32), dtype=np.uint32)
    z = rng.standard_normal((experts, N // 32, K // G, 32), dtype=np.float32)
    scale = np.maximum((np.float32(0.01) * np.abs(z)).astype(np.float16), np.float16(2 ** -14))
    offset = (scale.astype(np.float32) * np.float32(-8.0)).astype(np.float16)
    meta = scale.view(np.uint16).astype(np.uint32) | (offset.view(np.uint16).astype(np.uint32) << 16)
    return codes, meta


def make_dense_bank(rng, N, K):
    """One dense G256 bank in the reference's N16 storage (dense_g256_api.h:27-29):
    codes uint32 [N/16, K/256, 32, 16], metadata uint32 [N/16, K/256, 16], with
    the value distribution of make_bank.  Draw order: codes, then scales."""
    codes = rng.integers(0, 2 ** 32, size=(N // 16, K // G, 32, 16), dtype=np.uint32)
    z = rng.standard_normal((N // 16, K // G, 16), dtype=np.float32)
    scale = np.maximum((np.float32(0.01) * np.abs(z)).astype(np.float16), np.float16(2 ** -14))
    offset = (scale.astype(np.float32) * np.float32(-8.0)).astype(np.float16)
    meta = scale.view(np.uint16).astype(np.uint32) | (offset.view(np.uint16).astype(np.uint32) << 16)
    return codes, meta


def make_head_bank(rng, N, K=2048):
    """An int8 head bank in the reference's physical layout (head_i8_tile_api.h:1-2,
    :21-26): words uint32 [N/16, K/16, 4, 16], four signed codes per word
    (lowest k first) uniform over [-127, 127], and fp16 scales [N, 16] (one per
    128-group) = 0.01*|N(0,1)| floored at 2^-14, as uint16 bits.
    Draw order: codes, then scales."""
    codes = rng.integers(-127, 128, size=(N // 16, K // 16, 4, 16, 4), dtype=np.int8)
    words = np.ascontiguousarray(codes).view(np.uint32).reshape(N // 16, K // 16, 4, 16)
    z = rng.standard_normal((N, K // 128), dtype=np.float32)
    scales = np.maximum((np.float32(0.01) * np.abs(z)).astype(np.float16), np.float16(2 ** -14))
    return words, scales.view(np.uint16)


def make_rows(rng, M, K):
    """bf16 bits of x ~ N(0,1) [M, K]."""
    return f32_to_bf16_bits(rng.standard_normal((M, K), dtype=np.float32))


@dataclass
class LayerWeights:
    gate_codes: np.ndarray   # [E, 32, 8, 32, 32]
    gate_meta: np.ndarray    # [E, 32, 8, 32]
    down_codes: np.ndarray   # [E, 64, 2, 32, 32]
    down_meta: np.ndarray    # [E, 64, 2, 32]
    sgate_codes: np.ndarray  # [1, 32, 8, 32, 32]
    sgate_meta: np.ndarray
    sdown_codes: np.ndarray  # [1, 64, 2, 32, 32]
    sdown_meta: np.ndarray
    shared_gate_w: np.ndarray  # bf16 bits [2048]


def make_layer(rng, experts=E):
    """Draw order: routed gate/up bank, routed down bank, shared gate/up bank,
    shared down bank, shared gate weight."""
    gc, gm = make_bank(rng, experts, GATE_N, GATE_K)
    dc, dm = make_bank(rng, experts, DOWN_N, DOWN_K)
    sgc, sgm = make_bank(rng, 1, GATE_N, GATE_K)
    sdc, sdm = make_bank(rng, 1, DOWN_N, DOWN_K)
    sg = f32_to_bf16_bits(np.float32(0.02) * rng.standard_normal(H, dtype=np.float32))
    return LayerWeights(gc, gm, dc, dm, sgc, sgm, sdc, sdm, sg)


def make_tokens(rng, T):
    """bf16 bits of x ~ N(0,1) [T, 2048]."""
    return f32_to_bf16_bits(rng.standard_normal((T, H), dtype=np.float32))


def make_router(rng):
    """bf16 bits of the router weight ~ N(0, 0.02) [256, 2048]."""
    return f32_to_bf16_bits(np.float32(0.02) * rng.standard_normal((E, H), dtype=np.float32))


def config1(seed=0):
    """Reference CPU-runnable case: T=4, router linear included.  Draw order:
    x, router weight, layer banks (make_layer)."""
    rng = np.random.default_rng(seed)
    x = make_tokens(rng, 4)
    router = make_router(rng)
    layer = make_layer(rng)
    return x, router, layer


def random_routes(rng, T, pad_fraction=0.0, experts=E, bias=None):
    """Random top-8 routes: distinct experts per token (optionally drawn with a
    per-expert logit bias), softmax-like positive weights, and optional -1
    padding ids.  Draw order: logits, padding mask."""
    logits = rng.standard_normal((T, experts), dtype=np.float32)
    if bias is not None:
        logits = logits + bias[None, :experts].astype(np.float32)
    order = np.argsort(-logits, axis=1, kind='stable')[:, :TOP]
    top = np.take_along_axis(logits, order, axis=1)
    ex = np.exp(top - top[:, :1])
    w = (ex / ex.sum(axis=1, keepdims=True)).astype(np.float32)
    ids = order.astype(np.int32)
    if pad_fraction > 0:
        mask = rng.random((T, TOP)) < pad_fraction
        ids = np.where(mask, -1, ids).astype(np.int32)
    return np.ascontiguousarray(w), np.ascontiguousarray(ids)


def hot_routes(rng, T, counts, pad_fraction=0.0, experts=E):
    """Routes in which chosen experts receive exactly the given numbers of
    routes (`counts`: {expert: routes}), so that an expert's rows span several
    128-row tiles of the grouped projection, end one short of, exactly at or
    one past a tile, or take more routes than there are tokens (the same
    expert in several slots of one token, which the reference treats as
    independent routes).  The other slots get random top-8 routes over the
    remaining experts.  Draw order: random_routes (logits, padding mask), then
    one permutation of the T*8 (token, slot) positions, whose leading runs go
    to the hot experts in the order of `counts`."""
    total = sum(counts.values())
    if total > T * TOP:
        raise ValueError(f'{total} hot routes do not fit in {T} tokens x {TOP} slots')
    bias = np.zeros(experts, np.float32)
    bias[list(counts)] = -np.inf          # hot experts only where placed below
    w, ids = random_routes(rng, T, pad_fraction=pad_fraction, experts=experts, bias=bias)
    flat = ids.reshape(-1)
    pos = rng.permutation(T * TOP)
    at = 0
    for e, c in counts.items():
        flat[pos[at:at + c]] = e
        at += c
    return w, np.ascontiguousarray(flat.reshape(T, TOP))


def zipf_bias(rng, experts=E, s=1.2):
    """Per-expert logit bias giving a Zipf(s) load skew: a seeded permutation
    ranks the experts, bias_e = -s*ln(rank_e)."""
    perm = rng.permutation(experts)
    rank = np.empty(experts, np.float64)
    rank[perm] = np.arange(1, experts + 1)
    return (-s * np.log(rank)).astype(np.float32)
