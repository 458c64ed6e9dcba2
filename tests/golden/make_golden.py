"""Regenerate the committed golden fixtures (run in the build container only).

  shared_math_tables.npz
      The reference's pinned SiLU fp32 / sigmoid bf16 tables for every bf16
      bit pattern (native/shared_math_reference.safetensors), copied after
      checking the sha256 recorded in native/shared_math_reference.json.
  dense_reference_outputs.npz
      Outputs of the reference's own dense library (kernels/dense_n32/,
      compiled for the CPU) on the seeded DENSE_CASES: the A8 projection from
      N16 banks (every geometry), from the N32 shadow, and the bf16 prefill
      preparation.  Inputs are regenerated from their seeds, as below.
  head_reference_outputs.npz
      Outputs of the reference's own W8 head library (kernels/head/, compiled
      for the CPU) on the seeded HEAD_CASES: logits, fp32 projections, raw
      group dots and flags.
  routed_reference_digests.npz
      sha256 digests of the reference routed library's outputs (and its flags)
      on the larger DIGEST_CASES (T = 32, 64, 1120), whose outputs are too big
      to commit.
  routed_reference_outputs.npz
      Outputs of the reference's own routed library (kernels/routed_storage/,
      compiled for the CPU by oracle/build_ref.py) on seeded synthetic cases.
      Inputs are not stored: each case is regenerated from its seed by the
      synthetic generator, and the sha256 of the regenerated inputs is stored
      so that generator drift is detected.

Usage: python tests/golden/make_golden.py [--reference DIR] [--only dense|head|digests]
(default reference: ORNITH_REFERENCE, else BASELINE.json's reference_path)
"""
import argparse
import hashlib
import importlib.util
import json
import sys
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(ROOT))
from oracle import oracle as O  # noqa: E402

OUT = Path(__file__).resolve().parent


def _synthetic():
    spec = importlib.util.spec_from_file_location('ornith_synthetic', ROOT / 'ornith-ciru-halo-agent_b200' / 'synthetic.py')
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


# (name, layer seed, case seed, T, pad fraction, hot experts with +6 bias, entry, special)
CASES = [
    ('t1_a8', 1, 11, 1, 0.0, 0, 'ornith_routed_direct_launch', ''),
    ('t3_a8_pad', 1, 12, 3, 0.2, 0, 'ornith_routed_direct_launch', ''),
    ('t8_a4', 1, 13, 8, 0.1, 0, 'ornith_routed_direct_launch_a4', ''),
    ('t16_a8', 1, 14, 16, 0.1, 0, 'ornith_routed_direct_launch', ''),
    ('t17_a8_grouped', 1, 15, 17, 0.05, 12, 'ornith_routed_direct_launch', ''),
    ('t33_a4_grouped', 1, 16, 33, 0.05, 12, 'ornith_routed_direct_launch_a4', ''),
    ('t65_a4prefill', 1, 17, 65, 0.05, 24, 'ornith_routed_direct_launch_a4_prefill', ''),
    ('t5_a8_edges', 1, 18, 5, 0.0, 0, 'ornith_routed_direct_launch', 'edges'),
]


def make_case(S, layer, case_seed, T, pad, hot, special):
    rng = np.random.default_rng(case_seed)
    x = S.make_tokens(rng, T)
    bias = None
    if hot:
        bias = np.zeros(S.E, np.float32)
        bias[:hot] = 6.0
    w, ids = S.random_routes(rng, T, pad_fraction=pad, bias=bias)
    if special == 'edges':
        # token 0: all-zero row (zero groups -> scale 1); token 1: one huge
        # element saturating its group; token 2: all ids padded (-1) -> zero
        # output; token 3: one invalid id 300 (flag 4) and one -5 (flag 4);
        # token 4: a NaN input element (flags 1/2 and propagation).
        x[0, :] = 0
        x[1, 7] = S.f32_to_bf16_bits(np.array([3.0e4], np.float32))[0]
        ids[2, :] = -1
        ids[3, 2] = 300
        ids[3, 5] = -5
        x[4, 100] = 0x7FC0
    return x, w, ids


# (name, seed, M, N, K, entry, geometry, special); entry 'n16', 'n32' or 'prepare'
DENSE_CASES = [
    ('d_m1_n32', 31, 1, 64, 2048, 'n32', 2, ''),
    ('d_m1_n16', 32, 1, 96, 2048, 'n16', 2, ''),
    ('d_m3_g1_n48', 33, 3, 48, 512, 'n16', 1, ''),
    ('d_m16_g0', 34, 16, 128, 768, 'n16', 0, ''),
    ('d_m37_g0', 35, 37, 64, 256, 'n16', 0, ''),
    ('d_m7_n32_k8192', 36, 7, 32, 8192, 'n32', 2, ''),
    ('d_m5_edges', 37, 5, 64, 512, 'n16', 2, 'edges'),
    ('d_prep_m5', 38, 5, 48, 512, 'prepare', 0, 'edges'),
]


# (name, seed, M, N, geometry, special)
HEAD_CASES = [
    ('h_m1_n1024', 41, 1, 1024, 2, ''),
    ('h_m3_n256_compact', 42, 3, 256, 1, ''),
    ('h_m16_n1024_wmma', 43, 16, 1024, 0, ''),
    ('h_m64_n256_shared64', 44, 64, 256, 2, ''),
    ('h_m5_edges', 45, 5, 256, 2, 'edges'),
]


def make_head_case(S, seed, M, N, special):
    """Rows and an int8 head bank.  Draw order: bank (make_head_bank), then rows."""
    rng = np.random.default_rng(seed)
    words, scales = S.make_head_bank(rng, N)
    x = S.make_rows(rng, M, 2048)
    if special == 'edges':
        # row 0 all zero; row 1 a NaN element; row 2 a saturating 3e4; row 3 at
        # the bf16 maximum (the Hadamard overflows: flags 1 and 2); column 5
        # has an infinite scale in group 3 (flags 4 and 8)
        x[0, :] = 0
        x[1, 300] = 0x7FC0
        x[2, 1000] = S.f32_to_bf16_bits(np.array([3.0e4], np.float32))[0]
        x[3, :] = 0x7F7F
        scales = scales.copy()
        scales[5, 3] = 0x7C00
    return x, words, scales


def make_dense_case(S, seed, M, N, K, special):
    """Rows and an N16 bank.  Draw order: bank (make_dense_bank), then rows."""
    rng = np.random.default_rng(seed)
    codes, meta = S.make_dense_bank(rng, N, K)
    x = S.make_rows(rng, M, K)
    if special == 'edges':
        # row 0 all zero (zero groups -> scale 1); row 1 a NaN element; row 2
        # an element of 3e4 saturating its group; row 3 every element at the
        # bf16 maximum (the Hadamard overflows: flags 1 and 2); column 3 of
        # tile 1 has an infinite offset in group 0 (flags 4 and 8)
        x[0, :] = 0
        x[1, 5] = 0x7FC0
        x[2, 7] = S.f32_to_bf16_bits(np.array([3.0e4], np.float32))[0]
        x[3, :] = 0x7F7F
        meta = meta.copy()
        meta[1, 0, 3] = (meta[1, 0, 3] & 0xFFFF) | (0x7C00 << 16)
    return x, codes, meta


def digest(*arrays):
    h = hashlib.sha256()
    for a in arrays:
        h.update(np.ascontiguousarray(a).tobytes())
    return h.hexdigest()


def main():
    parser = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    parser.add_argument('--reference', default=None,
                        help='reference checkout (default: ORNITH_REFERENCE, else BASELINE.json reference_path)')
    parser.add_argument('--only', choices=['dense', 'head', 'digests'], default=None)
    args = parser.parse_args()
    from oracle import build_ref
    ref = Path(args.reference) if args.reference else build_ref.reference_root()
    if ref is None:
        raise SystemExit('reference checkout not found: pass --reference or set ORNITH_REFERENCE')
    if args.only in (None, 'dense'):
        write_dense()
    if args.only in (None, 'head'):
        write_head()
    if args.only in (None, 'digests'):
        write_digests()
    if args.only:
        return
    import torch
    from safetensors.torch import load_file

    tables_path = ref / 'native' / 'shared_math_reference.safetensors'
    receipt = json.loads((ref / 'native' / 'shared_math_reference.json').read_text())
    sha = hashlib.sha256(tables_path.read_bytes()).hexdigest()
    if sha != receipt['sha256']:
        raise SystemExit('shared math table sha256 differs from the reference receipt')
    t = load_file(str(tables_path))
    silu = t['silu_fp32'].numpy()
    sigmoid = t['sigmoid_bf16'].view(torch.int16).numpy().view(np.uint16)
    np.savez_compressed(OUT / 'shared_math_tables.npz', silu_fp32=silu, sigmoid_bf16=sigmoid,
                        source_sha256=np.array(sha))

    S = _synthetic()
    layer = S.make_layer(np.random.default_rng(1))
    banks = (layer.gate_codes, layer.gate_meta, layer.down_codes, layer.down_meta)
    sbanks = (layer.sgate_codes, layer.sgate_meta, layer.sdown_codes, layer.sdown_meta)
    store = {'layer_seed': np.array(1), 'layer_sha256': np.array(digest(*banks, *sbanks, layer.shared_gate_w))}
    for name, _, case_seed, T, pad, hot, entry, special in CASES:
        x, w, ids = make_case(S, layer, case_seed, T, pad, hot, special)
        out, final, flags, st = O.ref_routed(x, w, ids, *banks, entry=entry)
        assert st == 0, (name, st)
        store[f'{name}/inputs_sha256'] = np.array(digest(x, w, ids))
        store[f'{name}/out'] = out
        if T <= 5:
            store[f'{name}/final_f32'] = final
        store[f'{name}/flags'] = np.array(flags, np.uint32)
        print(name, 'flags', flags)
    # fused shared slot (T <= 16) with the reference's tables
    for name, case_seed, T in (('shared_t1', 21, 1), ('shared_t7', 22, 7), ('shared_t16', 23, 16)):
        x, w, ids = make_case(S, layer, case_seed, T, 0.1, 0, '')
        logit = S.f32_to_bf16_bits(np.random.default_rng(case_seed + 100).standard_normal(T).astype(np.float32))
        out, shared, flags, st = O.ref_routed_shared(x, w, ids, *banks, *sbanks, logit, silu, sigmoid)
        assert st == 0
        store[f'{name}/inputs_sha256'] = np.array(digest(x, w, ids, logit))
        store[f'{name}/out'] = out
        store[f'{name}/shared_out'] = shared
        store[f'{name}/flags'] = np.array(flags, np.uint32)
        print(name, 'flags', flags)
    # configuration 1 of the benchmark: T=4, router linear, seed 0
    x, router, l1 = S.config1(0)
    logits = O.router_logits(x, router)
    w, ids = O.route_topk(logits)
    b1 = (l1.gate_codes, l1.gate_meta, l1.down_codes, l1.down_meta)
    store['config1/layer_sha256'] = np.array(digest(*b1, l1.sgate_codes, l1.sgate_meta, l1.sdown_codes,
                                                    l1.sdown_meta, l1.shared_gate_w))
    store['config1/logits'] = logits
    store['config1/ids'] = ids
    store['config1/weights'] = w
    for entry, key in (('ornith_routed_direct_launch', 'a8'), ('ornith_routed_direct_launch_a4', 'a4')):
        out, final, flags, st = O.ref_routed(x, w, ids, *b1, entry=entry)
        assert st == 0
        store[f'config1/out_{key}'] = out
        store[f'config1/flags_{key}'] = np.array(flags, np.uint32)
    np.savez_compressed(OUT / 'routed_reference_outputs.npz', **store)
    print('wrote', OUT / 'routed_reference_outputs.npz')


# (name, case seed, T, pad fraction, entry) on the seed-1 layer
DIGEST_CASES = [
    ('t32_a8', 51, 32, 0.05, 'ornith_routed_direct_launch'),
    ('t64_a4', 52, 64, 0.05, 'ornith_routed_direct_launch_a4'),
    ('t1120_a4prefill', 53, 1120, 0.05, 'ornith_routed_direct_launch_a4_prefill'),
]

# Experts with exactly these route counts: one short of, exactly at and one
# past a 128-row tile, two tiles, two tiles plus one, and more routes than
# tokens (duplicates inside tokens).  The grouped projection of the reference
# splits each expert into 16-row jobs (routed_storage_n32_prefill.h:19-42);
# the tensor-core path here into 128-row tiles.
HOT_COUNTS = {3: 127, 40: 128, 77: 129, 128: 256, 200: 257, 255: 1100}

# (name, case seed, T, pad fraction, entry, hot counts) on the seed-1 layer
HOT_DIGEST_CASES = [
    ('t300_hot_a8', 54, 300, 0.02, 'ornith_routed_direct_launch', HOT_COUNTS),
    ('t300_hot_a4', 55, 300, 0.02, 'ornith_routed_direct_launch_a4', HOT_COUNTS),
]


def make_hot_case(S, case_seed, T, pad, counts):
    """Tokens, then hot routes (synthetic.hot_routes), from one generator."""
    rng = np.random.default_rng(case_seed)
    x = S.make_tokens(rng, T)
    w, ids = S.hot_routes(rng, T, counts, pad_fraction=pad)
    return x, w, ids


def write_digests():
    S = _synthetic()
    layer = S.make_layer(np.random.default_rng(1))
    banks = (layer.gate_codes, layer.gate_meta, layer.down_codes, layer.down_meta)
    store = {}
    for name, case_seed, T, pad, entry in DIGEST_CASES:
        x, w, ids = make_case(S, layer, case_seed, T, pad, 0, '')
        out, _, flags, st = O.ref_routed(x, w, ids, *banks, entry=entry)
        assert st == 0, (name, st)
        store[f'{name}/inputs_sha256'] = np.array(digest(x, w, ids))
        store[f'{name}/out_sha256'] = np.array(digest(out))
        store[f'{name}/flags'] = np.array(flags, np.uint32)
        print(name, 'flags', flags)
    for name, case_seed, T, pad, entry, counts in HOT_DIGEST_CASES:
        x, w, ids = make_hot_case(S, case_seed, T, pad, counts)
        out, _, flags, st = O.ref_routed(x, w, ids, *banks, entry=entry)
        assert st == 0, (name, st)
        store[f'{name}/inputs_sha256'] = np.array(digest(x, w, ids))
        store[f'{name}/out_sha256'] = np.array(digest(out))
        store[f'{name}/flags'] = np.array(flags, np.uint32)
        print(name, 'flags', flags)
    np.savez_compressed(OUT / 'routed_reference_digests.npz', **store)
    print('wrote', OUT / 'routed_reference_digests.npz')


def write_head():
    S = _synthetic()
    store = {}
    for name, seed, M, N, geometry, special in HEAD_CASES:
        x, words, scales = make_head_case(S, seed, M, N, special)
        store[f'{name}/inputs_sha256'] = np.array(digest(x, words, scales))
        out, proj, flags, st, dots = O.ref_head(x, words, scales, N, geometry=geometry, group_dots=True)
        assert st == 0, (name, st)
        store[f'{name}/out'] = out
        store[f'{name}/projection'] = proj
        if M * N <= 4096:  # raw dots only for the small cases (fixture size)
            store[f'{name}/group_dots'] = dots
        store[f'{name}/flags'] = np.array(flags, np.uint32)
        print(name, 'flags', flags)
    np.savez_compressed(OUT / 'head_reference_outputs.npz', **store)
    print('wrote', OUT / 'head_reference_outputs.npz')


def write_dense():
    S = _synthetic()
    store = {}
    for name, seed, M, N, K, entry, geometry, special in DENSE_CASES:
        x, codes, meta = make_dense_case(S, seed, M, N, K, special)
        store[f'{name}/inputs_sha256'] = np.array(digest(x, codes, meta))
        if entry == 'prepare':
            xt, w, flags, st = O.ref_dense_prepare_bf16(x, codes, meta, N, K)
            assert st == 0, (name, st)
            store[f'{name}/transformed'] = xt
            store[f'{name}/weights'] = w
        else:
            if entry == 'n32':
                codes, meta = O.repack_n16_to_n32(codes[None], meta[None], N, K)
                codes, meta = codes[0], meta[0]
                fn = 'ornith_dense_g256_launch_n32'
            else:
                fn = 'ornith_dense_g256_launch'
            out, proj, flags, st = O.ref_dense(x, codes, meta, N, K, entry=fn, geometry=geometry)
            assert st == 0, (name, st)
            store[f'{name}/out'] = out
            store[f'{name}/projection'] = proj
        store[f'{name}/flags'] = np.array(flags, np.uint32)
        print(name, 'flags', flags)
    np.savez_compressed(OUT / 'dense_reference_outputs.npz', **store)
    print('wrote', OUT / 'dense_reference_outputs.npz')


if __name__ == '__main__':
    main()
