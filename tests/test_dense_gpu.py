"""GPU: the dense G256 projections through the C ABI, bit for bit against the
reference's golden outputs and the oracle (A8 from N16 and N32 banks, the
bf16 prefill preparation), and the `ornith_b200::dense_out` operator."""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu
DEV = torch.device('cuda:0')


def assert_bits_equal(got, want, err_msg=''):
    """Bit equality, except that a NaN matches any NaN: the bits of a NaN made
    by arithmetic (inf*0 from an infinite weight scale or offset) are the
    hardware's default NaN (0x7FFFFFFF on NVIDIA GPUs, 0xFFC00000 on x86,
    where the reference's source was compiled for the golden vectors), and
    x86 passes an input NaN's bits through arithmetic where NVIDIA GPUs
    return their default NaN."""
    got, want = np.asarray(got), np.asarray(want)
    if got.dtype == np.uint16:
        nan = lambda b: ((b & 0x7F80) == 0x7F80) & ((b & 0x7F) != 0)  # noqa: E731
    else:
        got, want = got.view(np.uint32), want.view(np.uint32)
        nan = lambda b: ((b & 0x7F800000) == 0x7F800000) & ((b & 0x7FFFFF) != 0)  # noqa: E731
    np.testing.assert_array_equal(nan(got), nan(want), err_msg=err_msg)
    keep = ~nan(want)
    np.testing.assert_array_equal(got[keep], want[keep], err_msg=err_msg)


def _dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).to(DEV)


def _bf16(x_bits):
    return _dev(x_bits.view(np.int16)).view(torch.bfloat16)


def _u32(a):
    return _dev(np.ascontiguousarray(a).view(np.int32)).view(torch.uint32)


def _bits(t):
    return t.view(torch.int16).cpu().numpy().view(np.uint16)


def run_dense(native, x_bits, codes, meta, N, K, entry='n16', geometry=2, Mcap=None):
    """One launch; returns (status, out bf16 bits, fp32 projection, flags)."""
    lib = native.lib()
    M = x_bits.shape[0]
    Mcap = max(M, 1) if Mcap is None else Mcap
    layout = native.dense_get_layout(Mcap, N, K)
    ws = torch.empty(layout.workspace_bytes, dtype=torch.uint8, device=DEV)
    x = _bf16(x_bits)
    c, m = _u32(codes), _u32(meta)
    out = torch.full((M, N), -1, dtype=torch.int16, device=DEV).view(torch.bfloat16)
    flags = torch.zeros(1, dtype=torch.int32, device=DEV)
    fn = lib.ornith_dense_g256_launch if entry == 'n16' else lib.ornith_dense_g256_launch_n32
    st = fn(native.ptr(x), native.ptr(c), native.ptr(m), native.ptr(ws), ws.numel(), native.ptr(out),
            native.ptr(flags), M, Mcap, N, K, 8, 128, geometry, native.stream(x))
    torch.cuda.synchronize()
    proj = ws[layout.projection:layout.projection + M * N * 4].view(torch.float32).view(M, N).cpu().numpy()
    return st, _bits(out), proj, int(flags.item())


def run_prepare(native, x_bits, codes, meta, N, K):
    lib = native.lib()
    M = x_bits.shape[0]
    # device copies held in locals until the kernels have run (a temporary
    # freed after ptr() would hand its memory to the next allocation)
    x, c, m = _bf16(x_bits), _u32(codes), _u32(meta)
    xt = torch.empty((M, K), dtype=torch.bfloat16, device=DEV)
    w = torch.empty((N, K), dtype=torch.bfloat16, device=DEV)
    flags = torch.zeros(1, dtype=torch.int32, device=DEV)
    st = lib.ornith_dense_g256_prepare_bf16(native.ptr(x), native.ptr(c), native.ptr(m),
                                            native.ptr(xt), native.ptr(w), native.ptr(flags), M, N, K,
                                            native.stream(x))
    torch.cuda.synchronize()
    return st, _bits(xt), _bits(w), int(flags.item())


def _fp32_reduced_gemm(fn):
    """Run fn with cuBLAS told to keep split-K reductions in fp32: by default
    torch lets bf16 GEMMs reduce partial sums in bf16, whose error the fp32
    summation bound of these checks does not cover."""
    flag = torch.backends.cuda.matmul.allow_bf16_reduced_precision_reduction
    torch.backends.cuda.matmul.allow_bf16_reduced_precision_reduction = False
    try:
        result = fn()
        torch.cuda.synchronize()
        return result
    finally:
        torch.backends.cuda.matmul.allow_bf16_reduced_precision_reduction = flag


def test_dense_golden_cases(native, dense_golden, make_golden, S, O):
    """Every golden case of the compiled reference, bit for bit (out, fp32
    projection, flags), on the GPU."""
    for name, seed, M, N, K, entry, geometry, special in make_golden.DENSE_CASES:
        x, codes, meta = make_golden.make_dense_case(S, seed, M, N, K, special)
        assert make_golden.digest(x, codes, meta) == str(dense_golden[f'{name}/inputs_sha256']), name
        if entry == 'prepare':
            st, xt, w, flags = run_prepare(native, x, codes, meta, N, K)
            assert st == 0, name
            assert_bits_equal(xt, dense_golden[f'{name}/transformed'], err_msg=name)
            assert_bits_equal(w, dense_golden[f'{name}/weights'], err_msg=name)
        else:
            if entry == 'n32':
                codes, meta = O.repack_n16_to_n32(codes[None], meta[None], N, K)
                codes, meta = codes[0], meta[0]
            st, out, proj, flags = run_dense(native, x, codes, meta, N, K, entry, geometry)
            assert st == 0, name
            assert_bits_equal(out, dense_golden[f'{name}/out'], err_msg=name)
            assert_bits_equal(proj, dense_golden[f'{name}/projection'], err_msg=name)
        assert flags == int(dense_golden[f'{name}/flags']), name


@pytest.mark.parametrize('M,N,K,entry,geometry', [
    (1, 12288, 2048, 'n16', 2),    # QKVZ decode row
    (1, 12288, 2048, 'n32', 2),
    (4, 2048, 4096, 'n16', 1),
    (16, 512, 8192, 'n32', 2),     # largest K, a full 16-row block
    (17, 1024, 2048, 'n16', 0),    # two row blocks, the second with one row
    (5, 80, 768, 'n16', 2),        # N a multiple of 16 only: half-live last CTA
    (300, 96, 256, 'n16', 0),      # many ragged row blocks
])
def test_dense_matches_oracle(native, S, O, M, N, K, entry, geometry):
    rng = np.random.default_rng(1000 + M + N)
    codes, meta = S.make_dense_bank(rng, N, K)
    x = S.make_rows(rng, M, K)
    ref_out, ref_proj, ref_flags = O.dense_project(x, codes, meta, N, K, 16)
    if entry == 'n32':
        codes, meta = O.repack_n16_to_n32(codes[None], meta[None], N, K)
        codes, meta = codes[0], meta[0]
    st, out, proj, flags = run_dense(native, x, codes, meta, N, K, entry, geometry)
    assert st == 0
    np.testing.assert_array_equal(out, ref_out)
    np.testing.assert_array_equal(proj.view(np.uint32), ref_proj.view(np.uint32))
    assert flags == ref_flags == 0


def test_dense_zero_rows_touch_nothing(native):
    lib = native.lib()
    flags = torch.zeros(1, dtype=torch.int32, device=DEV)
    assert lib.ornith_dense_g256_launch(None, None, None, None, 0, None, native.ptr(flags), 0, 4, 64, 256, 8, 128,
                                        2, None) == 0
    assert int(flags.item()) == 0


def test_dense_n32_shadow_on_device(native, S, O):
    """The device repack of an N16 dense bank equals the reference's
    permutation, and the N32 launch equals the N16 launch."""
    N, K = 256, 1024
    rng = np.random.default_rng(77)
    codes, meta = S.make_dense_bank(rng, N, K)
    c32, m32 = native.dense_n32_shadow(_u32(codes), _u32(meta), N, K)
    rc, rm = O.repack_n16_to_n32(codes[None], meta[None], N, K)
    assert np.array_equal(c32.view(torch.int32).cpu().numpy().view(np.uint32), rc[0])
    assert np.array_equal(m32.view(torch.int32).cpu().numpy().view(np.uint32), rm[0])
    for M in (1, 16):
        x = S.make_rows(rng, M, K)
        a = run_dense(native, x, codes, meta, N, K, 'n16')
        b = run_dense(native, x, rc[0], rm[0], N, K, 'n32')
        assert a[0] == b[0] == 0
        np.testing.assert_array_equal(a[1], b[1])


def test_dense_out_operator_both_paths(native, S, O):
    """ornith_b200::dense_out: rows up to a8_max_rows take the A8 projection
    (bit for bit); longer batches take the bf16 prefill path, whose bf16 GEMM
    has an unspecified summation order, so it is compared with the exact
    product of the oracle's bf16 operands rounded to bf16: within one bf16
    ulp plus 2^-16 of the sum of |products| per element (an fp32 summation
    error bound), and relative L2 <= 1e-3."""
    N, K, capacity = 512, 2048, 64
    rng = np.random.default_rng(5)
    codes, meta = S.make_dense_bank(rng, N, K)
    c, m = _u32(codes), _u32(meta)
    ws = torch.empty(native.dense_workspace_bytes(capacity, [(N, K)]), dtype=torch.uint8, device=DEV)
    flags = torch.zeros(1, dtype=torch.int32, device=DEV)
    # A8 decode rows
    x = S.make_rows(rng, 8, K)
    out = torch.empty((8, N), dtype=torch.bfloat16, device=DEV)
    native.dense_out(_bf16(x), c, m, ws, out, flags, capacity, N, K, 2, 16)
    torch.cuda.synchronize()
    np.testing.assert_array_equal(_bits(out), O.dense_project(x, codes, meta, N, K, 16)[0])
    # bf16 prefill rows
    x = S.make_rows(rng, 48, K)
    out = torch.empty((48, N), dtype=torch.bfloat16, device=DEV)
    _fp32_reduced_gemm(lambda: native.dense_out(_bf16(x), c, m, ws, out, flags, capacity, N, K, 2, 16))
    xt, w, pf = O.dense_prepare_bf16(x, codes, meta, N, K)
    xa, wa = S.bf16_bits_to_f32(xt).astype(np.float64), S.bf16_bits_to_f32(w).astype(np.float64)
    exact = xa @ wa.T
    magnitude = np.abs(xa) @ np.abs(wa).T   # sum of |products|: scale of the fp32 summation error
    want = S.bf16_bits_to_f32(S.f32_to_bf16_bits(exact.astype(np.float32)))
    got = S.bf16_bits_to_f32(_bits(out))
    # one bf16 ulp of the result plus an fp32 summation error bound over K terms
    assert np.all(np.abs(got - want) <= np.abs(want) * 2.0 ** -7 + magnitude * 2.0 ** -16)
    assert np.linalg.norm(got - want) <= 1e-3 * np.linalg.norm(want)
    assert int(flags.item()) == pf == 0
