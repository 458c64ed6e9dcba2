"""GPU: the W8 LM head through the C ABI, bit for bit against the reference's
golden outputs and the oracle (logits, fp32 projections, raw group dots,
flags), and the `ornith_b200::head_out` operator at the full vocabulary."""
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


def _u32(a):
    return torch.from_numpy(np.ascontiguousarray(a).view(np.int32)).to(DEV).view(torch.uint32)


def _f16(bits):
    return torch.from_numpy(np.ascontiguousarray(bits).view(np.int16)).to(DEV).view(torch.float16)


def _bf16(bits):
    return torch.from_numpy(np.ascontiguousarray(bits).view(np.int16)).to(DEV).view(torch.bfloat16)


def run_head(native, x_bits, words, scales, N, geometry=2, dots=False, Mcap=None):
    M = x_bits.shape[0]
    Mcap = max(M, 1) if Mcap is None else Mcap
    layout = native.head_get_layout(Mcap, N)
    ws = torch.empty(layout.workspace_bytes, dtype=torch.uint8, device=DEV)
    out = torch.full((M, N), -1, dtype=torch.int16, device=DEV).view(torch.bfloat16)
    flags = torch.zeros(1, dtype=torch.int32, device=DEV)
    gd = torch.full((M, N, 16), 7, dtype=torch.int32, device=DEV) if dots else None
    native.head_launch(_bf16(x_bits), _u32(words), _f16(scales), ws, out, flags, N, Mcap, geometry, gd)
    torch.cuda.synchronize()
    proj = ws[layout.projection:layout.projection + M * N * 4].view(torch.float32).view(M, N).cpu().numpy()
    return (out.view(torch.int16).cpu().numpy().view(np.uint16), proj, int(flags.item()),
            gd.cpu().numpy() if dots else None)


def test_head_golden_cases(native, head_golden, make_golden, S):
    for name, seed, M, N, geometry, special in make_golden.HEAD_CASES:
        x, words, scales = make_golden.make_head_case(S, seed, M, N, special)
        has_dots = f'{name}/group_dots' in head_golden
        out, proj, flags, dots = run_head(native, x, words, scales, N, geometry, dots=has_dots)
        assert_bits_equal(out, head_golden[f'{name}/out'], err_msg=name)
        assert_bits_equal(proj, head_golden[f'{name}/projection'], err_msg=name)
        if has_dots:
            np.testing.assert_array_equal(dots, head_golden[f'{name}/group_dots'], err_msg=name)
        assert flags == int(head_golden[f'{name}/flags']), name


@pytest.mark.parametrize('M,N', [(1, 65536), (4, 4096), (33, 1024), (64, 256)])
def test_head_matches_oracle(native, S, O, M, N):
    rng = np.random.default_rng(300 + M)
    words, scales = S.make_head_bank(rng, N)
    x = S.make_rows(rng, M, 2048)
    ref_out, ref_proj, ref_flags, ref_dots = O.head_project(x, words, scales, N, group_dots=True)
    out, proj, flags, dots = run_head(native, x, words, scales, N, dots=True)
    np.testing.assert_array_equal(out, ref_out)
    np.testing.assert_array_equal(proj.view(np.uint32), ref_proj.view(np.uint32))
    np.testing.assert_array_equal(dots, ref_dots)
    assert flags == ref_flags == 0


def test_head_out_full_vocabulary(native, S, O):
    """ornith_b200::head_out over the 248,320-column vocabulary, 2 rows,
    checked bit for bit against the oracle on a column sample."""
    N = native.HEAD_VOCAB
    rng = np.random.default_rng(9)
    codes = torch.randint(-127, 128, (N // 16, 128, 4, 16, 4), dtype=torch.int8, device=DEV,
                          generator=torch.Generator(device=DEV).manual_seed(9))
    words = codes.view(torch.int32).view(N // 16, 128, 4, 16).view(torch.uint32)
    scales = (0.01 * torch.randn((N, 16), device=DEV, generator=torch.Generator(device=DEV).manual_seed(10)).abs()
              ).to(torch.float16).clamp_min(2 ** -14)
    x = S.make_rows(rng, 2, 2048)
    ws = torch.empty(native.head_get_layout(native.HEAD_ROWS).workspace_bytes, dtype=torch.uint8, device=DEV)
    out = torch.empty((2, N), dtype=torch.bfloat16, device=DEV)
    flags = torch.zeros(1, dtype=torch.int32, device=DEV)
    native.head_out(_bf16(x), words, scales, ws, out, flags, 2)
    torch.cuda.synchronize()
    got = out.view(torch.int16).cpu().numpy().view(np.uint16)
    # oracle on the first, a middle and the last 16-column tiles
    w_np = words.view(torch.int32).cpu().numpy().view(np.uint32)
    s_np = scales.view(torch.int16).cpu().numpy().view(np.uint16)
    for t in (0, 7777, N // 16 - 1):
        ref, _, ref_flags = O.head_project(x, w_np[t:t + 1], s_np[16 * t:16 * t + 16], 16)
        np.testing.assert_array_equal(got[:, 16 * t:16 * t + 16], ref)
    assert int(flags.item()) == 0
