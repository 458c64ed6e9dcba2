"""CPU: properties the oracle's building blocks must have for any input
(hypothesis-generated groups), beside the golden vectors that pin them to the
reference: the A8/A4 quantiser's scale rule, code range, rounding and sums,
and the Hadamard transform's self-inverse."""
import math

import numpy as np
import pytest
from hypothesis import given, settings, strategies as st
from hypothesis.extra.numpy import arrays

finite32 = st.floats(min_value=-1e4, max_value=1e4, allow_nan=False, allow_infinity=False, width=32)


@settings(max_examples=300, deadline=None)
@given(v=arrays(np.float32, 256, elements=finite32), a8=st.booleans(), scale_exp=st.integers(-20, 8))
def test_quantiser_properties(O, v, a8, scale_exp):
    y = (v * np.float32(2.0 ** scale_exp)).astype(np.float32)[None, :]
    q, scales, sums, flags = O.quantize_rows(y, a8=a8)
    qmax = 127 if a8 else 7
    absmax = float(np.abs(y).max())
    s = float(np.array([scales[0, 0]], np.uint16).view(np.float16)[0])
    assert int(sums[0, 0]) == int(q.astype(np.int64).sum())
    assert np.abs(q).max() <= qmax
    if np.float32(absmax) / np.float32(qmax) > 65504:
        # the scale would overflow fp16: invalid group (flag 2), scale 1, codes 0
        assert flags == 2 and s == 1.0 and not q.any()
        return
    assert flags == 0
    if absmax == 0.0:
        assert s == 1.0 and not q.any()
        return
    # scale = fp16_rne(max(absmax / qmax, 2^-14))
    want = np.float16(max(np.float32(absmax) / np.float32(qmax), np.float32(2.0 ** -14)))
    assert s == float(want)
    # every unclamped code is v / scale rounded to nearest (ties to even)
    ratio = y[0].astype(np.float64) / s
    inside = np.abs(ratio) < qmax
    assert np.all(np.abs(ratio[inside] - q[0][inside]) <= 0.5 + 1e-6)
    assert np.all(np.abs(q[0][~inside]) >= qmax - 1)


@settings(max_examples=100, deadline=None)
@given(v=arrays(np.float32, 128, elements=st.floats(-100, 100, width=32)))
def test_hadamard_is_its_own_inverse(O, v):
    # H/sqrt(128) is symmetric and orthogonal: applying it twice returns v
    twice = O.wht128(O.wht128(v))
    np.testing.assert_allclose(twice, v, rtol=1e-4, atol=1e-4 * max(1.0, float(np.abs(v).max())))
    # and it preserves the norm
    assert math.isclose(float(np.linalg.norm(O.wht128(v))), float(np.linalg.norm(v)), rel_tol=1e-5, abs_tol=1e-5)


@pytest.mark.parametrize('N,K', [(64, 256), (96, 512), (32, 2048)])
def test_repack_is_a_permutation(O, N, K):
    rng = np.random.default_rng(N + K)
    codes = rng.integers(0, 2 ** 32, size=(2, N // 16, K // 256, 32, 16), dtype=np.uint32)
    meta = rng.integers(0, 2 ** 32, size=(2, N // 16, K // 256, 16), dtype=np.uint32)
    c32, m32 = O.repack_n16_to_n32(codes, meta, N, K)
    assert np.array_equal(np.sort(c32.ravel()), np.sort(codes.ravel()))
    assert np.array_equal(np.sort(m32.ravel()), np.sort(meta.ravel()))
    # column 16h + l of N32 tile t is column l of N16 tile 2t + h
    assert np.array_equal(c32[:, :, :, :, 16:], codes[:, 1::2])
    assert np.array_equal(m32[:, :, :, :16], meta[:, 0::2])
