"""GPU: the shared expert in the reference's dense decode form
(shared_kernel.py:33-62) through this library's dense N32 launches, against
the oracle composition.  Its elementwise tail (vLLM's silu_and_mul, torch's
sigmoid, an fp32 logit sum) is not pinned by the reference, so the output is
compared within the north-star bound: relative L2 <= 1e-3, and per element
within two bf16 ulps of the oracle (or 2e-2, the larger)."""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu
DEV = torch.device('cuda:0')


def _u32(a):
    return torch.from_numpy(np.ascontiguousarray(a).view(np.int32)).to(DEV).view(torch.uint32)


def _bf16(bits):
    return torch.from_numpy(np.ascontiguousarray(bits).view(np.int16)).to(DEV).view(torch.bfloat16)


@pytest.mark.parametrize('M', [1, 8, 16, 17, 40])
def test_shared_dense_matches_oracle(native, layer1, S, O, M):
    x = S.make_tokens(np.random.default_rng(70 + M), M)
    banks = [_u32(b) for b in (layer1.sgate_codes, layer1.sgate_meta, layer1.sdown_codes, layer1.sdown_meta)]
    gate_w = _bf16(layer1.shared_gate_w)
    ws = torch.empty(native.shared_dense_workspace_bytes(), dtype=torch.uint8, device=DEV)
    gate_flags = torch.zeros(1, dtype=torch.int32, device=DEV)
    down_flags = torch.zeros(1, dtype=torch.int32, device=DEV)
    xd = _bf16(x)
    out = native.shared_dense_out(xd, *banks, gate_w, ws, gate_flags, down_flags)
    torch.cuda.synchronize()
    got = S.bf16_bits_to_f32(out.view(torch.int16).cpu().numpy().view(np.uint16))
    ref, gf, df = O.shared_dense(x, layer1.sgate_codes, layer1.sgate_meta, layer1.sdown_codes, layer1.sdown_meta,
                                 layer1.shared_gate_w)
    want = S.bf16_bits_to_f32(ref)
    ulp = 2.0 ** (np.floor(np.log2(np.maximum(np.abs(want), 2.0 ** -126))) - 7)
    assert np.all(np.abs(got - want) <= np.maximum(2 * ulp, 2e-2))
    assert np.linalg.norm(got - want) <= 1e-3 * np.linalg.norm(want)
    assert (int(gate_flags.item()), int(down_flags.item())) == (gf, df) == (0, 0)
