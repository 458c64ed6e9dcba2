"""GPU: the device dispatch plan (ornith_moe_b200_ep_plan, one launch) equals
the torch form of the plan on the same CUDA ids, field for field, with
padding and invalid ids, for 1-8 ranks and both placements, up to 8192
tokens.  One GPU: the plan involves no peer."""
import sys
from pathlib import Path

import pytest
import torch

sys.path.insert(0, str(Path(__file__).resolve().parent))
from test_ep_plan_cpu import _ids, _placements, torch_plan  # noqa: E402

pytestmark = pytest.mark.gpu
DEV = torch.device('cuda:0')


@pytest.mark.parametrize('world', [1, 2, 4, 8])
@pytest.mark.parametrize('T', [0, 1, 37, 1025, 4096, 8192])
def test_device_plan_matches_torch_plan(world, T):
    ep, placements = _placements(world)
    ids = _ids(T, 300 + T + world, world).to(DEV)
    for placement in placements:
        placement = ep.Placement(placement.rank.to(DEV), placement.local.to(DEV))
        counts, plan, row_index = torch_plan(ep, ids, world, placement)
        planner = ep.NativePlanner(world, placement, DEV)
        state, got_counts = planner.start(ids)
        got = planner.finish(state, ids, got_counts[:, 0].tolist(), got_counts[:, 1].tolist())
        torch.cuda.synchronize()
        assert torch.equal(got_counts, counts)
        for field in ('token_index', 'dest', 'local_ids', 'slot_mask'):
            assert torch.equal(getattr(got, field), getattr(plan, field)), field
        assert torch.equal(ep.route_row_index(T, got, DEV), row_index)
