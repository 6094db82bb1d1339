"""The host planner (povs_plan_for_resources_v1) fed this GPU's resources gives the plan the device
entry (povs_describe_plan_v1) reports, for unpacked, packed, slabbed and plain-load decks."""

from __future__ import annotations

import pytest
import torch

from povs import _native

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize(
    "n_rows,row_bytes,P,V",
    [(1 << 20, 256, 32, 4), (1 << 20, 16, 64, 2), (50_000, 12288, 16, 2), (1 << 20, 12, 128, 2), (1 << 18, 512, 32, 2),
     (1 << 20, 48, 64, 2), (1 << 20, 3, 32, 2), (100_003, 1040, 8, 2)],
)
def test_host_plan_equals_device_plan(n_rows, row_bytes, P, V):
    deck = torch.empty((n_rows, row_bytes), dtype=torch.uint8, device="cuda:0")
    prop = torch.cuda.get_device_properties(0)
    resources = (prop.multi_processor_count, prop.shared_memory_per_block_optin,
                 prop.shared_memory_per_multiprocessor, prop.max_threads_per_multi_processor)
    device_plan = _native.describe_plan(deck, row_bytes, P, V)
    host_plan = _native.plan_for_resources(n_rows, row_bytes, P, V, resources=resources, address=deck.data_ptr())
    assert host_plan == device_plan
