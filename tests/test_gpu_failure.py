"""Failure detection on one GPU without a fault: a cross-GPU barrier whose peer never arrives.

Rank 0 of a two-shard deck runs alone (both shards and both flag arrays are local buffers, and no
other kernel ever writes rank 1's flag), so its barrier waits on a flag that nothing sets; with a
0.3 s limit it gives up, reports POVS_DEV_PEER_TIMEOUT through the status word, and the context
stays usable.  Nothing here waits on another kernel.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

import povs
from povs import _native

pytestmark = pytest.mark.gpu
DEV = "cuda:0"


@pytest.mark.parametrize("double_buffer", [False, True])
def test_missing_peer_times_out_and_is_reported(oracle_api, double_buffer):
    n, row_bytes, P, V, offsets = 4096, 64, 16, 2, [0, 1, 3]
    rng = np.random.default_rng(1)
    host = rng.integers(0, 256, (2 * n, row_bytes), dtype=np.uint8)
    shards = [torch.from_numpy(host[:n].copy()).to(DEV), torch.from_numpy(host[n:].copy()).to(DEV)]
    scratch = [torch.empty_like(s) for s in shards] if double_buffer else None
    flags = [torch.zeros(2, dtype=torch.int32, device=DEV), torch.zeros(2, dtype=torch.int32, device=DEV)]
    povs.check_device_status(0)
    _native.set_peer_wait_limit(0.3)
    try:
        _native.shuffle_sharded(
            [s.data_ptr() for s in shards], [n, n], 0, row_bytes, offsets, 1, P, V, 5,
            [f.data_ptr() for f in flags], 0, 0, 0,
            scratch_ptrs=[b.data_ptr() for b in scratch] if scratch else None,
        )
        torch.cuda.synchronize()
        with pytest.raises(RuntimeError, match="0x4"):
            povs.check_device_status(0)
    finally:
        _native.set_peer_wait_limit(None)
    # Rank 0 published its arrival in both arrays; rank 1's slot stayed empty.
    assert int(flags[0][0]) >= 1 and int(flags[1][0]) >= 1 and int(flags[0][1]) == 0
    # The context is still usable.
    deck = torch.from_numpy(host.copy()).to(DEV)
    povs.shuffle(deck, iterations=2, options=povs.Options(V, P, offsets, 32), seed=9)
    torch.cuda.synchronize()
    povs.check_device_status(0)
    want = host.copy()
    oracle_api.shuffle(want, 2, P, V, offsets, 9)
    assert np.array_equal(deck.cpu().numpy(), want)
