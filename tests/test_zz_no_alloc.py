"""The allocation-free injection entry point (povs_apply_static_v1) against povs_apply_v1.

povs_apply_static_v1 serves callers that cannot allocate GPU memory at run time (a process whose
memory pool already holds the GPU's free memory, or a service that forbids allocation after
start-up): the injected randomness comes from host arrays and is staged in a fixed scratch array
inside the library instead of caller-allocated device buffers.  It must produce exactly the bytes
of povs_apply_v1, on consecutive calls that reuse the same scratch array.

This file is collected last, so a run that stops at the first failure has run everything else.
"""

from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch

from povs import _native

pytestmark = pytest.mark.gpu

DEV = "cuda:0"


def _deck(n_rows: int, row_bytes: int, seed: int) -> torch.Tensor:
    host = np.random.default_rng(seed).integers(0, 256, size=(n_rows, row_bytes), dtype=np.uint8)
    return torch.from_numpy(host).to(DEV)


@pytest.mark.parametrize(
    "n_rows,row_bytes,P,V,offsets,seed",
    [(1000, 64, 8, 2, list(range(8)), 3), (4099, 256, 32, 4, [0, 1, 2, 5], 7), (2000, 12, 16, 8, [0, 1, 3], 11)],
)
def test_static_entry_matches_apply_on_consecutive_calls(oracle_api, n_rows, row_bytes, P, V, offsets, seed):
    # Two calls in a row, each with its own randomness, on both entry points.
    offs, assign, perms = oracle_api.refcuda_randomness(seed, n_rows, P, V, offsets, 2)
    ref = _deck(n_rows, row_bytes, seed)
    got = ref.clone()
    for t in range(2):
        _native.apply(ref, row_bytes, P, V, [int(offs[t])], torch.from_numpy(assign[t]).to(DEV),
                      torch.from_numpy(perms[t]).to(DEV), True)
        torch.cuda.synchronize()
        _native.apply_static(got, row_bytes, P, V, [int(offs[t])], assign[t], perms[t], True)
        assert torch.equal(got, ref), f"call {t + 1}: the static-scratch entry differs from povs_apply_v1"
    assert _native.device_status(0) == 0


def test_static_entry_numpy_order_two_iterations_per_call(oracle_api):
    n_rows, row_bytes, P, V = 1024, 32, 16, 2
    from oracle import numpy_path

    offs, assign, perms = numpy_path.numpy_path_randomness(5, n_rows, P, V, list(range(16)), 4)
    ref = _deck(n_rows, row_bytes, 5)
    got = ref.clone()
    for call in range(2):
        sl = slice(2 * call, 2 * call + 2)
        _native.apply(ref, row_bytes, P, V, [int(o) for o in offs[sl]], torch.from_numpy(assign[sl].copy()).to(DEV),
                      torch.from_numpy(perms[sl].copy()).to(DEV), False)
        torch.cuda.synchronize()
        _native.apply_static(got, row_bytes, P, V, [int(o) for o in offs[sl]], assign[sl], perms[sl], False)
        assert torch.equal(got, ref)


def test_static_entry_rejects_decks_beyond_its_scratch():
    lib = _native.load()
    n_rows, row_bytes, P, V = 4_000_000, 16, 16, 2  # permutations alone need 16 MB > 8 MiB
    deck = torch.empty((16, 16), dtype=torch.uint8, device=DEV)  # never touched: rejected before launch
    n_p = n_rows // P
    assign = np.zeros(n_p, dtype=np.int64)
    perms = np.zeros(n_p * P, dtype=np.int32)
    offs = (ctypes.c_int64 * 1)(0)
    rc = lib.povs_apply_static_v1(ctypes.c_void_p(deck.data_ptr()), n_rows, row_bytes, P, V, 1, offs,
                                  ctypes.c_void_p(assign.ctypes.data), ctypes.c_void_p(perms.ctypes.data), 1, 0,
                                  None, 0)
    assert rc == -2
    assert b"scratch" in lib.povs_last_error_string()


def test_static_entry_reports_a_bad_injected_entry_only_when_synchronous():
    """An out-of-range permutation entry is ignored by the kernel (identity used) and flagged in the
    entry's own status word, which POVS_FLAG_SYNC reads back as POVS_ERR_DEVICE_STATUS."""
    lib = _native.load()
    n_rows, row_bytes, P, V = 256, 16, 16, 2
    n_p = n_rows // P
    n_v = n_p // V
    deck = _deck(n_rows, row_bytes, 13)
    assign = np.arange(n_v * V, dtype=np.int64)
    perms = np.tile(np.arange(V * P, dtype=np.int32), n_v)
    perms[5] = V * P + 3  # outside the vblock's rows
    offs = (ctypes.c_int64 * 1)(0)
    args = (ctypes.c_void_p(deck.data_ptr()), n_rows, row_bytes, P, V, 1, offs, ctypes.c_void_p(assign.ctypes.data),
            ctypes.c_void_p(perms.ctypes.data), 1, 0, None)
    assert lib.povs_apply_static_v1(*args, _native.FLAG_SYNC) == -4
    assert b"device status" in lib.povs_last_error_string()
    perms[5] = 5
    assert lib.povs_apply_static_v1(*args, _native.FLAG_SYNC) == 0
