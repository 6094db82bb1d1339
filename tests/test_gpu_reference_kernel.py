"""The reference's own CUDA path against this library, on the GPU.

The reference's ``src/povs/__cuda/lib/povs.cu`` (its host loop ``povs_cuda`` and its kernel
``povs_kernel``) is compiled for sm_100a into ``oracle/_ref/libref_povs_cuda.so`` by
``oracle/build.py`` and run here next to ``povs_apply_v1``:

* the reference's whole CUDA path with a seed (std::mt19937 host draws, per-call allocations, one
  kernel per iteration) leaves a deck exactly as ``povs_apply_v1`` with ``sort_members=1`` leaves it
  when fed the oracle's restatement of that seed's randomness (``oracle/ref_cuda_rng.cpp``), on
  small decks with a truncated last pblock and padding slots, and on the full-size decks;
* the reference kernel alone, fed assignments with padding anywhere among the members and arbitrary
  seeds, equals ``povs_apply_v1`` fed the restatement's Stage 0 + Stage 2 of the same members and
  seeds.

Together these pin the restatement (host draws, member sort, xorshift32 Fisher-Yates) and this
library's injected path to the reference's compiled code byte for byte.  Only shapes whose copy
partition stays inside the pblock run (``ref_povs_layout_check``; see the driver's header).
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

import povs
from povs import _native

pytestmark = pytest.mark.gpu

DEV = "cuda:0"


@pytest.fixture(scope="module")
def ref(oracle_api):
    if oracle_api.ref_cuda_lib() is None:
        pytest.skip("oracle/_ref/libref_povs_cuda.so is not built (needs the reference checkout)")
    return oracle_api


def _shape(ref, V: int, P: int, row_bytes: int) -> int:
    idx = ref.ref_cuda_shape(V, P, row_bytes)
    assert idx is not None, f"no reference instantiation for V={V} P={P} row_bytes={row_bytes}"
    assert ref.ref_cuda_lib().ref_povs_layout_check(idx) == 0
    return idx


def _random_deck(n_rows: int, row_bytes: int, seed: int) -> torch.Tensor:
    g = torch.Generator(device=DEV).manual_seed(seed)
    return torch.randint(0, 256, (n_rows, row_bytes), dtype=torch.uint8, device=DEV, generator=g)


def _equal_in_chunks(a: torch.Tensor, b: torch.Tensor, chunk_rows: int = 1 << 22) -> bool:
    """torch.equal over row chunks (a whole-deck comparison would allocate a mask as large as the deck)."""
    assert a.shape == b.shape
    for s in range(0, a.shape[0], chunk_rows):
        if not torch.equal(a[s:s + chunk_rows], b[s:s + chunk_rows]):
            return False
    return True


def _apply_restated(ref, deck: torch.Tensor, row_bytes: int, P: int, V: int, offsets: list[int], iterations: int,
                    seed: int) -> None:
    """povs_apply_v1 fed the restatement of the reference CUDA path's randomness for ``seed``."""
    offs, assign, perms = ref.refcuda_randomness(seed, deck.shape[0], P, V, offsets, iterations)
    _native.apply(deck, row_bytes, P, V, [int(o) for o in offs], torch.from_numpy(assign).to(DEV),
                  torch.from_numpy(perms).to(DEV), True)
    torch.cuda.synchronize()
    povs.check_device_status(0)


# (V, P, row_bytes, n_rows, offsets, iterations): every instantiated shape, each deck with a
# truncated last pblock and, where the counts allow, padding slots in the last vblock.
SMALL = [
    (2, 16, 64, 1000, list(range(16)), 3),  # 63 pblocks (last has 8 rows), 32 vblocks, 1 padding slot
    (4, 16, 64, 1000, [0, 1, 2, 3, 5], 3),  # 16 vblocks, 1 padding slot
    (2, 64, 256, 4099, list(range(16)), 4),  # 65 pblocks (last has 3 rows), 1 padding slot
    (4, 32, 256, 5000, list(range(16)), 4),  # 157 pblocks (last has 8 rows), 3 padding slots
    (4, 64, 128, 3001, list(range(16)), 3),  # 47 pblocks (last has 57 rows), 1 padding slot
    (8, 16, 128, 2500, [0, 1, 2, 7, 9], 3),  # 157 pblocks, 3 padding slots
    (2, 32, 512, 1030, [0, 1, 2, 3], 3),  # 33 pblocks (last has 6 rows), 1 padding slot
    (16, 16, 128, 3333, [0, 3, 5], 2),  # 209 pblocks: the last vblock holds 1 pblock and 15 padding slots
]


@pytest.mark.parametrize("V,P,row_bytes,n_rows,offsets,iterations", SMALL)
@pytest.mark.parametrize("seed", [0, 2024])
def test_reference_cuda_path_equals_injected_restatement(ref, V, P, row_bytes, n_rows, offsets, iterations, seed):
    shape = _shape(ref, V, P, row_bytes)
    original = _random_deck(n_rows, row_bytes, seed=n_rows + V)
    theirs = original.clone()
    ours = original.clone()
    torch.cuda.synchronize()
    ref.ref_povs_cuda(shape, theirs.data_ptr(), n_rows, offsets, iterations, seed)
    _apply_restated(ref, ours, row_bytes, P, V, offsets, iterations, seed)
    assert not torch.equal(theirs, original), "the reference left the deck unchanged"
    assert torch.equal(ours, theirs), "povs_apply_v1 with the restated randomness differs from the reference"


@pytest.mark.parametrize("V,P,row_bytes,n_rows,offsets,iterations", SMALL)
def test_reference_kernel_with_any_members_equals_apply(ref, V, P, row_bytes, n_rows, offsets, iterations):
    """Members in any order with padding anywhere (the reference's host loop only ever leaves padding
    in the last vblock), seeds over the whole int32 range: the kernel's member sort and Fisher-Yates."""
    shape = _shape(ref, V, P, row_bytes)
    n_p, n_v = ref.block_counts(n_rows, P, V)
    rng = np.random.default_rng(n_rows * V)
    original = _random_deck(n_rows, row_bytes, seed=P + V)
    theirs = original.clone()
    ours = original.clone()
    for it in range(iterations):
        slots = rng.permutation(n_v * V)
        assign = np.where(slots < n_p, slots, -1).astype(np.int64).reshape(n_v, V)
        seeds = rng.integers(1, 2**31 - 1, size=n_v, dtype=np.int64).astype(np.int32)
        seeds[: n_v // 2] = rng.integers(1, 1000, size=n_v // 2)
        offset = int(offsets[it % len(offsets)])
        perms = ref.refcuda_perms(n_rows, P, V, assign, seeds)
        assign_d = torch.from_numpy(assign).to(DEV)
        seeds_d = torch.from_numpy(seeds).to(DEV)
        torch.cuda.synchronize()
        ref.ref_povs_kernel(shape, theirs.data_ptr(), n_rows, assign_d.data_ptr(), seeds_d.data_ptr(), offset)
        torch.cuda.synchronize()
        _native.apply(ours, row_bytes, P, V, [offset], assign_d, torch.from_numpy(perms).to(DEV), True)
        torch.cuda.synchronize()
        povs.check_device_status(0)
        assert torch.equal(ours, theirs), f"iteration {it}: povs_apply_v1 differs from the reference kernel"
    assert not torch.equal(theirs, original)


def _full_size(ref, V: int, P: int, row_bytes: int, deck: torch.Tensor, offsets: list[int], iterations: int,
               seed: int) -> None:
    shape = _shape(ref, V, P, row_bytes)
    rows = deck.view(torch.uint8).reshape(deck.shape[0], row_bytes)
    ours = rows.clone()
    torch.cuda.synchronize()
    ref.ref_povs_cuda(shape, rows.data_ptr(), rows.shape[0], offsets, iterations, seed)
    _apply_restated(ref, ours, row_bytes, P, V, offsets, iterations, seed)
    assert _equal_in_chunks(ours, rows), "full-size deck differs from the reference's CUDA path"


def test_full_size_fp16_deck_equals_reference_cuda_path(ref):
    """1,048,576 x 128 fp16 (256 MiB), V=2, P=64, 4 iterations, the reference chooser's offsets and
    thread-block size (64)."""
    host = np.random.default_rng(0).standard_normal((1_048_576, 128)).astype(np.float16)
    deck = torch.from_numpy(host).to(DEV)
    _full_size(ref, 2, 64, 256, deck, povs.common.choose_offsets(1_048_576, 128, 2, 64), 4, seed=0)


def test_full_size_bf16_deck_equals_reference_cuda_path(ref):
    """134,217,728 x 128 bf16 (32 GiB), V=4, P=32, 4 iterations: the deck moved as 2-byte values, as
    the reference's c10::Half instantiation moves it (its dtype list has no bf16)."""
    n_rows = 134_217_728
    g = torch.Generator(device=DEV).manual_seed(1)
    deck = torch.rand((n_rows, 128), generator=g, device=DEV, dtype=torch.bfloat16) * 2 - 1
    _full_size(ref, 4, 32, 256, deck, povs.common.choose_offsets(n_rows, 128, 2, 32), 4, seed=1)
    del deck
    torch.cuda.empty_cache()


def test_sharded_fp32_rows_equal_reference_cuda_path(ref):
    """fp32 x 32 rows (128 B), V=4, P=64, 4 iterations, on one GPU's share of the sharded deck at 8 GPUs
    (134,217,728 rows, 16 GiB) plus 5 rows so the last pblock is truncated.  Thread-block size 32:
    the reference's chooser picks 64 for these rows, which its copy partition overruns."""
    n_rows = 134_217_728 + 5
    g = torch.Generator(device=DEV).manual_seed(3)
    deck = torch.randn((n_rows, 32), generator=g, device=DEV, dtype=torch.float32)
    _full_size(ref, 4, 64, 128, deck, povs.common.choose_offsets(n_rows, 32, 4, 64), 4, seed=3)
    del deck
    torch.cuda.empty_cache()
