"""GPU parity: the CUDA library (called through its C ABI) against the oracle and the reference.

* default mode (device randomness) == the oracle's restatement of it, byte for byte;
* injected reference randomness (NumPy path, CUDA path) == the reference's output / the oracle;
* full-size runs keep the multiset of rows (every row intact, each exactly once).
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

import povs
from povs import _native
from oracle import numpy_path

pytestmark = pytest.mark.gpu

DEV = "cuda:0"


def random_rows(n_rows: int, row_bytes: int, seed: int) -> np.ndarray:
    return np.random.default_rng(seed).integers(0, 256, size=(n_rows, row_bytes), dtype=np.uint8)


def gpu_shuffle_bytes(host: np.ndarray, P: int, V: int, offsets: list[int], iterations: int, seed: int,
                      flags: int = 0) -> np.ndarray:
    dev = torch.from_numpy(host.copy()).to(DEV)
    _native.shuffle_device(dev, host.shape[1], offsets, iterations, P, V, seed, flags)
    torch.cuda.synchronize()
    povs.check_device_status(0)
    return dev.cpu().numpy()


# (n_rows, row_bytes, P, V, offsets, iterations): bulk (TMA) and plain-load paths, ragged decks,
# truncated last pblocks, padding slots, column slabs, every sort width.
DEFAULT_CASES = [
    (64, 16, 16, 2, [0, 4], 1),
    (1000, 64, 8, 2, list(range(8)), 4),
    (1000, 12, 16, 4, [0, 1, 3], 3),
    (4099, 256, 32, 4, [0, 1, 2, 5], 2),
    (5000, 3, 64, 2, [0, 2, 4], 2),
    (777, 2, 16, 8, [0, 1, 2], 2),
    (3000, 8, 128, 8, [0, 1, 5], 2),
    (2048, 4096, 16, 2, [0, 1, 3], 2),
    (1200, 12288, 16, 2, [0, 1, 2], 3),
    (100_000, 128, 64, 4, list(range(16)), 4),
    (2, 4, 8, 2, [0, 1], 3),
    (4100, 20, 32, 16, [0, 1, 2], 2),
    (70_000, 48, 32, 32, [0, 7, 9], 2),
    (50_000, 32, 64, 8, [0, 3, 6, 11], 3),
    (9999, 24, 16, 2, [0, 5], 2),
    (1 << 16, 256, 8, 2, [0, 1], 1),
    # Rows of 32 to 128 16-byte chunks (several chunk loads in flight per lane), small and large units.
    (3001, 512, 16, 2, [0, 1, 3], 3),
    (2500, 768, 32, 2, [0, 2], 2),
    (1500, 1040, 8, 2, [0, 1], 2),
    # Vblocks of 1024 and 512 rows: whole narrow rows in two or three large stages, or two slabs.
    (4000, 64, 512, 2, [0, 1], 2),
    (5000, 96, 512, 2, [0, 2], 2),
    (3000, 128, 256, 2, [0, 1], 2),
]


@pytest.mark.parametrize("n_rows,row_bytes,P,V,offsets,iterations", DEFAULT_CASES)
@pytest.mark.parametrize("seed", [0, 2**40 + 17])
def test_default_mode_matches_oracle(oracle_api, n_rows, row_bytes, P, V, offsets, iterations, seed):
    host = random_rows(n_rows, row_bytes, seed=n_rows + row_bytes)
    got = gpu_shuffle_bytes(host, P, V, offsets, iterations, seed)
    want = host.copy()
    oracle_api.shuffle(want, iterations, P, V, offsets, seed)
    assert np.array_equal(got, want)


@pytest.mark.parametrize(
    "n_rows,row_bytes,P,V,offsets,iterations",
    [(1000, 64, 8, 2, list(range(8)), 4), (4099, 256, 32, 4, [0, 1, 2, 5], 3), (20_000, 12, 16, 8, [0, 1, 3], 2),
     (3000, 8, 128, 8, [0, 1, 5], 2)],
)
def test_reference_cuda_randomness_mode_matches_oracle(oracle_api, n_rows, row_bytes, P, V, offsets, iterations):
    host = random_rows(n_rows, row_bytes, seed=11)
    got = gpu_shuffle_bytes(host, P, V, offsets, iterations, 77, flags=_native.FLAG_REFERENCE_RNG)
    want = host.copy()
    oracle_api.shuffle(want, iterations, P, V, offsets, 77, "reference_cuda")
    assert np.array_equal(got, want)


# (n_decks, n_rows, row_bytes, P, V, offsets, iterations): small vblocks that travel several per unit.
PACKED_CASES = [
    (1, 1000, 64, 8, 2, list(range(8)), 4),  # 63 vblocks: 16 per unit, the last unit has 15
    (1, 20_011, 16, 16, 2, [0, 1, 3, 5], 3),  # truncated last pblock; bulk loads
    (1, 30_000, 12, 16, 4, [0, 1, 2], 2),  # plain 4-byte loads
    (1, 7_777, 3, 32, 2, [0, 1, 2], 3),  # byte rows
    (1, 65_536, 256, 8, 2, [0, 1], 2),  # 4 KiB vblocks, 4 per unit
    (1, 999, 32, 4, 8, [0, 1, 2, 3], 3),  # V = 8, 4 vblocks per unit
    (37, 1000, 64, 8, 2, list(range(8)), 3),  # batched decks: units never straddle two decks
    (1, 30_011, 48, 64, 2, [0, 1, 3, 5], 3),  # 48-byte rows: 8 vblocks, 48 KiB units beyond the stage cap
    (1, 20_003, 96, 32, 2, [0, 2], 2),  # 96-byte rows: 4 vblocks, 24 KiB units
    # Plain-load rows stored as 16-byte chunks of each member's run (runs start at any 4-byte offset).
    (1, 20_011, 12, 128, 2, [0, 1, 3, 5], 3),
    (1, 10_007, 20, 64, 2, [0, 1, 2], 2),
    (1, 40_003, 4, 128, 2, [0, 1, 3], 3),
    (5, 3001, 24, 64, 2, [0, 1, 2, 3], 2),
]


@pytest.mark.parametrize("n_decks,n_rows,row_bytes,P,V,offsets,iterations", PACKED_CASES)
@pytest.mark.parametrize("randomness", ["uniform", "reference_cuda", "reference_numpy"])
def test_packed_units_match_single_vblock_units_and_oracle(oracle_api, n_decks, n_rows, row_bytes, P, V, offsets,
                                                          iterations, randomness):
    """Small vblocks travel several per unit; the shuffle is the one-vblock-per-unit plan's and the oracle's."""
    flags = {"uniform": 0, "reference_cuda": _native.FLAG_REFERENCE_RNG,
             "reference_numpy": _native.FLAG_REFERENCE_NUMPY}[randomness]
    host = np.random.default_rng(n_rows + row_bytes).integers(0, 256, size=(n_decks, n_rows, row_bytes), dtype=np.uint8)
    seeds = torch.arange(7, 7 + n_decks, dtype=torch.int64, device=DEV)
    results = []
    try:
        for pack_bytes in (16 * 1024, 0):
            _native.set_pack_bytes(pack_bytes)
            decks = torch.from_numpy(host.copy()).to(DEV)
            plan = _native.describe_plan(decks[0], row_bytes, P, V)
            assert (plan["vblocks_per_unit"] > 1) == (pack_bytes > 0), plan
            if n_decks == 1:
                _native.shuffle_device(decks[0], row_bytes, offsets, iterations, P, V, 7, flags)
            else:
                _native.shuffle_batch(decks, row_bytes, offsets, iterations, P, V, seeds, flags)
            torch.cuda.synchronize()
            povs.check_device_status(0)
            results.append(decks.cpu().numpy())
    finally:
        _native.set_pack_bytes(16 * 1024)
    assert np.array_equal(results[0], results[1])
    for d in range(n_decks):
        want = host[d].copy()
        oracle_api.shuffle(want, iterations, P, V, offsets, 7 + d, randomness)
        assert np.array_equal(results[0][d], want), f"deck {d}"


@pytest.mark.parametrize(
    "n_rows,row_bytes,P,V,offsets,iterations",
    [(1000, 64, 8, 2, list(range(8)), 4), (4099, 256, 32, 4, [0, 1, 2, 5], 3), (20_003, 12, 16, 8, [0, 1, 3], 2),
     (3001, 8, 64, 4, [0, 1, 5], 2), (1200, 12288, 16, 2, [0, 1, 2], 2), (777, 2, 16, 8, [0, 1, 2], 3)],
)
def test_reference_numpy_randomness_mode_matches_oracle(oracle_api, n_rows, row_bytes, P, V, offsets, iterations):
    """randomness="reference_numpy": the library's tables (host MT19937 restatement) against the oracle
    fed tables made by numpy.random.RandomState itself; packed and unpacked units, column slabs,
    truncated last pblocks."""
    host = random_rows(n_rows, row_bytes, seed=13)
    got = gpu_shuffle_bytes(host, P, V, offsets, iterations, 91, flags=_native.FLAG_REFERENCE_NUMPY)
    want = host.copy()
    oracle_api.shuffle(want, iterations, P, V, offsets, 91, "reference_numpy")
    assert np.array_equal(got, want)


def test_reference_modes_exclude_each_other():
    deck = torch.zeros((1000, 16), dtype=torch.uint8, device=DEV)
    with pytest.raises(RuntimeError, match="exclude each other"):
        _native.shuffle_device(deck, 16, [0, 1], 1, 8, 2, 1, _native.FLAG_REFERENCE_RNG | _native.FLAG_REFERENCE_NUMPY)


@pytest.mark.parametrize("row_bytes", [4, 64, 256])
def test_b200_tuned_options_shuffle_like_the_oracle(oracle_api, row_bytes):
    """``tuning="b200"`` picks the pblock for this kernel; the shuffle is still the oracle's."""
    from povs.common import choose_pblock_size_b200

    n_rows = 50_003
    host = random_rows(n_rows, row_bytes, seed=row_bytes)
    deck = torch.from_numpy(host.copy()).to(DEV)
    opts = povs.optim_options_for_dataset(deck, tuning="b200")
    assert opts.physical_block_size == choose_pblock_size_b200(row_bytes, 2, n_rows)
    assert opts.gpu_thread_block_size is not None
    povs.shuffle(deck, iterations=3, options=opts, seed=21)
    torch.cuda.synchronize()
    povs.check_device_status(0)
    want = host.copy()
    oracle_api.shuffle(want, 3, opts.physical_block_size, opts.virtual_block_size, opts.offsets, 21)
    assert np.array_equal(deck.cpu().numpy(), want)


@pytest.mark.parametrize("pinned", [False, True, "interior"])
@pytest.mark.parametrize("row_bytes", [48, 12])
def test_mapped_host_deck_matches_oracle(oracle_api, pinned, row_bytes):
    """A host deck shuffled where it lies (mapped, page-locked for the call or already pinned,
    or a view that starts inside a pinned block)."""
    n, P, V, offsets = 100_003, 32, 4, [0, 1, 2, 5]
    host = random_rows(n, row_bytes, seed=row_bytes + (pinned is True))
    if pinned == "interior":
        buf = torch.empty((n + 7, row_bytes), dtype=torch.uint8, pin_memory=True)
        arr = buf.numpy()[7:]
        arr[...] = host
    elif pinned:
        buf = torch.empty((n, row_bytes), dtype=torch.uint8, pin_memory=True)
        arr = buf.numpy()
        arr[...] = host
    else:
        arr = host.copy()
    povs.shuffle_mapped(arr, iterations=3, options=povs.Options(V, P, offsets), seed=8)
    povs.check_device_status(0)
    want = host.copy()
    oracle_api.shuffle(want, 3, P, V, offsets, 8)
    assert np.array_equal(arr, want)


def test_host_decks_that_do_not_fit_stay_in_host_memory(oracle_api, monkeypatch):
    """povs.shuffle on a host deck switches to the mapped route when the device lacks room; a
    non-contiguous deck is staged through a contiguous copy either way."""
    from povs import _native as native_mod

    calls = []
    real = native_mod.shuffle_mapped
    monkeypatch.setattr(native_mod, "shuffle_mapped", lambda *a, **k: (calls.append(1), real(*a, **k)))
    monkeypatch.setattr(torch.cuda, "mem_get_info", lambda *a, **k: (1 << 20, 1 << 34))
    n, R, P, V, offsets = 20_011, 32, 16, 2, [0, 1, 2]
    host = random_rows(n, 2 * R, seed=4)
    arr = host.copy()
    view = arr[:, :R]  # every other half-row: not C-contiguous
    povs.shuffle(view, iterations=2, options=povs.Options(V, P, offsets), seed=3)
    assert calls, "the mapped route was not taken"
    want = np.ascontiguousarray(host[:, :R])
    oracle_api.shuffle(want, 2, P, V, offsets, 3)
    assert np.array_equal(arr[:, :R], want) and np.array_equal(arr[:, R:], host[:, R:])


def test_randomness_option_selects_the_mode():
    deck = torch.arange(4096 * 4, dtype=torch.float32, device=DEV).view(4096, 4)
    a, b = deck.clone(), deck.clone()
    opts = povs.Options(2, 16, [0, 4], 32)
    povs.shuffle(a, iterations=2, options=opts, seed=5)
    povs.shuffle(b, iterations=2, options=opts._replace(randomness="reference_cuda"), seed=5)
    assert not torch.equal(a, b)
    with pytest.raises(AssertionError):
        povs.shuffle(deck, iterations=1, options=opts._replace(randomness="bogus"), seed=5)


def test_graph_and_direct_launches_agree(oracle_api):
    host = random_rows(20_000, 64, seed=3)
    a = gpu_shuffle_bytes(host, 16, 4, [0, 1, 2, 3], 5, seed=9)
    b = gpu_shuffle_bytes(host, 16, 4, [0, 1, 2, 3], 5, seed=9, flags=_native.FLAG_NO_GRAPH)
    assert np.array_equal(a, b)
    # Chained iterations without programmatic dependent launches (graph and direct).
    for flags in (_native.FLAG_NO_PDL, _native.FLAG_NO_PDL | _native.FLAG_NO_GRAPH):
        assert np.array_equal(a, gpu_shuffle_bytes(host, 16, 4, [0, 1, 2, 3], 5, seed=9, flags=flags))
    want = host.copy()
    oracle_api.shuffle(want, 5, 16, 4, [0, 1, 2, 3], 9)
    assert np.array_equal(a, want)
    c = gpu_shuffle_bytes(host, 16, 4, [0, 1, 2, 3], 5, seed=10)
    assert not np.array_equal(a, c)


def test_back_to_back_calls_on_a_large_deck(oracle_api):
    """Decks of 32 MiB and more launch every iteration chained to the kernel before it on the
    stream, the previous call's last iteration included: two calls in a row and a host-side
    write in between must still see each other's results."""
    n, R, P, V, offsets = 300_007, 128, 32, 4, [0, 1, 2, 3]
    host = random_rows(n, R, seed=17)
    deck = torch.from_numpy(host.copy()).to(DEV)
    assert n * R >= 32 << 20
    _native.shuffle_device(deck, R, offsets, 3, P, V, 5)
    _native.shuffle_device(deck, R, offsets, 2, P, V, 6)
    deck[:1000] = 0  # a torch kernel between two shuffle calls
    _native.shuffle_device(deck, R, offsets, 1, P, V, 7)
    torch.cuda.synchronize()
    povs.check_device_status(0)
    want = host.copy()
    oracle_api.shuffle(want, 3, P, V, offsets, 5)
    oracle_api.shuffle(want, 2, P, V, offsets, 6)
    want[:1000] = 0
    oracle_api.shuffle(want, 1, P, V, offsets, 7)
    assert np.array_equal(deck.cpu().numpy(), want)


def test_misaligned_deck_uses_plain_loads(oracle_api):
    n_rows, row_bytes, P, V, offsets = 3000, 16, 16, 2, [0, 1, 2]
    host = random_rows(n_rows, row_bytes, seed=5)
    buf = torch.zeros(n_rows * row_bytes + 4, dtype=torch.uint8, device=DEV)
    view = buf[4:].view(n_rows, row_bytes)
    view.copy_(torch.from_numpy(host))
    assert view.data_ptr() % 16 == 4
    plan = _native.describe_plan(view, row_bytes, P, V)
    assert plan["bulk"] == 0 and plan["vec_bytes"] == 4
    _native.shuffle_device(view, row_bytes, offsets, 3, P, V, 77)
    torch.cuda.synchronize()
    want = host.copy()
    oracle_api.shuffle(want, 3, P, V, offsets, 77)
    assert np.array_equal(view.cpu().numpy(), want)


# (n_rows, row_bytes, P, V, byte offset of the deck in its buffer): plain loads of whole rows.
ASYNC_PLAIN_CASES = [
    (20_011, 12, 16, 4, 0),   # 12-byte rows: runs agree mod 16 with the stage (bulk middle + 4-byte ends)
    (20_011, 12, 32, 2, 0),
    (9_999, 24, 32, 2, 0),    # 24-byte rows
    (5_003, 20, 64, 2, 0),    # 20-byte rows: runs agree mod 4 only
    (4_000, 64, 16, 2, 4),    # 16-byte multiple rows on a deck 4 bytes past a 16-byte boundary
    (4_000, 48, 8, 4, 8),     # 8 bytes past: 8-byte copies
    (3_000, 4, 128, 2, 0),    # 4-byte rows
    (70_001, 28, 64, 4, 0),   # vblocks too large to pack
]


@pytest.mark.parametrize("n_rows,row_bytes,P,V,shift", ASYNC_PLAIN_CASES)
def test_async_plain_loads_match_synchronous_loads_and_oracle(oracle_api, n_rows, row_bytes, P, V, shift):
    """Rows that are not a 16-byte multiple (or a deck off a 16-byte boundary) are copied into the stages
    asynchronously; the result equals the synchronous plain loads' and the oracle's."""
    offsets = [0, 1, 2, 5]
    host = random_rows(n_rows, row_bytes, seed=n_rows + shift)
    results = []
    try:
        for force_plain in (0, 2):  # 2: plain loads issued synchronously
            assert _native.load().povs_set_tuning_v1(32 * 1024, 8, 4, 4, force_plain, 8192) == 0
            buf = torch.zeros(n_rows * row_bytes + shift, dtype=torch.uint8, device=DEV)
            view = buf[shift:].view(n_rows, row_bytes)
            view.copy_(torch.from_numpy(host))
            plan = _native.describe_plan(view, row_bytes, P, V)
            assert plan["bulk"] == 0
            _native.shuffle_device(view, row_bytes, offsets, 3, P, V, 31)
            torch.cuda.synchronize()
            povs.check_device_status(0)
            results.append(view.cpu().numpy())
    finally:
        _native.set_tuning()
    want = host.copy()
    oracle_api.shuffle(want, 3, P, V, offsets, 31)
    assert np.array_equal(results[1], want), "synchronous plain loads differ from the oracle"
    assert np.array_equal(results[0], want), "asynchronous plain loads differ from the oracle"


def test_plans_cover_bulk_and_slab_paths():
    t = torch.empty((1200, 12288), dtype=torch.uint8, device=DEV)
    plan = _native.describe_plan(t, 12288, 16, 2)
    assert plan["bulk"] == 1 and plan["n_slabs"] > 1
    t2 = torch.empty((4096, 256), dtype=torch.uint8, device=DEV)
    plan2 = _native.describe_plan(t2, 256, 32, 4)
    assert plan2["bulk"] == 1 and plan2["n_slabs"] == 1


def test_injected_numpy_path_matches_reference_golden(golden_numpy_path):
    """Reference NumPy-path randomness injected into the kernels reproduces the reference's output."""
    for case in golden_numpy_path:
        offs, assign, perms = numpy_path.numpy_path_randomness(
            case["seed"], case["n_rows"], case["P"], case["V"], case["offsets"], case["iterations"]
        )
        dev = torch.from_numpy(case["input"].copy()).to(DEV)
        povs.apply_randomness(dev, offs, assign, perms, case["P"], case["V"], sort_members=False)
        povs.check_device_status(0)
        assert np.array_equal(dev.cpu().numpy(), case["output"]), case["name"]


REFCUDA_CASES = [
    (64, (4,), np.float32, 16, 2, [0], 1, 13),  # the reference's standalone program (povs.cu:477-520)
    (128, (8,), np.float32, 16, 2, [4, 8], 3, 42),
    (1000, (16,), np.int32, 8, 2, list(range(8)), 4, 0),
    (1000, (5,), np.uint8, 16, 4, [0, 2, 6], 3, 1),  # truncated last pblock + padding
    (4099, (64,), np.float32, 32, 4, [0, 1, 2, 5], 2, 7),
    (20_000, (3, 16), np.float16, 64, 8, [0, 8, 16 + 3], 2, 999),
]


@pytest.mark.parametrize("n_rows,shape,dtype,P,V,offsets,iterations,seed", REFCUDA_CASES)
def test_injected_refcuda_randomness_matches_oracle(oracle_api, n_rows, shape, dtype, P, V, offsets, iterations, seed):
    rng = np.random.default_rng(seed + 100)
    deck = (rng.standard_normal((n_rows, *shape)) * 50).astype(dtype)
    offs, assign, perms = oracle_api.refcuda_randomness(seed, n_rows, P, V, offsets, iterations)
    want = deck.copy()
    for t in range(iterations):
        oracle_api.apply_iteration(want, P, V, int(offs[t]), assign[t], perms[t], sort_members=True)
    dev = torch.from_numpy(deck.copy()).to(DEV)
    povs.apply_randomness(dev, offs, assign, perms, P, V, sort_members=True)
    povs.check_device_status(0)
    assert np.array_equal(dev.cpu().numpy(), want)


def test_injected_out_of_range_permutation_is_reported():
    n_rows, P, V = 256, 16, 2
    dev = torch.arange(n_rows * 4, dtype=torch.float32, device=DEV).view(n_rows, 4)
    n_p = n_rows // P
    assign = np.arange(n_p, dtype=np.int64).reshape(1, n_p // V, V)
    perms = np.tile(np.arange(V * P, dtype=np.int32), (1, n_p // V, 1))
    perms[0, 3, 5] = 4000
    povs.apply_randomness(dev, [0], assign, perms, P, V, validate=False)
    with pytest.raises(RuntimeError, match="device status 0x2"):
        povs.check_device_status(0)
    povs.check_device_status(0)  # cleared by the read


def _integrity(data: torch.Tensor, n_rows: int, k: int) -> None:
    flat = data.reshape(n_rows, k)
    ids = flat[:, 0].to(torch.int64) // k
    assert torch.equal(torch.sort(ids).values, torch.arange(n_rows, device=data.device)), "deck integrity failed"
    assert not torch.equal(ids, torch.arange(n_rows, device=data.device)), "deck was not shuffled"
    expected = ids[:, None] * k + torch.arange(k, device=data.device)[None, :]
    assert torch.equal(flat.to(torch.int64), expected), "instance integrity failed"


_OPTS_SMALL = povs.Options(physical_block_size=16, virtual_block_size=2, offsets=[4, 8])


@pytest.mark.parametrize("shape", [(8,), (2, 4), (2, 2, 2)])
@pytest.mark.parametrize("iterations", [1, 3])
@pytest.mark.parametrize("opts", [_OPTS_SMALL, None])
@pytest.mark.parametrize("deck", [32, 128])
def test_reference_integrity_cases_on_cuda(deck, shape, iterations, opts):
    """The reference's end-to-end integrity test (src/tests/test_pov_shuffle.py:40-96) on CUDA tensors."""
    k = int(np.prod(shape))
    data = torch.arange(deck * k, dtype=torch.float32, device=DEV).reshape(deck, *shape)
    options = povs.optim_options_for_dataset(data) if opts is None else opts
    povs.shuffle(data, iterations=iterations, options=options, seed=42)
    torch.cuda.synchronize()
    _integrity(data, deck, k)


@pytest.mark.parametrize("container", ["numpy", "cpu"])
@pytest.mark.parametrize("shape", [(8,), (2, 4), (2, 2, 2)])
@pytest.mark.parametrize("iterations", [1, 3])
@pytest.mark.parametrize("opts", [_OPTS_SMALL, None])
@pytest.mark.parametrize("deck", [32, 128])
def test_reference_integrity_cases_host_data(deck, shape, iterations, opts, container):
    """Host decks (NumPy arrays, CPU tensors) go through the GPU and come back shuffled in place."""
    k = int(np.prod(shape))
    flat = np.arange(deck * k, dtype=np.float32).reshape(deck, *shape)
    data = flat if container == "numpy" else torch.from_numpy(flat)
    options = povs.optim_options_for_dataset(data) if opts is None else opts
    povs.shuffle(data, iterations=iterations, options=options, seed=42)
    arr = flat
    ids = arr.reshape(deck, k)[:, 0].astype(np.int64) // k
    assert sorted(ids.tolist()) == list(range(deck))
    assert ids.tolist() != list(range(deck))
    assert np.array_equal(arr.reshape(deck, k), (ids[:, None] * k + np.arange(k)).astype(np.float32))


def test_host_route_matches_device_route():
    host = np.random.default_rng(1).standard_normal((5000, 24)).astype(np.float32)
    opts = povs.Options(virtual_block_size=4, physical_block_size=16, offsets=[0, 1, 2, 3])
    a = host.copy()
    povs.shuffle(a, iterations=3, options=opts, seed=5)
    dev = torch.from_numpy(host.copy()).to(DEV)
    povs.shuffle(dev, iterations=3, options=opts._replace(gpu_thread_block_size=32), seed=5)
    assert np.array_equal(a, dev.cpu().numpy())
    nc = np.asfortranarray(host.copy())
    povs.shuffle(nc, iterations=3, options=opts, seed=5)
    assert np.array_equal(nc, a)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.uint8, torch.float16, torch.float64, torch.int16, torch.bool])
def test_any_dtype_is_shuffled_as_bytes(dtype):
    n_rows, k = 4096, 32
    ids = torch.arange(n_rows, device=DEV)
    data = (ids[:, None] % 2).to(dtype).repeat(1, k) if dtype == torch.bool else ids[:, None].repeat(1, k).to(dtype)
    raw = data.view(torch.uint8).reshape(n_rows, -1).clone()
    povs.shuffle(data, iterations=2, options=None, seed=3)
    torch.cuda.synchronize()
    got = data.view(torch.uint8).reshape(n_rows, -1)
    # Every row survives intact: compare the sorted multisets of rows.
    key = lambda x: torch.unique(x, dim=0, return_counts=True)  # noqa: E731
    a, ca = key(raw)
    b, cb = key(got)
    assert torch.equal(a, b) and torch.equal(ca, cb)


def test_full_size_cfg1_matches_oracle(oracle_api):
    """1,048,576 x 128 fp16 (256 MiB), 4 iterations, V=2, P=64, auto offsets: bit-exact with the oracle."""
    rng = np.random.default_rng(0)
    deck = rng.standard_normal((1_048_576, 128)).astype(np.float16)
    offsets = povs.common.choose_offsets(1_048_576, 128, 2, 64)
    dev = torch.from_numpy(deck).to(DEV)
    povs.shuffle(dev, iterations=4, options=povs.Options(2, 64, offsets, 64), seed=0)
    want = deck.copy()
    oracle_api.shuffle(want, 4, 64, 2, offsets, 0)
    assert np.array_equal(dev.cpu().numpy(), want)


def test_full_size_cfg3_keeps_every_row():
    """134,217,728 x 128 bf16 (32 GiB), 4 iterations, V=4, P=32: every row intact, each exactly once."""
    n_rows, k = 134_217_728, 128
    data = torch.empty((n_rows, k), dtype=torch.bfloat16, device=DEV)
    words = data.view(torch.int64)  # 32 int64 per row
    ids = torch.arange(n_rows, device=DEV, dtype=torch.int64)
    words.copy_((ids[:, None] * 1_000_003 + torch.arange(32, device=DEV)[None, :]))
    offsets = povs.common.choose_offsets(n_rows, k, 2, 32)
    povs.shuffle(data, iterations=4, options=povs.Options(4, 32, offsets, 64), seed=1)
    torch.cuda.synchronize()
    povs.check_device_status(0)
    got_ids = torch.div(words[:, 0], 1_000_003, rounding_mode="floor")
    assert torch.equal(words - got_ids[:, None] * 1_000_003, torch.arange(32, device=DEV).expand(n_rows, 32))
    del words
    assert torch.equal(torch.sort(got_ids).values, ids)
    moved = (got_ids != ids).float().mean().item()
    assert moved > 0.99


def _matches_host_rows(deck: torch.Tensor, want: np.ndarray, chunk_rows: int) -> bool:
    """Compare a device deck with host rows chunk by chunk on the GPU (no second host copy)."""
    rows = deck.view(torch.uint8).reshape(deck.shape[0], -1)
    for s in range(0, rows.shape[0], chunk_rows):
        if not torch.equal(rows[s:s + chunk_rows], torch.from_numpy(want[s:s + chunk_rows]).to(DEV)):
            return False
    return True


@pytest.mark.parametrize(
    "name,n_rows,elems,dtype,P,V,iterations,seed",
    [
        ("bf16 32 GiB", 134_217_728, 128, torch.bfloat16, 32, 4, 4, 1),
        ("uint8 12,288 B rows", 1_000_000, 12_288, torch.uint8, 16, 2, 3, 2),
    ],
)
def test_full_size_decks_match_oracle_byte_for_byte(oracle_api, name, n_rows, elems, dtype, P, V, iterations, seed):
    """The two largest single-GPU decks at full size, byte for byte against the oracle run on every
    host core: 134,217,728 x 128 bf16 (32 GiB, uniform [-1, 1) from seed 1, V=4, P=32, 4 iterations)
    and 1,000,000 x 3x64x64 uint8 (12.3 GB, column slabs, V=2, P=16, 3 iterations).  The host holds
    one copy of the deck, shuffled by the oracle in place; the GPU result is compared chunk by chunk."""
    import os

    g = torch.Generator(device=DEV).manual_seed(seed)
    if dtype == torch.uint8:
        deck = torch.randint(0, 256, (n_rows, elems), generator=g, device=DEV, dtype=torch.uint8)
    else:
        deck = torch.rand((n_rows, elems), generator=g, device=DEV, dtype=dtype) * 2 - 1
    elem_bytes = deck.element_size()
    row_bytes = elems * elem_bytes
    want = deck.view(torch.uint8).reshape(n_rows, row_bytes).cpu().numpy()
    offsets = povs.common.choose_offsets(n_rows, elems, elem_bytes, P)
    povs.shuffle(deck, iterations=iterations, options=povs.Options(V, P, offsets, min(64, V * P)), seed=seed)
    torch.cuda.synchronize()
    povs.check_device_status(0)
    oracle_api.shuffle_threads(want, iterations, P, V, offsets, seed, os.cpu_count() or 1)
    assert _matches_host_rows(deck, want, max(1, (1 << 30) // row_bytes)), f"{name}: differs from the oracle"
    del deck
    torch.cuda.empty_cache()


@pytest.mark.parametrize(
    "rows,row_bytes,P,V,offsets,iterations",
    [
        ([1000, 1500, 2599], 256, 32, 4, [0, 1, 2, 5, 31], 3),
        ([64, 64], 16, 16, 2, [0, 4, 12], 4),
        ([3000, 37, 2000, 999], 24, 16, 8, [0, 1, 2], 2),
        ([300, 500], 12288, 16, 2, [0, 1, 3], 2),
        ([1 << 15] * 8, 128, 64, 4, list(range(16)), 2),
    ],
)
@pytest.mark.parametrize("randomness", ["uniform", "reference_cuda", "reference_numpy"])
@pytest.mark.parametrize("double_buffer", [False, True])
def test_shards_match_the_concatenated_deck(oracle_api, rows, row_bytes, P, V, offsets, iterations, randomness,
                                            double_buffer):
    """A deck split into shards (one process) shuffles exactly like the concatenated deck, in
    place and in the double-buffered order (pblocks pushed to their destination slots)."""
    n = sum(rows)
    host = random_rows(n, row_bytes, seed=n)
    shards, start = [], 0
    for r in rows:
        shards.append(torch.from_numpy(host[start:start + r].copy()).to(DEV))
        start += r
    opts = povs.Options(V, P, offsets, 32, randomness)
    scratch = [torch.full_like(s, 0xA5) for s in shards] if double_buffer else None
    povs.shuffle_shards(shards, iterations=iterations, options=opts, seed=123, scratch=scratch)
    torch.cuda.synchronize()
    povs.check_device_status(0)
    got = torch.cat(shards).cpu().numpy()
    whole = torch.from_numpy(host.copy()).to(DEV)
    povs.shuffle(whole, iterations=iterations, options=opts, seed=123)
    assert np.array_equal(got, whole.cpu().numpy())
    want = host.copy()
    oracle_api.shuffle(want, iterations, P, V, offsets, 123, randomness)
    assert np.array_equal(got, want)


@pytest.mark.parametrize("iterations", [1, 2, 5])
def test_double_buffered_shards_one_shard(oracle_api, iterations):
    """One shard in the double-buffered order: odd iteration counts end with the copy back."""
    n, row_bytes, P, V, offsets = 100_003, 64, 32, 4, [0, 3, 7, 31]
    host = random_rows(n, row_bytes, seed=9)
    deck = torch.from_numpy(host.copy()).to(DEV)
    scratch = torch.empty_like(deck)
    povs.shuffle_shards([deck], iterations=iterations, options=povs.Options(V, P, offsets, 32), seed=77,
                        scratch=[scratch])
    torch.cuda.synchronize()
    povs.check_device_status(0)
    want = host.copy()
    oracle_api.shuffle(want, iterations, P, V, offsets, 77)
    assert np.array_equal(deck.cpu().numpy(), want)


def test_shards_smaller_than_a_pblock_are_rejected():
    shards = [torch.zeros((8, 4), device=DEV), torch.zeros((100, 4), device=DEV)]
    with pytest.raises(AssertionError, match="at least physical_block_size"):
        povs.shuffle_shards(shards, iterations=1, options=povs.Options(2, 16, [0, 4], 32), seed=1)


def test_host_batch_repeated_decks_with_three_buffers(oracle_api):
    """Host decks A, B, A, C, A through three device buffers: each listing of A starts from the
    previous listing's result (its copy in waits for that copy back), whichever buffer it uses."""
    n, R, P, V, offsets = 30_011, 32, 16, 4, [0, 1, 2]
    pins = [torch.empty((n, R), dtype=torch.uint8, pin_memory=True) for _ in range(3)]
    originals = [random_rows(n, R, seed=60 + i) for i in range(3)]
    for t, o in zip(pins, originals):
        t.numpy()[...] = o
    order = [0, 1, 0, 2, 0]
    seeds = [11, 12, 13, 14, 15]
    buffers = [torch.empty(n * R, dtype=torch.uint8, device=DEV) for _ in range(3)]
    _native.shuffle_host_batch([pins[i].data_ptr() for i in order], buffers, n, R, offsets, 2, P, V, seeds)
    want = [o.copy() for o in originals]
    for i, sd in zip(order, seeds):
        oracle_api.shuffle(want[i], 2, P, V, offsets, sd)
    for t, w in zip(pins, want):
        assert np.array_equal(t.numpy(), w)


@pytest.mark.parametrize("free_bytes", [None, 1 << 20])
def test_shuffle_many_strided_deck_listed_twice(oracle_api, monkeypatch, free_bytes):
    """A non-contiguous deck listed twice is shuffled twice in order, through device buffers or,
    when the device has no room (``free_bytes``), in host memory."""
    if free_bytes is not None:
        monkeypatch.setattr(torch.cuda, "mem_get_info", lambda *a, **k: (free_bytes, 1 << 34))
    n, R, P, V, offsets = 12_007, 16, 16, 2, [0, 1, 2]
    base = random_rows(n, 2 * R, seed=31)
    whole = base.copy()
    strided = whole[:, R:]
    other = random_rows(n, R, seed=32)
    other_copy = other.copy()
    povs.shuffle_many([strided, other, strided], iterations=2, options=povs.Options(V, P, offsets), seed=40)
    want = np.ascontiguousarray(base[:, R:])
    oracle_api.shuffle(want, 2, P, V, offsets, 40)
    oracle_api.shuffle(want, 2, P, V, offsets, 42)
    assert np.array_equal(whole[:, R:], want) and np.array_equal(whole[:, :R], base[:, :R])
    oracle_api.shuffle(other_copy, 2, P, V, offsets, 41)
    assert np.array_equal(other, other_copy)


def test_shuffle_many_matches_one_deck_at_a_time():
    """Pipelined host decks: deck d gets seed + d, exactly like separate host-route calls."""
    rng = np.random.default_rng(4)
    decks = [rng.standard_normal((20_000, 24)).astype(np.float32) for _ in range(3)]
    expected = [d.copy() for d in decks]
    opts = povs.Options(virtual_block_size=4, physical_block_size=16, offsets=[0, 1, 2, 3])
    for i, e in enumerate(expected):
        povs.shuffle(e, iterations=3, options=opts, seed=50 + i)
    povs.shuffle_many(decks, iterations=3, options=opts, seed=50)
    for d, e in zip(decks, expected):
        assert np.array_equal(d, e)
    # The same deck twice: shuffled again after its first copy back.
    again = rng.standard_normal((20_000, 24)).astype(np.float32)
    twice = again.copy()
    povs.shuffle(twice, iterations=2, options=opts, seed=7)
    povs.shuffle(twice, iterations=2, options=opts, seed=8)
    povs.shuffle_many([again, again], iterations=2, options=opts, seed=7)
    assert np.array_equal(again, twice)
