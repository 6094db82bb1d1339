"""CPU checks that pin the oracle before the GPU parity tests compare the library against it."""

from __future__ import annotations

import numpy as np
import pytest

from oracle import numpy_path

# Random123 known-answer vectors for philox4x32 with 10 rounds: (counter, key) -> output.
PHILOX_KAT = [
    ((0, 0, 0, 0), (0, 0), (0x6627E8D5, 0xE169C58D, 0xBC57AC4C, 0x9B00DBD8)),
    ((0xFFFFFFFF,) * 4, (0xFFFFFFFF, 0xFFFFFFFF), (0x408F276D, 0x41C83B0E, 0xA20BC7C6, 0x6D5451FD)),
    (
        (0x243F6A88, 0x85A308D3, 0x13198A2E, 0x03707344),
        (0xA4093822, 0x299F31D0),
        (0xD16CFE09, 0x94FDCCEB, 0x5001E420, 0x24126EA1),
    ),
]


@pytest.mark.parametrize("ctr,key,expected", PHILOX_KAT)
def test_philox_known_answers(oracle_api, ctr, key, expected):
    assert oracle_api.philox(ctr, key) == expected


def test_golden_numpy_path_through_oracle(oracle_api, golden_numpy_path):
    """Replayed NumPy-path randomness + the oracle's iteration == the reference's own output."""
    assert len(golden_numpy_path) >= 10
    for case in golden_numpy_path:
        offs, assign, perms = numpy_path.numpy_path_randomness(
            case["seed"], case["n_rows"], case["P"], case["V"], case["offsets"], case["iterations"]
        )
        deck = case["input"].copy()
        for t in range(case["iterations"]):
            oracle_api.apply_iteration(deck, case["P"], case["V"], int(offs[t]), assign[t], perms[t], sort_members=False)
        assert np.array_equal(deck, case["output"]), case["name"]


@pytest.mark.parametrize(
    "n_rows,P,V,n_offsets,iterations",
    [(64, 16, 2, 2, 3), (1000, 8, 2, 8, 5), (5000, 16, 4, 16, 4), (77, 16, 2, 2, 6), (4099, 32, 8, 5, 2)],
)
@pytest.mark.parametrize("seed", [0, 1, 13, 999])
def test_refcuda_assignment_matches_reference_code(oracle_api, n_rows, P, V, n_offsets, iterations, seed):
    """The C++ restatement's assignment sequence == the reference's compiled shuffle_array."""
    ref = oracle_api.ref_assign_sequence(seed, n_rows, P, V, n_offsets, iterations)
    if ref is None:
        pytest.skip("reference helper (oracle/_ref) not built: no reference checkout")
    ref_assign, ref_idx = ref
    offsets = list(range(100, 100 + n_offsets))
    offs, assign, _ = oracle_api.refcuda_randomness(seed, n_rows, P, V, offsets, iterations)
    assert np.array_equal(assign, ref_assign)
    assert np.array_equal(offs, np.array(offsets)[ref_idx])


def test_refcuda_permutations_are_gap_free(oracle_api):
    n_rows, P, V = 1000, 16, 4  # truncated last pblock (8 rows) and one padding slot
    offs, assign, perms = oracle_api.refcuda_randomness(5, n_rows, P, V, [0, 2, 6], 3)
    n_p = -(-n_rows // P)
    for t in range(3):
        for v in range(assign.shape[1]):
            rows = sum(min(P, n_rows - b * P) for b in assign[t, v] if b >= 0)
            assert sorted(perms[t, v, :rows]) == list(range(rows))
            assert (perms[t, v, rows:] == -1).all()
        assert sorted(b for b in assign[t].ravel() if b >= 0) == list(range(n_p))


@pytest.mark.parametrize("n_slots", [2, 3, 4, 5, 17, 64, 100, 1000, 4097, 65536])
@pytest.mark.parametrize("seed", [0, 7, 2**40 + 3])
def test_device_assignment_is_bijection(oracle_api, n_slots, seed):
    for it in range(3):
        a = oracle_api.assignment(seed, it, n_slots)
        assert np.array_equal(np.sort(a), np.arange(n_slots))


@pytest.mark.parametrize(
    "n_rows,row_shape,dtype,P,V,offsets,iterations",
    [
        (64, (4,), np.float32, 16, 2, [0, 4], 1),
        (1000, (16,), np.int32, 8, 2, list(range(8)), 4),
        (1001, (3,), np.int32, 16, 4, [0, 1, 3], 3),
        (37, (1,), np.uint8, 8, 2, [0, 2, 4, 6], 5),
    ],
)
def test_oracle_shuffle_is_a_row_permutation(oracle_api, n_rows, row_shape, dtype, P, V, offsets, iterations):
    k = int(np.prod(row_shape))
    ids = np.arange(n_rows, dtype=np.int64)
    deck = (ids[:, None] * k + np.arange(k)[None, :]).astype(dtype).reshape(n_rows, *row_shape)
    before = deck.copy()
    oracle_api.shuffle(deck, iterations, P, V, offsets, seed=123)
    flat = deck.reshape(n_rows, k)
    src = flat[:, 0].astype(np.int64) // k if dtype != np.uint8 else None
    if src is not None:
        assert sorted(src.tolist()) == list(range(n_rows))
        assert np.array_equal(flat, before.reshape(n_rows, k)[src])
        assert not np.array_equal(src, ids)
    else:
        assert sorted(flat[:, 0].tolist()) == sorted(before.reshape(n_rows, k)[:, 0].tolist())


def test_oracle_rejects_out_of_range_permutation(oracle_api):
    deck = np.arange(64, dtype=np.float32).reshape(32, 2)
    P, V = 8, 2
    assign = np.array([[0, 1], [2, 3]], dtype=np.int64)
    perms = np.tile(np.arange(16, dtype=np.int32), (2, 1))
    perms[1, 3] = 99
    with pytest.raises(ValueError):
        oracle_api.apply_iteration(deck, P, V, 0, assign, perms, sort_members=True)


def test_numpy_replay_flags_reference_row_loss():
    """N % P != 0 with V = 4: the reference's NumPy path loses rows; the replay must refuse it."""
    with pytest.raises(numpy_path.CorruptingDraw):
        numpy_path.numpy_path_randomness(0, 1000, 16, 4, [0, 2, 6], 3)


def test_numpy_replay_padding_before_member_is_identity():
    """V = 2 with the padding id first: the reference leaves that member's rows untouched."""
    src = numpy_path._effective_vblock_perm([10**6, 3], n_rows=64, pblock=16, p=np.arange(16)[::-1].copy())
    assert np.array_equal(src, np.arange(16))


def test_reference_cuda_library_shapes_stay_in_bounds(oracle_api):
    """The reference's CUDA path compiled into oracle/_ref (no GPU needed to load it or run the host
    check): every instantiated shape's Stage 1 copy partition stays inside the pblock, while the
    options the reference's chooser picks for 32-byte float rows on a B200 do not."""
    lib = oracle_api.ref_cuda_lib()
    if lib is None:
        pytest.skip("oracle/_ref/libref_povs_cuda.so is not built (needs the reference checkout)")
    shapes = oracle_api.ref_cuda_shapes()
    assert len(shapes) >= 8
    assert {(s["V"], s["P"], s["row_bytes"]) for s in shapes} >= {(2, 64, 256), (4, 32, 256), (4, 64, 128)}
    for s in shapes:
        assert lib.ref_povs_layout_check(s["index"]) == 0, s
        assert s["inst"] % s["block"] == 0
    assert lib.ref_povs_layout_check_small_rows() != 0
    assert lib.ref_povs_layout_check(len(shapes)) == -1
