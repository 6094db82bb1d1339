"""Option logic: the reference's option tests (src/tests/test_choose_*.py, test_utils.py) against
this package, plus the P = 8 extension."""

from __future__ import annotations

from dataclasses import dataclass
from itertools import product
from types import SimpleNamespace
from unittest.mock import patch

import numpy as np
import povs
import pytest

from povs.common import (
    _validate_offsets,
    _validate_pblock_size,
    _validate_vblock_size,
    choose_offsets,
    get_block_counts,
    get_int_seed,
)
from povs.torch import _choose_pblock_size, _choose_thr_block_size, _validate_thr_block_size
from povs.utils import is_power_of_2, least_factor_to_make_multiple, round_down_to_power_of_2


@pytest.mark.parametrize(
    "deck,inst,dbytes,pblock,max_offsets",
    list(product([16, 32], [1, 2, 4], [16, 32, 64], [16, 32, 64], [None, 2, 4])),
)
def test_choose_offsets_valid(deck, inst, dbytes, pblock, max_offsets):
    _validate_pblock_size(pblock)
    offsets = choose_offsets(deck, inst, dbytes, pblock, max_offsets)
    _validate_offsets(offsets, deck, inst, dbytes, pblock)


@pytest.mark.parametrize("dbytes", [1, 2, 4, 8])
@pytest.mark.parametrize("inst", [1, 2, 3, 16])
def test_choose_offsets_pblock8(dbytes, inst):
    offsets = choose_offsets(1000, inst, dbytes, 8)
    _validate_offsets(offsets, 1000, inst, dbytes, 8)
    assert len(offsets) >= 2


def test_choose_offsets_known_values():
    # Rows of a multiple of 128 bits: base offset 1, residues 0..P-1 (at most 16 offsets).
    assert choose_offsets(1_048_576, 128, 2, 64) == list(range(16))
    assert choose_offsets(1000, 16, 4, 8) == list(range(8))
    # 8-bit rows, P = 16: 128-bit base 16 is a pblock multiple, 64-bit base 8 is not.
    assert choose_offsets(32, 1, 1, 16) == [0, 8]


@dataclass(frozen=True)
class _PblockCase:
    instance_size: int
    dtype_bytes: int
    vblock_size: int
    sm_smem_bytes: int
    major: int
    minor: int


@pytest.mark.parametrize(
    "case",
    [
        _PblockCase(1, 4, 2, 73728, 9, 0),
        _PblockCase(1, 4, 2, 55296, 9, 0),
        _PblockCase(1, 4, 2, 41472, 9, 0),
        _PblockCase(1, 4, 2, 18432, 9, 0),
        _PblockCase(1, 4, 2, 36864, 8, 0),
        _PblockCase(2, 4, 2, 61440, 99, 0),
        _PblockCase(128, 2, 4, 233472, 10, 0),
        _PblockCase(32, 4, 4, 233472, 10, 0),
    ],
)
def test_choose_pblock_size(case):
    dev = SimpleNamespace(major=case.major, minor=case.minor, shared_memory_per_multiprocessor=case.sm_smem_bytes)
    _validate_vblock_size(case.vblock_size)
    with patch("povs.torch.torch.cuda.get_device_properties", return_value=dev):
        pblock = _choose_pblock_size(case.instance_size, case.dtype_bytes, case.vblock_size, device_id=0)
    _validate_pblock_size(pblock)


def test_choose_pblock_size_known_values():
    # Arithmetic of the reference's comments: 73728 // 36 = 2048 instances/SM, 32 CTAs -> 64 per CTA -> P = 32.
    dev = SimpleNamespace(major=9, minor=0, shared_memory_per_multiprocessor=73728)
    with patch("povs.torch.torch.cuda.get_device_properties", return_value=dev):
        assert _choose_pblock_size(1, 4, 2, device_id=0) == 32
    # 1536 instances/SM -> P = 24 -> upper (32) is closer to 32 CTAs/SM.
    dev = SimpleNamespace(major=9, minor=0, shared_memory_per_multiprocessor=55296)
    with patch("povs.torch.torch.cuda.get_device_properties", return_value=dev):
        assert _choose_pblock_size(1, 4, 2, device_id=0) == 32
    # 1152 instances/SM -> P = 18 -> lower (16) wins.
    dev = SimpleNamespace(major=9, minor=0, shared_memory_per_multiprocessor=41472)
    with patch("povs.torch.torch.cuda.get_device_properties", return_value=dev):
        assert _choose_pblock_size(1, 4, 2, device_id=0) == 16


@pytest.mark.parametrize(
    "inst,dbytes,V,P,smem,threads,major,minor",
    [
        (1, 4, 4, 32, 147456, 2048, 9, 0),
        (1, 4, 2, 16, 73728, 2048, 9, 0),
        (1, 4, 2, 32, 73728, 1536, 9, 0),
        (1, 4, 2, 32, 73728, 768, 9, 0),
        (1, 4, 2, 32, 73728, 512, 9, 0),
        (1, 4, 2, 32, 36864, 2048, 8, 0),
        (128, 2, 4, 32, 233472, 2048, 10, 0),
    ],
)
def test_choose_thr_block_size(inst, dbytes, V, P, smem, threads, major, minor):
    dev = SimpleNamespace(
        shared_memory_per_multiprocessor=smem, max_threads_per_multi_processor=threads, major=major, minor=minor
    )
    with patch("povs.torch.torch.cuda.get_device_properties", return_value=dev):
        size = _choose_thr_block_size(inst, dbytes, V, P, device_id=0)
    _validate_thr_block_size(size, V, P)


@pytest.mark.parametrize("x,expected", [(1, True), (2, True), (4, True), (1024, True), (0, False), (-1, False), (3, False), (6, False)])
def test_is_power_of_2(x, expected):
    assert is_power_of_2(x) == expected


@pytest.mark.parametrize("x,expected", [(1, 1), (2, 2), (3, 2), (4, 4), (7, 4), (8, 8), (9, 8)])
def test_round_down_to_power_of_2(x, expected):
    assert round_down_to_power_of_2(x) == expected


@pytest.mark.parametrize("x,y,expected", [(1, 6, 6), (6, 6, 1), (3, 6, 2), (6, 3, 1), (4, 6, 3), (3, 4, 4), (1, 1, 1)])
def test_least_factor_to_make_multiple(x, y, expected):
    k = least_factor_to_make_multiple(x, y)
    assert k == expected and (k * x) % y == 0


def test_block_counts():
    assert get_block_counts(1_048_576, 64, 2) == (16384, 8192)
    assert get_block_counts(1000, 8, 2) == (125, 63)
    assert get_block_counts(134_217_728, 32, 4) == (4_194_304, 1_048_576)
    assert get_block_counts(1_000_000, 16, 2) == (62_500, 31_250)


@pytest.mark.parametrize("bad", [dict(virtual_block_size=3), dict(virtual_block_size=1), dict(physical_block_size=12), dict(physical_block_size=4)])
def test_invalid_sizes_raise(bad):
    if "virtual_block_size" in bad:
        with pytest.raises(AssertionError):
            _validate_vblock_size(bad["virtual_block_size"])
    else:
        with pytest.raises(AssertionError):
            _validate_pblock_size(bad["physical_block_size"])


@pytest.mark.parametrize(
    "offsets,msg",
    [([0], "at least"), ([0, 64], "less than deck"), ([0, 16], "not divisible"), ([0, 3], "alignment")],
)
def test_invalid_offsets_raise(offsets, msg):
    # deck 64 rows of 1 x uint8 (8 bits), P = 16: offset 3 gives 24 bits, not a 16-bit multiple.
    with pytest.raises(AssertionError, match=msg):
        _validate_offsets(offsets, deck_size=64, instance_size=1, dtype_bytes=1, pblock_size=16)


def test_seed_normalisation():
    import torch

    assert get_int_seed(5) == 5
    assert get_int_seed(np.int64(9)) == 9
    g = np.random.default_rng(0)
    s = get_int_seed(g)
    assert 1 <= s < 2**63
    assert get_int_seed(np.random.default_rng(0)) == s
    tg = torch.Generator().manual_seed(3)
    assert 1 <= get_int_seed(tg) < 2**63
    assert isinstance(get_int_seed(None), int)
    with pytest.raises(TypeError):
        get_int_seed("seed")


def test_thread_block_hint_for_small_vblocks():
    """V * P below 32 (P = 8) is accepted with the minimum hint; larger hints are still rejected."""
    _validate_thr_block_size(32, 2, 8)
    with pytest.raises(AssertionError, match="must not exceed total instances"):
        _validate_thr_block_size(64, 2, 8)
    with pytest.raises(AssertionError, match="must not exceed total instances"):
        _validate_thr_block_size(128, 4, 16)


@pytest.mark.parametrize(
    "row_bytes,V,deck,expected",
    [
        (256, 2, 1 << 30, 128),   # 64 KiB vblocks
        (256, 4, 1 << 30, 64),
        (128, 2, 1 << 30, 256),   # 512 rows
        (96, 2, 1 << 30, 256),
        (64, 2, 1 << 30, 128),    # measured best vblock lengths for small rows (packed units)
        (80, 2, 1 << 30, 256),
        (56, 2, 1 << 30, 64),
        (48, 2, 1 << 30, 64),
        (40, 2, 1 << 30, 512),
        (20, 2, 1 << 30, 128),
        (32, 4, 1 << 30, 64),
        (24, 2, 1 << 30, 128),
        (16, 2, 1 << 30, 64),
        (12, 2, 1 << 30, 128),
        (8, 2, 1 << 30, 128),
        (4, 2, 1 << 30, 128),
        (4, 4, 1 << 30, 64),
        (1024, 4, 1 << 30, 16),
        (12288, 2, 1 << 30, 16),  # wide rows: 32-row vblocks of 2 KiB slabs
        (12288, 4, 1 << 30, 8),
        (256, 32, 1 << 30, 8),    # never below the minimum pblock
        (256, 2, 1000, 128),      # at least two vblocks' worth of pblocks in a small deck
    ],
)
def test_b200_pblock_choice(row_bytes, V, deck, expected):
    from povs.common import choose_pblock_size_b200

    assert choose_pblock_size_b200(row_bytes, V, deck) == expected


def test_tuning_option_on_host_decks():
    deck = np.zeros((100_000, 64), dtype=np.float32)
    ref = povs.optim_options_for_dataset(deck)
    b200 = povs.optim_options_for_dataset(deck, tuning="b200")
    assert ref.physical_block_size == 16 and b200.physical_block_size == 128  # 256-byte rows: 64 KiB vblocks
    assert b200.offsets == list(range(16)) and b200.virtual_block_size == 2
    given = povs.optim_options_for_dataset(deck, povs.Options(physical_block_size=32), tuning="b200")
    assert given.physical_block_size == 32
    with pytest.raises(AssertionError, match="tuning"):
        povs.optim_options_for_dataset(deck, tuning="fast")


def test_generator_seeds_follow_the_randomness_mode():
    """A generator seed is a 63-bit draw for the uniform mode and the reference's [1, 1000) draw when
    the options ask for the reference CUDA path's distribution (its common.py:29-42)."""
    import numpy as np
    import torch

    from povs.common import get_int_seed
    from povs.types import Options

    ref = Options(randomness="reference_cuda")
    draws = [get_int_seed(np.random.default_rng(s), ref) for s in range(200)]
    assert all(1 <= d < 1000 for d in draws)
    assert draws[:5] == [int(np.random.default_rng(s).integers(1, 1000, dtype=np.int64)) for s in range(5)]
    g = torch.Generator().manual_seed(3)
    assert 1 <= get_int_seed(g, ref) < 1000
    wide = [get_int_seed(np.random.default_rng(s), Options()) for s in range(50)]
    assert max(wide) > 1000
    assert get_int_seed(12345, ref) == 12345
