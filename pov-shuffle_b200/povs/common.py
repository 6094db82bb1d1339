"""Option logic shared by the GPU and CPU-data routes.

Same functions, arguments and error behaviour (``AssertionError`` for invalid options) as the
reference's src/povs/common.py:23-193, so callers and the reference's option tests work
unchanged.  The offset rules are the reference's: an offset is valid when it is below the deck
size, zero or not a multiple of the pblock size, and keeps pblock starts aligned to
``MIN_MEM_ALIGNMENT_BITS`` (common.py:94-129).
"""

from __future__ import annotations

import json
import math
import warnings
from importlib.resources import files

import numpy as np
import torch

from .constants import (
    MAX_MEM_ALIGNMENT_BITS,
    MAX_SEED,
    MIN_MEM_ALIGNMENT_BITS,
    MIN_OFFSETS,
    MIN_PBLOCK_SIZE,
    MIN_SEED,
    MIN_VBLOCK_SIZE,
    REFERENCE_MAX_SEED,
)
from .types import BuildParams, Options
from .utils import is_power_of_2, least_factor_to_make_multiple, round_down_to_power_of_2


def get_build_params() -> BuildParams:
    """Return the build-time parameters of the native library (written by the in-tree build)."""
    data = json.loads(files("povs").joinpath("build_params.json").read_text())
    return BuildParams(**data)


def get_int_seed(seed: int | np.random.Generator | torch.Generator | None, options: Options | None = None) -> int:
    """Normalise a seed: ints pass through, generators (or None -> fresh entropy) draw one integer,
    from [1, 2**63 - 1), or from the reference's [1, 1000) (common.py:29-42 there) when ``options``
    ask for one of the reference's distributions (``randomness="reference_cuda"`` or
    ``"reference_numpy"``)."""
    if isinstance(seed, (int, np.integer)) and not isinstance(seed, bool):
        return int(seed)
    high = REFERENCE_MAX_SEED if options is not None and options.randomness in REFERENCE_MODES else MAX_SEED
    if seed is None:
        seed = np.random.default_rng()
    if isinstance(seed, np.random.Generator):
        return int(seed.integers(MIN_SEED, high, dtype=np.int64))
    if isinstance(seed, torch.Generator):
        return int(torch.randint(MIN_SEED, high, (1,), generator=seed, dtype=torch.int64).item())
    raise TypeError(f"Unsupported seed type: {type(seed)}")


def seed_to_u64(seed: int) -> int:
    """Map any Python int seed to the 64-bit key of the device RNG."""
    return int(seed) & 0xFFFF_FFFF_FFFF_FFFF


RANDOMNESS_MODES = ("uniform", "reference_cuda", "reference_numpy")
REFERENCE_MODES = ("reference_cuda", "reference_numpy")


def randomness_flags(options: Options) -> int:
    """Native flags selecting the randomness mode of ``options`` (AssertionError if unknown)."""
    mode = options.randomness or "uniform"
    assert mode in RANDOMNESS_MODES, f"randomness ({mode!r}) must be one of {RANDOMNESS_MODES}"
    return {"uniform": 0, "reference_cuda": 4, "reference_numpy": 16}[mode]


def get_dtype_bytes(dataset: np.ndarray | torch.Tensor) -> int:
    return dataset.element_size() if isinstance(dataset, torch.Tensor) else dataset.itemsize


def get_instance_size(dataset: np.ndarray | torch.Tensor) -> int:
    """Elements per instance: the product of dimensions 1.. (1 for a 1-D dataset)."""
    if dataset.ndim <= 1:
        return 1
    return int(math.prod(dataset.shape[1:]))


def get_instance_bytes(dataset: np.ndarray | torch.Tensor) -> int:
    return get_instance_size(dataset) * get_dtype_bytes(dataset)


def purge_dependent_param(options: Options, upstream: str, dependent: str) -> Options:
    warnings.warn(f"Param `{upstream}` is not specified, ignoring specification of dependent param {dependent}")
    return options._replace(**{dependent: None})


def povs_preflight(data: np.ndarray | torch.Tensor, iterations: int, options: Options) -> None:
    """Validations common to every route."""
    assert data.ndim >= 1, f"dataset must have at least one dimension, but has {data.ndim}"
    deck_size = data.shape[0]
    assert deck_size >= 2, f"dataset must have at least 2 instances, but has {deck_size}"
    assert iterations >= 1, f"iterations ({iterations}) must be at least 1"
    _validate_vblock_size(options.virtual_block_size)
    pblock = _validate_pblock_size(options.physical_block_size)
    _validate_offsets(
        options.offsets,
        deck_size=deck_size,
        instance_size=get_instance_size(data),
        dtype_bytes=get_dtype_bytes(data),
        pblock_size=pblock,
    )


def _validate_vblock_size(vblock_size: int | None) -> int:
    assert vblock_size is not None, "vblock size must be specified"
    assert is_power_of_2(vblock_size), f"vblock size ({vblock_size}) must be a power of 2"
    assert vblock_size >= MIN_VBLOCK_SIZE, f"vblock size ({vblock_size}) must be at least {MIN_VBLOCK_SIZE}"
    return vblock_size


def _validate_pblock_size(pblock_size: int | None) -> int:
    assert pblock_size is not None, "pblock size must be specified"
    assert is_power_of_2(pblock_size), f"pblock size ({pblock_size}) must be a power of 2"
    assert pblock_size >= MIN_PBLOCK_SIZE, f"pblock size ({pblock_size}) must be at least {MIN_PBLOCK_SIZE}"
    return pblock_size


def _validate_offsets(
    offsets: list[int] | None,
    deck_size: int,
    instance_size: int,
    dtype_bytes: int,
    pblock_size: int,
) -> None:
    assert offsets is not None, "offsets must be specified"
    assert len(offsets) >= MIN_OFFSETS, f"at least {MIN_OFFSETS} offsets must be specified"
    instance_bits = instance_size * dtype_bytes * 8
    for i, offset in enumerate(offsets):
        below_deck, not_pblock_multiple, aligned = _offset_is_valid(offset, deck_size, instance_bits, pblock_size)
        what = f"offset at index {i} ({offset})"
        assert offset >= 0, f"{what} must be non-negative"
        assert below_deck, f"{what} must be less than deck size {deck_size}"
        assert not_pblock_multiple, f"{what} must be zero or not divisible by pblock size {pblock_size}"
        assert aligned, (
            f"{what} * instance_bits ({instance_bits}) must be a multiple of the minimum memory alignment "
            f"({MIN_MEM_ALIGNMENT_BITS}bits)"
        )


def _offset_is_valid(offset: int, deck_size: int, instance_bits: int, pblock_size: int) -> tuple[bool, bool, bool]:
    return (
        offset < deck_size,
        offset == 0 or offset % pblock_size != 0,
        (offset * instance_bits) % MIN_MEM_ALIGNMENT_BITS == 0,
    )


def get_block_counts(deck_size: int, physical_block_size: int, virtual_block_size: int, **__) -> tuple[int, int]:
    """Number of physical and virtual blocks, rounding up."""
    n_pblocks = -(-deck_size // physical_block_size)
    n_vblocks = -(-n_pblocks // virtual_block_size)
    return n_pblocks, n_vblocks


def choose_offsets(
    deck_size: int,
    instance_size: int,
    dtype_bytes: int,
    pblock_size: int,
    max_offsets: int | None = 16,
) -> list[int]:
    """Offsets for ``Options``: multiples of an aligned base offset with pairwise distinct residues mod P."""
    assert max_offsets is None or max_offsets >= MIN_OFFSETS
    limit = max_offsets or MIN_OFFSETS
    base = _choose_base_offset(instance_size * dtype_bytes * 8, pblock_size, deck_size)
    chosen: list[int] = []
    residues: set[int] = set()
    for k in range(limit):
        off = k * base
        if off >= deck_size:
            break
        res = off % pblock_size if off else 0
        if res in residues:
            continue
        residues.add(res)
        chosen.append(off)
    return chosen


def _choose_base_offset(
    instance_bits: int,
    pblock_size: int,
    deck_size: int,
    alignment: int = MAX_MEM_ALIGNMENT_BITS,
) -> int:
    """Smallest aligned multiple of the instance size, relaxing alignment (128 -> 16 bits) until usable."""
    while True:
        base = least_factor_to_make_multiple(instance_bits, alignment)
        if base % pblock_size != 0 and base < deck_size:
            return base
        if alignment <= MIN_MEM_ALIGNMENT_BITS:
            raise ValueError(
                "Cannot find a memory-aligned base offset that is less than the dataset size and not a multiple "
                "of the physical block size"
            )
        alignment //= 2


# B200 option tuning (``tuning="b200"``): the iteration kernel stages one vblock (V * P rows) per
# unit in shared memory, or several small vblocks per unit (packed units).  Measured on B200 (GB/s
# of 2 x deck bytes per iteration, V = 2, 2 GiB decks, a sweep of P for every row size): rows of
# 96 B and more stream best in vblocks of 32-64 KiB (5.7-6.2 TB/s) and at most 512 rows; rows of
# 2 KiB and more are staged as 2 KiB column slabs of 32 rows (6.1-6.2 TB/s).  Rows under 96 B
# travel in packed units; their best vblock lengths, which balance the sort network per key
# against the fixed costs per unit and member, were 256 rows below 16 B (4 B: 997 GB/s, 8 B:
# 2014, 12 B: 2288), 128 below 20 B (16 B: 4956), 256 below 40 B (20 B: 2839,
# 24 B: 3874, 28 B: 4298, 32 B: 5649), 1024 below 48 B (40 B: 4183), 128 below 64 B (48 B: 5353,
# 56 B: 5169), 256 below 80 B (64 B: 5936) and 512 below 96 B (80 B: 5864).
B200_VBLOCK_BYTES = 64 * 1024
B200_MAX_VBLOCK_ROWS = 512
B200_WIDE_ROW_BYTES = 2048
B200_WIDE_VBLOCK_ROWS = 32
B200_SMALL_ROW_VBLOCK_ROWS = ((16, 256), (20, 128), (40, 256), (48, 1024), (64, 128), (80, 256),
                              (96, 512))  # (row bytes below, vblock rows)


def choose_pblock_size_b200(row_bytes: int, vblock_size: int, deck_size: int) -> int:
    """Physical block size for the B200 kernel: the largest power of two that keeps a vblock within
    64 KiB and 512 rows (32 rows for rows of 2 KiB and more; the measured best length, 128 to 1024
    rows, for rows under 96 bytes, which travel in packed units), at least ``MIN_PBLOCK_SIZE``, and
    at most what leaves the deck two vblocks."""
    if row_bytes >= B200_WIDE_ROW_BYTES:
        rows = B200_WIDE_VBLOCK_ROWS
    else:
        rows = min(B200_MAX_VBLOCK_ROWS, B200_VBLOCK_BYTES // max(1, row_bytes))
        for below, small_rows in B200_SMALL_ROW_VBLOCK_ROWS:
            if row_bytes < below:
                rows = small_rows
                break
    pblock = max(MIN_PBLOCK_SIZE, round_down_to_power_of_2(max(1, rows // vblock_size)))
    room = deck_size // (2 * vblock_size)
    if room >= MIN_PBLOCK_SIZE:
        pblock = min(pblock, round_down_to_power_of_2(room))
    return max(MIN_PBLOCK_SIZE, pblock)


TUNINGS = ("reference", "b200")
