"""POV shuffle for host data (NumPy arrays and CPU tensors).

The reference runs a pseudo-parallel NumPy version of the algorithm on the CPU for these inputs
(src/povs/numpy.py:18-61).  Here host data takes the same GPU path as CUDA tensors: the rows are
copied to a device staging buffer, shuffled by the sm_100a kernels and copied back, in one native
call (``povs_shuffle_host_v1``).  Option resolution and validation are the reference's NumPy
rules (numpy.py:70-109): V defaults to 2, P to 16, offsets from ``choose_offsets``.
A CUDA device is required; without one the call raises ``RuntimeError``.
"""

from __future__ import annotations

import typing
import warnings

import numpy as np
import torch

from . import _native
from .common import (
    TUNINGS,
    choose_pblock_size_b200,
    choose_offsets,
    get_dtype_bytes,
    get_instance_size,
    povs_preflight,
    purge_dependent_param,
    randomness_flags,
    seed_to_u64,
)
from .constants import DEFAULT_CPU_PBLOCK_SIZE, MIN_VBLOCK_SIZE
from .types import Options


# Decks whose staging copy would leave less than this much device memory free are shuffled in
# place in host memory (mapped) instead of through a device copy.
DEVICE_HEADROOM_BYTES = 2 << 30


def shuffle(data: np.ndarray, iterations: int, options: Options | None, seed: int, flags: int = 0,
            mapped: bool | None = None) -> None:
    """Shuffle a host array in place along axis 0 on the current CUDA device.

    ``mapped``: None chooses: the deck is copied to the device and back when it fits the device's
    free memory, else the kernels work on it in host memory (``povs_shuffle_mapped_v1``, bound by
    the interconnect); True / False force one or the other.
    """
    options = typing.cast(
        "_HostOptions",
        options if options_is_complete(options) else optim_options_for_dataset(data, options),
    )
    preflight(data, iterations, options)
    row_bytes = get_instance_size(data) * get_dtype_bytes(data)
    if row_bytes == 0:
        return
    if not torch.cuda.is_available():
        raise RuntimeError("povs requires a CUDA device (B200, sm_100a); none is available")

    contiguous = data.flags.c_contiguous
    host = data if contiguous else np.ascontiguousarray(data)
    n_rows = host.shape[0]
    device = torch.device("cuda", torch.cuda.current_device())
    if mapped is None:
        free, _ = torch.cuda.mem_get_info(device)
        mapped = n_rows * row_bytes + DEVICE_HEADROOM_BYTES > free
    if mapped:
        _native.shuffle_mapped(
            host.ctypes.data, n_rows, row_bytes, list(options.offsets), iterations, options.physical_block_size,
            options.virtual_block_size, seed_to_u64(seed), device.index, flags | randomness_flags(options),
        )
        if not contiguous:
            data[...] = host
        return
    staging = torch.empty(n_rows * row_bytes, dtype=torch.uint8, device=device)
    _native.shuffle_host(
        host.ctypes.data,
        staging,
        n_rows,
        row_bytes,
        list(options.offsets),
        iterations,
        options.physical_block_size,
        options.virtual_block_size,
        seed_to_u64(seed),
        flags | randomness_flags(options),
    )
    if not contiguous:
        data[...] = host


class _HostOptions(Options):
    virtual_block_size: int
    physical_block_size: int
    offsets: list[int]


def options_is_complete(options: Options | None) -> bool:
    return options is not None and None not in (
        options.virtual_block_size,
        options.physical_block_size,
        options.offsets,
    )


def optim_options_for_dataset(data: np.ndarray, options: Options | None, tuning: str = "reference") -> Options:
    """Complete the options for a host dataset (``tuning`` as in ``povs.torch``: the reference's
    default pblock, or the B200 kernel's choice)."""
    assert tuning in TUNINGS, f"tuning ({tuning!r}) must be one of {TUNINGS}"
    options = options or Options()
    if options_is_complete(options):
        warnings.warn("All parameters already specified, skipping optimization")
        return options
    if options.physical_block_size is None and options.offsets is not None:
        purge_dependent_param(options, "physical_block_size", "offsets")
    vblk = options.virtual_block_size or MIN_VBLOCK_SIZE
    if options.physical_block_size:
        pblk = options.physical_block_size
    elif tuning == "b200":
        pblk = choose_pblock_size_b200(get_instance_size(data) * get_dtype_bytes(data), vblk, data.shape[0])
    else:
        pblk = DEFAULT_CPU_PBLOCK_SIZE
    return Options(
        randomness=options.randomness,
        virtual_block_size=vblk,
        physical_block_size=pblk,
        offsets=choose_offsets(
            deck_size=data.shape[0],
            instance_size=get_instance_size(data),
            dtype_bytes=get_dtype_bytes(data),
            pblock_size=pblk,
        ),
    )


def preflight(data: np.ndarray, iterations: int, options: Options) -> None:
    povs_preflight(data, iterations, options)


def shuffle_many(decks: list, iterations: int, options: Options | None, seeds: list[int], flags: int = 0) -> None:
    """Shuffle several host decks of one shape in place, overlapping their copies with the GPU work.

    Up to three device staging buffers (as many as fit the device's free memory) are used in
    rotation, so one deck's copy back overlaps another's copy in and a third's iterations; decks
    that do not fit at all are shuffled in host memory one by one (mapped).  Arrays that are not
    C-contiguous are staged through contiguous copies (one per distinct array).
    """
    if not decks:
        return
    first = decks[0]
    for d in decks:
        assert d.shape == first.shape and d.dtype == first.dtype, "all decks must share shape and dtype"
    options = typing.cast(
        "_HostOptions",
        options if options_is_complete(options) else optim_options_for_dataset(first, options),
    )
    preflight(first, iterations, options)
    row_bytes = get_instance_size(first) * get_dtype_bytes(first)
    if row_bytes == 0:
        return
    if not torch.cuda.is_available():
        raise RuntimeError("povs requires a CUDA device (B200, sm_100a); none is available")
    staged: dict[int, np.ndarray] = {}
    for d in decks:
        if not d.flags.c_contiguous and id(d) not in staged:
            staged[id(d)] = np.ascontiguousarray(d)
    hosts = [staged.get(id(d), d) for d in decks]
    n_rows = first.shape[0]
    device = torch.device("cuda", torch.cuda.current_device())
    deck_bytes = n_rows * row_bytes
    free, _ = torch.cuda.mem_get_info(device)
    n_buffers = min(3, len(decks))
    while n_buffers > 0 and n_buffers * deck_bytes + DEVICE_HEADROOM_BYTES > free:
        n_buffers -= 1
    if n_buffers == 0:
        for h, sd in zip(hosts, seeds):
            _native.shuffle_mapped(
                h.ctypes.data, n_rows, row_bytes, list(options.offsets), iterations, options.physical_block_size,
                options.virtual_block_size, seed_to_u64(sd), device.index, flags | randomness_flags(options),
            )
    else:
        buffers = [torch.empty(deck_bytes, dtype=torch.uint8, device=device) for _ in range(n_buffers)]
        _native.shuffle_host_batch(
            [h.ctypes.data for h in hosts], buffers, n_rows, row_bytes, list(options.offsets), iterations,
            options.physical_block_size, options.virtual_block_size, [seed_to_u64(sd) for sd in seeds],
            flags | randomness_flags(options),
        )
    for d in decks:
        h = staged.get(id(d))
        if h is not None:
            d[...] = h
