"""B200-native POV shuffle: a drop-in for the reference's ``povs`` package (src/povs/__init__.py).

Public API kept from the reference: ``shuffle``, ``Options``, ``BuildParams``, ``get_build_params``,
``optim_options_for_dataset``.  Additions: ``apply_randomness`` (inject offsets, block assignments
and per-vblock permutations, for bit-exact comparison with other implementations),
``check_device_status``, decks split into shards: ``shuffle_shards`` (one process) and
``ShardedDeck`` (one process per GPU, host shards streamed through it by ``shuffle_host_shards``),
many host decks streamed through the GPU (``shuffle_many``) and many independent CUDA decks
shuffled together (``shuffle_batch``).  ``povs.eval`` holds the
shuffle-bias metrics and exercises on the GPU.
"""

from __future__ import annotations

from typing import Any

import numpy as np
import torch as t

from . import numpy as povs_numpy
from . import torch as povs_torch
from .common import get_build_params, get_int_seed
from .distributed import ShardedDeck, shuffle_host_shards, shuffle_shards
from .injection import apply_randomness
from .types import BuildParams, Options

__all__ = [
    "shuffle",
    "Options",
    "BuildParams",
    "get_build_params",
    "optim_options_for_dataset",
    "apply_randomness",
    "check_device_status",
    "shuffle_shards",
    "shuffle_host_shards",
    "ShardedDeck",
    "shuffle_many",
    "shuffle_batch",
    "shuffle_mapped",
]


def shuffle(
    data: np.ndarray | t.Tensor,
    iterations: int = 1,
    options: Options | None = None,
    seed: int | np.random.Generator | Any | None = None,
) -> None:
    """POV Shuffle, in place along axis 0.

    :param data: ``torch.Tensor`` (CUDA or CPU) or ``numpy.ndarray``.
    :param iterations: Number of shuffling iterations.
    :param options: POV options; partial or missing options are resolved as in ``optim_options_for_dataset``.
    :param seed: Integer seed, ``np.random.Generator`` or ``torch.Generator`` (None draws fresh entropy).
    """
    seed = get_int_seed(seed, options)

    if isinstance(data, np.ndarray):
        povs_numpy.shuffle(data, iterations, options, seed)
        return

    if isinstance(data, t.Tensor):
        if data.get_device() == -1:
            shuffle(data.numpy(), iterations, options, seed)
            return
        povs_torch.shuffle(data, iterations, options, seed)
        return

    raise TypeError(f"Unsupported data type: {type(data)}")


def shuffle_mapped(
    data: np.ndarray | t.Tensor,
    iterations: int = 1,
    options: Options | None = None,
    seed: int | np.random.Generator | Any | None = None,
) -> None:
    """Shuffle a host deck (NumPy array or CPU tensor) in place WITHOUT copying it to the GPU: the
    kernels read and write it in host memory over the interconnect.  For decks larger than the
    GPU's memory (``povs.shuffle`` switches to this by itself when a host deck does not fit).
    Same result as ``povs.shuffle`` with the same arguments.  Addition to the reference API.
    """
    seed = get_int_seed(seed, options)
    if isinstance(data, t.Tensor):
        if data.get_device() != -1:
            raise TypeError("shuffle_mapped takes host decks; use shuffle for CUDA tensors")
        data = data.numpy()
    if not isinstance(data, np.ndarray):
        raise TypeError(f"Unsupported data type: {type(data)}")
    povs_numpy.shuffle(data, iterations, options, seed, mapped=True)


def shuffle_many(
    decks: list,
    iterations: int = 1,
    options: Options | None = None,
    seed: int | np.random.Generator | Any | None = None,
) -> None:
    """Shuffle several host decks (NumPy arrays or CPU tensors) of one shape, each in place.

    The decks stream through the GPU with their host/device copies overlapped; deck ``d`` is
    shuffled with seed ``seed + d``.  Addition to the reference API.
    """
    base = get_int_seed(seed, options)
    arrays = [d.numpy() if isinstance(d, t.Tensor) else d for d in decks]
    for d in decks:
        if isinstance(d, t.Tensor):
            assert d.get_device() == -1, "shuffle_many takes host decks; use shuffle for CUDA tensors"
        elif not isinstance(d, np.ndarray):
            raise TypeError(f"Unsupported data type: {type(d)}")
    povs_numpy.shuffle_many(arrays, iterations, options, [base + i for i in range(len(arrays))])


def shuffle_batch(
    decks: t.Tensor,
    iterations: int = 1,
    options: Options | None = None,
    seeds: Any = None,
) -> None:
    """Shuffle each deck ``decks[d]`` of a contiguous CUDA tensor (n_decks, rows, ...) independently, in place.

    One launch per iteration covers every deck.  ``seeds``: a sequence with one seed per deck, an int
    (deck d gets ``seeds + d``), or a generator / None from which one seed per deck is drawn in deck
    order; deck d ends exactly as ``shuffle(decks[d], iterations, options, seed=<its seed>)`` would
    leave it.  Addition to the reference API (its bias exercises loop over decks one call at a time).
    """
    if not isinstance(decks, t.Tensor) or decks.get_device() == -1:
        raise TypeError("shuffle_batch takes a CUDA tensor of decks; use shuffle_many for host decks")
    n = decks.shape[0]
    if isinstance(seeds, (int, np.integer)) and not isinstance(seeds, bool):
        per_deck = [int(seeds) + d for d in range(n)]
    elif seeds is None or isinstance(seeds, (np.random.Generator, t.Generator)):
        per_deck = [get_int_seed(seeds, options) for _ in range(n)]
    else:
        per_deck = [get_int_seed(s, options) for s in seeds]
    povs_torch.shuffle_batch(decks, iterations, options, per_deck)


def optim_options_for_dataset(
    data: np.ndarray | t.Tensor, options: Options | None = None, tuning: str = "reference"
) -> Options:
    """Resolve partial or missing options for a dataset.

    :param data: ``torch.Tensor`` or ``numpy.ndarray``.
    :param options: Starting point.
    :param tuning: ``"reference"`` (default): the reference's choices, so the same dataset gets the
        same options; ``"b200"``: ``physical_block_size`` chosen for this library's B200 kernel
        (vblocks of up to 64 KiB / 512 rows; several times faster than the reference's choice for
        small rows).  Addition to the reference API.
    :returns: Complete options for the dataset's route (CUDA options include ``gpu_thread_block_size``).
    """
    options = options or Options()

    if isinstance(data, np.ndarray):
        if povs_numpy.options_is_complete(options):
            return options
        return povs_numpy.optim_options_for_dataset(data, options, tuning)

    if isinstance(data, t.Tensor):
        if data.get_device() == -1:
            return optim_options_for_dataset(data.numpy(), options, tuning)
        if povs_torch.options_is_complete(options):
            return options
        return povs_torch.optim_options_for_dataset(data, options, tuning)

    raise TypeError(f"Unsupported data type: {type(data)}")


def check_device_status(device: int | t.device | None = None) -> None:
    """Synchronize ``device`` and raise ``RuntimeError`` if a kernel reported a failure since the last check."""
    from . import _native

    if device is None:
        index = t.cuda.current_device()
    elif isinstance(device, t.device):
        index = device.index if device.index is not None else t.cuda.current_device()
    else:
        index = int(device)
    status = _native.device_status(index)
    if status:
        raise RuntimeError(f"povs kernels on cuda:{index} reported device status 0x{status:x}")
