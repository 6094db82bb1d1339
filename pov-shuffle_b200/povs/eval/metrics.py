"""Shuffle-bias metrics computed on the GPU (reference: src/povs/eval/metrics.py).

Episodes are arrays of shape (num_episodes, deck_size) whose rows are permutations of the ids
0 .. deck_size-1 (shuffled ``arange`` decks).  They may be NumPy arrays or torch tensors; they
are moved to a CUDA device (the tensor's own, else ``device``, else the current one) and the
per-observation work - travel distances, their histograms, n-gram keys and their counts - runs in
the native library's kernels.  The O(deck) TVD arithmetic on the resulting counts is done on the host with
the reference's formulas, so results match the reference's NumPy implementation up to the
summation order of the final float64 sum.
"""

from __future__ import annotations

import math

import numpy as np
import torch

from .. import _native

_MAX_KEYS_BYTES = 512 * 1024 * 1024  # n-gram keys held at once (reference metrics.py:201-203)


def get_worker_data_scan_per_iter(vblock_size: int, pblock_size: int, deck_size: int) -> float:
    """Share of the deck one vblock (one parallel worker) sees per iteration (metrics.py:6-8)."""
    return (vblock_size * pblock_size) / deck_size


def get_cumulative_worker_exposure(worker_data_scan_per_iter: float, iterations: int) -> list[float]:
    """Cumulative share of the deck a worker has seen after each iteration (metrics.py:11-13)."""
    return [(i + 1) * worker_data_scan_per_iter for i in range(iterations)]


def get_pos_tvd_event_space(deck_size: int) -> int:
    """Positional TVD events: one travel distance per deck position (metrics.py:16-18)."""
    return deck_size


def get_ngram_tvd_event_space(deck_size: int, n: int) -> int:
    """n-gram TVD events: ordered choices of n-1 distinct non-zero distances (metrics.py:21-26)."""
    return math.perm(deck_size - 1, n - 1)


def get_sample_deficit(num_episodes: int, deck_size: int, event_space: int) -> int:
    """``event_space - observations``: positive when undersampled (metrics.py:29-35)."""
    return event_space - num_episodes * deck_size


def _episodes_on_device(episodes, device: torch.device | str | int | None) -> torch.Tensor:
    if not torch.cuda.is_available():
        raise RuntimeError("povs.eval metrics run on a CUDA device and none is available")
    if isinstance(episodes, torch.Tensor):
        t = episodes
        if not t.is_cuda:
            t = t.to(torch.device("cuda", torch.cuda.current_device()) if device is None else device)
    else:
        arr = np.asarray(episodes)
        t = torch.from_numpy(np.ascontiguousarray(arr)).to(
            torch.device("cuda", torch.cuda.current_device()) if device is None else device)
    assert t.dim() == 2, f"episodes must have shape (num_episodes, deck_size), got {tuple(t.shape)}"
    if t.dtype not in (torch.int32, torch.int64):
        t = t.to(torch.int64)
    return t


def get_tvd(episodes, device: torch.device | str | int | None = None) -> float:
    """TVD of the travel-distance distribution ``(position - id) mod deck`` against uniform.

    Reference: get_tvd (metrics.py:38-87).  The histogram is built on the GPU.
    """
    ids = _episodes_on_device(episodes, device)
    num_episodes, deck_size = ids.shape
    num_observations = int(num_episodes) * deck_size
    p_ref = 1.0 / min(num_observations, get_pos_tvd_event_space(deck_size))
    counts = torch.zeros(deck_size, dtype=torch.int64, device=ids.device)
    _native.travel_histogram(ids, 0, 1, counts)
    p_obs = counts.cpu().numpy() / num_observations
    return float(np.abs(p_obs - p_ref).sum() / 2)


def get_ngram_tvd(episodes, n: int, skip: int = 0, device: torch.device | str | int | None = None) -> float:
    """TVD of the n-gram relative-travel-distance distribution against uniform.

    Reference: get_ngram_tvd (metrics.py:90-248), adaptive formula included: for n = 2 a dense
    histogram of the ``deck - 1`` possible distances (built on the GPU); for n > 2 the distinct
    n-gram keys (computed and counted on the GPU in a hash table, ``povs_ngram_count_v1``) and the
    unobserved events accounted analytically.  When the keys would exceed 512 MiB, the same number of anchor
    positions per episode as the reference's is drawn from NumPy's global generator, as there.
    """
    assert n >= 2, f"n-gram degree ({n}) must be at least 2"
    ids = _episodes_on_device(episodes, device)
    num_episodes, deck_size = ids.shape
    num_observations = int(num_episodes) * deck_size
    event_space = get_ngram_tvd_event_space(deck_size, n)
    step = skip + 1

    if n == 2:
        p_ref = 1.0 / min(num_observations, event_space)
        counts = torch.zeros(deck_size, dtype=torch.int64, device=ids.device)
        _native.travel_histogram(ids, 1, step, counts)
        # A pair cannot hold the same id twice: that distance, (-step) mod deck, is not an event.
        key_counts = np.delete(counts.cpu().numpy(), (-step) % deck_size)
        p_obs = key_counts / num_observations
        return float(1 / 2 * np.abs(p_obs - p_ref).sum())

    max_keys = _MAX_KEYS_BYTES // 8
    positions = None
    effective = num_observations
    if num_observations > max_keys:
        per_episode = max(1, max_keys // int(num_episodes))
        chosen = np.sort(np.random.choice(deck_size, per_episode, replace=False))
        positions = torch.from_numpy(chosen.astype(np.int64)).to(ids.device)
        effective = int(num_episodes) * per_episode
    p_ref = 1.0 / min(effective, event_space)
    # Distinct keys counted in a hash table on the GPU; what comes back is how many keys were seen
    # exactly c times, so the reference's sum over keys of |count / effective - p_ref| is a sum over c.
    mult, big = _native.ngram_count(ids, n, step, positions)
    c = np.arange(1, len(mult), dtype=np.float64)
    per_key = mult[1:].astype(np.float64)
    observed = int(mult[1:].sum()) + int(mult[0])
    deviation = float(np.sum(per_key * np.abs(c / effective - p_ref)))
    deviation += float(np.sum(np.abs(np.sort(big).astype(np.float64) / effective - p_ref)))
    missing = min(event_space, effective) - observed
    return float(1 / 2 * (missing * p_ref + deviation))
