"""ORACLE - test infrastructure only.

Restatement of the reference's shuffle-bias metrics (src/povs/eval/metrics.py):

* positional TVD (metrics.py:38-87): for every element of every episode the travel distance
  ``(position - original_index) mod deck_size``; TVD of its histogram against the uniform
  distribution over ``deck_size`` values;
* bigram TVD (metrics.py:90-178, ``n = 2``, ``skip = 0``): for every position ``i`` the relative
  travel distance ``((v[i+1] - v[i]) - 1) mod deck_size`` of the adjacent pair (with wrap
  around), the impossible value ``deck_size - 1`` removed, TVD against uniform over the remaining
  ``deck_size - 1`` values (every observation still counts in the denominator).

* n-gram TVD for any n >= 2 and skip (metrics.py:90-248): relative travel distances of the n-1
  elements spaced ``skip + 1`` apart from the anchor, reduced mod deck_size; for n = 2 the dense
  histogram above, for n > 2 base-deck_size keys counted sparsely with the unobserved events
  added analytically (adaptive TVD), anchors subsampled from NumPy's global generator when the
  keys would exceed ``max_keys``.

Episodes are arrays of shape (episodes, deck_size) holding the original indices in shuffled order.
Pinned by the reference's known-answer tests (src/tests/eval/test_metrics.py) in tests/test_bias.py.
"""

from __future__ import annotations

import math

import numpy as np


def positional_tvd(episodes: np.ndarray) -> float:
    episodes = np.asarray(episodes, dtype=np.int64)
    n_ep, deck = episodes.shape
    dist = (np.arange(deck, dtype=np.int64)[None, :] - episodes) % deck
    counts = np.bincount(dist.ravel(), minlength=deck)
    return float(np.abs(counts / (n_ep * deck) - 1.0 / deck).sum() / 2)


def bigram_tvd(episodes: np.ndarray) -> float:
    episodes = np.asarray(episodes, dtype=np.int64)
    n_ep, deck = episodes.shape
    nxt = np.roll(episodes, -1, axis=1)
    rtd = ((nxt - episodes) - 1) % deck
    counts = np.bincount(rtd.ravel(), minlength=deck)
    counts = np.delete(counts, (-1) % deck)
    return float(np.abs(counts / (n_ep * deck) - 1.0 / min(n_ep * deck, deck - 1)).sum() / 2)


def ngram_tvd(episodes: np.ndarray, n: int, skip: int = 0, max_keys: int = (512 * 1024 * 1024) // 8) -> float:
    """n-gram TVD of the reference (metrics.py:90-248), any n >= 2."""
    episodes = np.asarray(episodes, dtype=np.int64)
    n_ep, deck = episodes.shape
    n_obs = n_ep * deck
    event_space = math.perm(deck - 1, n - 1)
    step = skip + 1
    offsets = step * np.arange(n, dtype=np.int64)
    if n == 2:
        nxt = episodes[:, (np.arange(deck) + step) % deck]
        counts = np.bincount((((nxt - episodes) - step) % deck).ravel(), minlength=deck)
        counts = np.delete(counts, (-step) % deck)
        return float(np.abs(counts / n_obs - 1.0 / min(n_obs, event_space)).sum() / 2)
    if n_obs > max_keys:
        per_ep = max(1, max_keys // n_ep)
        anchors = np.sort(np.random.choice(deck, per_ep, replace=False))
    else:
        per_ep = deck
        anchors = np.arange(deck)
    eff = n_ep * per_ep
    p_ref = 1.0 / min(eff, event_space)
    idx = (anchors[:, None] + offsets[None, :]) % deck  # (per_ep, n)
    grams = episodes[:, idx]  # (n_ep, per_ep, n)
    rtd = (grams[..., 1:] - grams[..., :1]) - offsets[None, None, 1:]
    digits = (rtd % deck).reshape(-1, n - 1)
    keys = np.zeros(len(digits), dtype=np.int64)
    with np.errstate(over="ignore"):
        for k in range(n - 1):
            keys = keys * np.int64(deck) + digits[:, k]
    _, counts = np.unique(keys, return_counts=True)
    missing = min(event_space, eff) - len(counts)
    return float(0.5 * (missing * p_ref + np.sum(np.abs(counts / eff - p_ref))))
