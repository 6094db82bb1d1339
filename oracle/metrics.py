"""ORACLE - test infrastructure only.

Restatement of the reference's shuffle-bias metrics (src/povs/eval/metrics.py):

* positional TVD (metrics.py:38-87): for every element of every episode the travel distance
  ``(position - original_index) mod deck_size``; TVD of its histogram against the uniform
  distribution over ``deck_size`` values;
* bigram TVD (metrics.py:90-178, ``n = 2``, ``skip = 0``): for every position ``i`` the relative
  travel distance ``((v[i+1] - v[i]) - 1) mod deck_size`` of the adjacent pair (with wrap
  around), the impossible value ``deck_size - 1`` removed, TVD against uniform over the remaining
  ``deck_size - 1`` values (every observation still counts in the denominator).

Episodes are arrays of shape (episodes, deck_size) holding the original indices in shuffled order.
Pinned by the reference's known-answer tests (src/tests/eval/test_metrics.py) in tests/test_bias.py.
"""

from __future__ import annotations

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
