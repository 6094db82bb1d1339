"""Shuffle-bias evaluation on the GPU (counterpart of the reference's ``povs.eval`` package).

* ``metrics``: positional and n-gram TVDs of shuffled episodes; the histograms and n-gram keys are
  computed by CUDA kernels of the native library, the O(deck) TVD arithmetic on the host;
* ``exercises``: ``bias_per_iteration``, ``breaking_point_per_deck_size`` and
  ``shuffle_time_per_deck_size``, with every episode of an iteration shuffled by one batched launch
  (``povs.shuffle_batch``) instead of one call per episode;
* ``types.NgramSpec`` and the timing helpers of ``utils``.

LSTM predictability, plots, YAML/CSV report files and checkpoints of the reference's evaluation
scripts are not part of this package.
"""

from .exercises import (
    BiasPerIterResult,
    BreakingPointPerDeckSizeResult,
    ShuffleTimePerDeckSizeResult,
    bias_per_iteration,
    breaking_point_per_deck_size,
    shuffle_time_per_deck_size,
    timings_table,
)
from .metrics import (
    get_cumulative_worker_exposure,
    get_ngram_tvd,
    get_ngram_tvd_event_space,
    get_pos_tvd_event_space,
    get_sample_deficit,
    get_tvd,
    get_worker_data_scan_per_iter,
)
from .types import NgramSpec

__all__ = [
    "BiasPerIterResult",
    "BreakingPointPerDeckSizeResult",
    "ShuffleTimePerDeckSizeResult",
    "bias_per_iteration",
    "breaking_point_per_deck_size",
    "shuffle_time_per_deck_size",
    "timings_table",
    "get_cumulative_worker_exposure",
    "get_ngram_tvd",
    "get_ngram_tvd_event_space",
    "get_pos_tvd_event_space",
    "get_sample_deficit",
    "get_tvd",
    "get_worker_data_scan_per_iter",
    "NgramSpec",
]
