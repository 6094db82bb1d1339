"""Bias-metric oracle pinned to the reference's own metric values, and the host-side helpers of
``povs.eval`` (no GPU)."""

from __future__ import annotations

import json
import math
import sys

import numpy as np
import pytest

from conftest import GOLDEN
from oracle import metrics

sys.path.insert(0, str(GOLDEN))
from make_metrics_golden import CASES, episodes_for  # noqa: E402

GOLD = json.loads((GOLDEN / "metrics_golden.json").read_text())["cases"]


@pytest.mark.parametrize("entry", GOLD, ids=lambda e: f"deck{e['deck']}")
def test_oracle_metrics_match_reference_values(entry):
    eps = episodes_for(entry["case"], entry["deck"], entry["episodes"])
    assert abs(metrics.positional_tvd(eps) - entry["positional"]) < 1e-12
    for g in entry["ngram"]:
        assert abs(metrics.ngram_tvd(eps, g["n"], g["skip"]) - g["tvd"]) < 1e-12, g
        if g["n"] == 2 and g["skip"] == 0:
            assert abs(metrics.bigram_tvd(eps) - g["tvd"]) < 1e-12


def test_golden_cases_cover_the_generator():
    assert [(e["deck"], e["episodes"]) for e in GOLD] == CASES


def test_event_spaces_and_deficits():
    from povs.eval import metrics as m

    assert m.get_pos_tvd_event_space(1000) == 1000
    assert m.get_ngram_tvd_event_space(1000, 2) == 999
    assert m.get_ngram_tvd_event_space(1000, 3) == math.perm(999, 2)
    assert m.get_sample_deficit(3000, 1000, 999) == 999 - 3_000_000
    assert m.get_worker_data_scan_per_iter(2, 8, 1000) == 16 / 1000
    assert m.get_cumulative_worker_exposure(0.25, 3) == [0.25, 0.5, 0.75]


def test_ngram_spec():
    from povs.eval import NgramSpec

    assert NgramSpec.parse(3) == NgramSpec(3, 0)
    assert NgramSpec.parse((2, 1)) == NgramSpec(2, 1)
    assert NgramSpec.parse(NgramSpec(4)) == NgramSpec(4, 0)
    assert NgramSpec(2).title == "2-gram" and NgramSpec(3, 1).title == "3-gram (skip 1)"


def test_timings_table_has_the_reference_columns():
    from povs.eval import ShuffleTimePerDeckSizeResult, timings_table

    res = ShuffleTimePerDeckSizeResult(
        pov_times_ms=[[1.0, 3.0], None], baseline_times_ms=[[10.0, 10.0], [5.0]], option_sets=[None, None],
        pov_errors=[None, RuntimeError("x")], baseline_errors=[None, None])
    df = timings_table([10, 20], res)
    assert list(df.columns) == ["deck_size", "pov_mean_ms", "pov_std_ms", "baseline_mean_ms", "baseline_std_ms",
                                "speedup"]
    assert df["pov_mean_ms"][0] == 2.0 and df["speedup"][0] == 5.0
    assert df["pov_mean_ms"][1] is None or np.isnan(df["pov_mean_ms"][1])


def test_metrics_fail_loudly_without_a_gpu():
    import torch

    from povs.eval import get_tvd

    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    with pytest.raises(RuntimeError, match="CUDA device"):
        get_tvd(np.arange(6).reshape(2, 3))


def test_lstm_settings_are_rejected():
    from povs.eval import bias_per_iteration

    with pytest.raises(NotImplementedError):
        bias_per_iteration(10, 2, 1, None, np.random.default_rng(0), [], None, "cpu", lstm_settings=object())
