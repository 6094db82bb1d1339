"""Bias and timing exercises (reference: src/povs/eval/exercises.py).

Same signatures and result types as the reference's, with two changes of means: every iteration
shuffles all episodes with one batched launch per iteration (``povs.shuffle_batch``; the episode
seeds are drawn from ``rng`` in episode order, as the reference's per-episode loop draws them),
and the metrics run on the GPU (``povs.eval.metrics``).  LSTM predictability is not part of this
package: passing ``lstm_settings`` raises ``NotImplementedError``.
"""

from __future__ import annotations

import json
import logging
from pathlib import Path
from typing import Any, NamedTuple

import numpy as np
import torch

from .. import optim_options_for_dataset, shuffle, shuffle_batch
from ..types import Options
from .metrics import get_ngram_tvd, get_ngram_tvd_event_space, get_pos_tvd_event_space, get_sample_deficit, get_tvd
from .types import NgramSpec
from .utils import time_cpu_op, time_cuda_op

_logger = logging.getLogger(__name__)


def _no_lstm(lstm_settings: Any) -> None:
    if lstm_settings is not None:
        raise NotImplementedError("LSTM predictability is not part of this package")


def _sample_deficits(num_episodes: int, deck_size: int, ngram_specs: list[NgramSpec]) -> dict[str, int]:
    return {
        "positional": get_sample_deficit(num_episodes, deck_size, get_pos_tvd_event_space(deck_size)),
        **{
            spec.title: get_sample_deficit(num_episodes, deck_size, get_ngram_tvd_event_space(deck_size, spec.n))
            for spec in ngram_specs
        },
    }


def _uniform_episodes(deck: torch.Tensor, num_episodes: int, rng: np.random.Generator) -> np.ndarray:
    """The reference's baseline: ``rng.shuffle`` of every episode of the identity deck (host)."""
    episodes = deck.unsqueeze(0).expand(num_episodes, -1).clone().cpu().numpy()
    for i in range(num_episodes):
        rng.shuffle(episodes[i])
    return episodes


# ---------------------------------------------------------------------------------------------
# Shuffle time per deck size (exercises.py:21-101).
# ---------------------------------------------------------------------------------------------


class ShuffleTimePerDeckSizeResult(NamedTuple):
    pov_times_ms: list[list[float] | None]  # per deck size: per-run times, None on error
    baseline_times_ms: list[list[float] | None]
    option_sets: list[Options | None]
    pov_errors: list[Exception | None]
    baseline_errors: list[Exception | None]


def shuffle_time_per_deck_size(
    deck_sizes: list[int],
    iterations: int,
    instance_size: int,
    num_runs: int,
    num_warmup_runs: int,
    povs_options_per_deck_size: dict[int, Options | None],
    default_options: Options | None,
    dtype: torch.dtype,
    seed: int,
    tolerate_errors: bool,
    cuda_device_id: int = 0,
) -> ShuffleTimePerDeckSizeResult:
    """POV shuffle time (CUDA events) and the host ``Generator.shuffle`` baseline per deck size."""
    pov_times, base_times, option_sets, pov_errors, base_errors = [], [], [], [], []
    for i, deck_size in enumerate(deck_sizes):
        data = torch.zeros(deck_size, instance_size, dtype=dtype, device=f"cuda:{cuda_device_id}")
        opts, pov_t, pov_e, base_t, base_e = None, None, None, None, None
        try:
            opts = optim_options_for_dataset(data, povs_options_per_deck_size.get(deck_size) or default_options)
            pov_t = time_cuda_op(lambda: shuffle(data, iterations=iterations, options=opts, seed=seed),
                                 num_warmup=num_warmup_runs, num_runs=num_runs)
        except Exception as e:  # recorded per deck size when tolerated, as in the reference
            if not tolerate_errors:
                raise
            pov_e = e
        try:
            base_rng = np.random.default_rng(seed + i + len(deck_sizes))
            base_data = torch.zeros(deck_size, instance_size, dtype=dtype).numpy()
            base_t = time_cpu_op(lambda: base_rng.shuffle(base_data), num_warmup=num_warmup_runs, num_runs=num_runs)
        except Exception as e:
            if not tolerate_errors:
                raise
            base_e = e
        option_sets.append(opts)
        pov_times.append(pov_t)
        base_times.append(base_t)
        pov_errors.append(pov_e)
        base_errors.append(base_e)
    return ShuffleTimePerDeckSizeResult(pov_times, base_times, option_sets, pov_errors, base_errors)


def timings_table(deck_sizes: list[int], result: ShuffleTimePerDeckSizeResult):
    """The timing report's table (reference eval/scripts/time_per_deck_size.py:56-82): a pandas
    DataFrame with columns deck_size, pov_mean_ms, pov_std_ms, baseline_mean_ms, baseline_std_ms,
    speedup (None where a run failed); ``.to_csv`` writes the reference's timings.csv schema."""
    import pandas as pd

    def stat(times, f):
        return [float(f(t)) if t is not None else None for t in times]

    pov_mean, pov_std = stat(result.pov_times_ms, np.mean), stat(result.pov_times_ms, np.std)
    base_mean, base_std = stat(result.baseline_times_ms, np.mean), stat(result.baseline_times_ms, np.std)
    speedup = [b / p if b is not None and p is not None else None for b, p in zip(base_mean, pov_mean)]
    return pd.DataFrame({
        "deck_size": list(deck_sizes),
        "pov_mean_ms": pov_mean,
        "pov_std_ms": pov_std,
        "baseline_mean_ms": base_mean,
        "baseline_std_ms": base_std,
        "speedup": speedup,
    })


# ---------------------------------------------------------------------------------------------
# Bias per iteration (exercises.py:340-423).
# ---------------------------------------------------------------------------------------------


class BiasPerIterResult(NamedTuple):
    options: Options
    sample_deficits: dict[str, int]
    baseline_pos_tvd: float
    pos_tvds: np.ndarray  # (max_iterations,)
    baseline_ngram_tvds: np.ndarray  # (len(ngram_specs),)
    ngram_tvds: np.ndarray  # (max_iterations, len(ngram_specs))
    baseline_lstm_predictability: float | None = None
    lstm_predictabilities: np.ndarray | None = None


def bias_per_iteration(
    deck_size: int,
    num_samples: int,
    max_iterations: int,
    options: Options | None,
    rng: np.random.Generator,
    ngram_specs: list[NgramSpec],
    dtype: torch.dtype,
    device: str,
    lstm_settings: Any = None,
) -> BiasPerIterResult:
    """Positional and n-gram TVDs after 1 .. max_iterations cumulative iterations, and of a
    uniform shuffle.  ``num_samples`` decks ``arange(deck_size)`` are shuffled together, one
    iteration at a time, each with a fresh seed from ``rng``."""
    _no_lstm(lstm_settings)
    ngram_specs = [NgramSpec.parse(s) for s in ngram_specs]
    deck = torch.arange(deck_size, dtype=dtype, device=device)
    options = optim_options_for_dataset(deck, options)
    tvds = np.zeros(max_iterations, dtype=float)
    ngram_tvds = np.zeros((max_iterations, len(ngram_specs)), dtype=float)

    samples = deck.unsqueeze(0).expand(num_samples, -1).clone()
    for i in range(max_iterations):
        shuffle_batch(samples, iterations=1, options=options, seeds=rng)
        tvds[i] = get_tvd(samples)
        ngram_tvds[i, :] = [get_ngram_tvd(samples, s.n, skip=s.skip) for s in ngram_specs]

    baseline = _uniform_episodes(deck, num_samples, rng)
    return BiasPerIterResult(
        options=options,
        sample_deficits=_sample_deficits(num_samples, deck_size, ngram_specs),
        baseline_pos_tvd=get_tvd(baseline, device=device),
        pos_tvds=tvds,
        baseline_ngram_tvds=np.array([get_ngram_tvd(baseline, s.n, skip=s.skip, device=device) for s in ngram_specs]),
        ngram_tvds=ngram_tvds,
    )


# ---------------------------------------------------------------------------------------------
# Breaking point per deck size (exercises.py:104-337).
# ---------------------------------------------------------------------------------------------


class _BreakingPointPerDeckSizeResult(NamedTuple):
    options: Options
    sample_deficit: dict[str, int]
    positional_breaking_point: int | None = None
    ngram_breaking_points: dict = {}  # NgramSpec -> iteration | None
    lstm_breaking_point: int | None = None
    non_convergences: list[str] | None = None


class BreakingPointPerDeckSizeResult(NamedTuple):
    deck_sizes: dict[int, _BreakingPointPerDeckSizeResult]


def _load_episodes(ckpt: Path | None, name: str) -> np.ndarray | None:
    f = ckpt / name / "episodes.npy" if ckpt is not None else None
    return np.load(f) if f is not None and f.exists() else None


def _save_episodes(ckpt: Path | None, name: str, episodes: np.ndarray) -> None:
    if ckpt is not None:
        (ckpt / name).mkdir(parents=True, exist_ok=True)
        np.save(ckpt / name / "episodes.npy", episodes)


def _load_metrics(ckpt: Path | None, name: str) -> dict:
    f = ckpt / name / "metrics.json" if ckpt is not None else None
    return json.loads(f.read_text()) if f is not None and f.exists() else {}


def _save_metrics(ckpt: Path | None, name: str, metrics: dict) -> None:
    if ckpt is not None:
        (ckpt / name).mkdir(parents=True, exist_ok=True)
        (ckpt / name / "metrics.json").write_text(json.dumps(metrics))


def breaking_point_per_deck_size(
    deck_sizes: list,
    num_episodes: int,
    ngram_specs: list[NgramSpec],
    positional_tolerance: float,
    ngram_tolerances: dict,
    default_ngram_tolerance: float,
    max_iterations_per_deck_size: dict,
    default_max_iterations: int,
    povs_options_per_deck_size: dict,
    default_options,
    rng: np.random.Generator,
    dtype,
    device: str,
    lstm_settings: Any = None,
    lstm_tolerance: float = 0.01,
    checkpoint_dir: Path | None = None,
) -> BreakingPointPerDeckSizeResult:
    """First iteration at which each metric's TVD is within its tolerance of the uniform
    baseline's, per deck size (None where the iteration cap is reached first).  Checkpoints, when
    ``checkpoint_dir`` is given, use the reference's layout: ``<dir>/<deck_size>/baseline`` and
    ``<dir>/<deck_size>/pov_<k>``, each with ``episodes.npy`` and ``metrics.json``."""
    _no_lstm(lstm_settings)
    ngram_specs = [NgramSpec.parse(s) for s in ngram_specs]
    final = BreakingPointPerDeckSizeResult(deck_sizes={})
    for deck_size in deck_sizes:
        deck = torch.arange(deck_size, dtype=dtype, device=device)
        opts = optim_options_for_dataset(deck, povs_options_per_deck_size.get(deck_size) or default_options)
        max_iter = max_iterations_per_deck_size.get(deck_size, default_max_iterations)
        ckpt = checkpoint_dir / str(deck_size) if checkpoint_dir is not None else None

        baseline = _load_episodes(ckpt, "baseline")
        if baseline is None:
            baseline = _uniform_episodes(deck, num_episodes, rng)
            _save_episodes(ckpt, "baseline", baseline)
        base_metrics = _load_metrics(ckpt, "baseline")
        if "positional" not in base_metrics:
            base_metrics["positional"] = get_tvd(baseline, device=device)
        for spec in ngram_specs:
            if spec.title not in base_metrics:
                base_metrics[spec.title] = get_ngram_tvd(baseline, spec.n, skip=spec.skip, device=device)
        _save_metrics(ckpt, "baseline", base_metrics)

        pos_bp: int | None = None
        ngram_bp: dict = {spec: None for spec in ngram_specs}
        episodes: torch.Tensor | None = None
        converged = False
        for iteration in range(1, max_iter + 1):
            name = f"pov_{iteration}"
            loaded = _load_episodes(ckpt, name)
            if loaded is not None:
                episodes = torch.as_tensor(loaded, dtype=dtype, device=device)
            else:
                if episodes is None:
                    episodes = deck.unsqueeze(0).expand(num_episodes, -1).clone()
                shuffle_batch(episodes, iterations=1, options=opts, seeds=rng)
                _save_episodes(ckpt, name, episodes.cpu().numpy())
            metrics = _load_metrics(ckpt, name)
            if pos_bp is None:
                if "positional" not in metrics:
                    metrics["positional"] = get_tvd(episodes)
                if metrics["positional"] - base_metrics["positional"] < positional_tolerance:
                    pos_bp = iteration
                    _logger.info("deck=%d iter=%d: positional breaking point", deck_size, iteration)
            for spec in ngram_specs:
                if ngram_bp[spec] is None:
                    if spec.title not in metrics:
                        metrics[spec.title] = get_ngram_tvd(episodes, spec.n, skip=spec.skip)
                    tol = ngram_tolerances.get(spec.n, default_ngram_tolerance)
                    if metrics[spec.title] - base_metrics[spec.title] < tol:
                        ngram_bp[spec] = iteration
                        _logger.info("deck=%d iter=%d: %s breaking point", deck_size, iteration, spec.title)
            _save_metrics(ckpt, name, metrics)
            if pos_bp is not None and all(v is not None for v in ngram_bp.values()):
                converged = True
                break
        non_conv = None
        if not converged:
            non_conv = (["positional"] if pos_bp is None else []) + [s.title for s, v in ngram_bp.items() if v is None]
        final.deck_sizes[deck_size] = _BreakingPointPerDeckSizeResult(
            options=opts,
            sample_deficit=_sample_deficits(num_episodes, deck_size, ngram_specs),
            positional_breaking_point=pos_bp,
            ngram_breaking_points=ngram_bp,
            non_convergences=non_conv,
        )
    return final
