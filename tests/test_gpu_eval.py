"""Batched decks and the GPU bias metrics (``povs.shuffle_batch``, ``povs.eval``) against the
per-deck path, the oracle and the reference's own metric values."""

from __future__ import annotations

import json
import sys
from itertools import permutations

import numpy as np
import pytest
import torch

import povs
import povs.eval
from conftest import GOLDEN
from oracle import metrics as oracle_metrics

sys.path.insert(0, str(GOLDEN))
from make_metrics_golden import episodes_for  # noqa: E402

pytestmark = pytest.mark.gpu
DEV = "cuda:0"
GOLD = json.loads((GOLDEN / "metrics_golden.json").read_text())["cases"]


def _bytes_deck(n_decks: int, n_rows: int, row_bytes: int, seed: int) -> torch.Tensor:
    g = np.random.default_rng(seed)
    return torch.from_numpy(g.integers(0, 256, (n_decks, n_rows, row_bytes), dtype=np.uint8)).to(DEV)


@pytest.mark.parametrize(
    "n_decks,n_rows,row_bytes,P,V,offsets,iterations",
    [
        (37, 1000, 64, 8, 2, list(range(8)), 3),
        (5, 4099, 256, 32, 4, [0, 1, 5, 31], 2),
        (9, 777, 12, 16, 8, [0, 3], 4),
        (3, 600, 12288, 16, 2, [0, 1], 2),
        (300, 50, 4, 8, 2, [0, 1, 2], 5),
    ],
)
@pytest.mark.parametrize("randomness", ["uniform", "reference_cuda", "reference_numpy"])
def test_batch_equals_one_deck_at_a_time(n_decks, n_rows, row_bytes, P, V, offsets, iterations, randomness):
    decks = _bytes_deck(n_decks, n_rows, row_bytes, seed=n_decks)
    single = decks.clone()
    opts = povs.Options(V, P, offsets, max(32, min(64, V * P)), randomness)
    seeds = [1000 + 17 * d for d in range(n_decks)]
    povs.shuffle_batch(decks, iterations, opts, seeds=seeds)
    for d in range(n_decks):
        povs.shuffle(single[d], iterations, opts, seed=seeds[d])
    torch.cuda.synchronize()
    povs.check_device_status(0)
    assert torch.equal(decks, single)


@pytest.mark.parametrize("n_rows,row_bytes", [(1000, 64), (200_000, 256)])
def test_batch_reads_seeds_written_by_the_kernel_just_before(n_rows, row_bytes):
    """The seed array is written on the stream by the kernel right before the batched call (one
    iteration, the launch shape that could be chained to that kernel): every deck gets the new seeds."""
    from povs import _native

    n_decks, P, V, offsets = 6, 16, 2, [0, 1, 2, 3]
    decks = _bytes_deck(n_decks, n_rows, row_bytes, seed=n_rows)
    single = decks.clone()
    want_seeds = [90_001 + 31 * d for d in range(n_decks)]
    seeds = torch.zeros(n_decks, dtype=torch.int64, device=DEV)
    increment = torch.tensor(want_seeds, dtype=torch.int64).to(DEV)
    torch.cuda.synchronize()
    # Long kernels first, then the kernel that writes the seeds, then the batched call.
    spin = torch.ones(1 << 26, dtype=torch.float32, device=DEV)
    for _ in range(4):
        spin.mul_(1.0001)
    seeds.add_(increment)
    _native.shuffle_batch(decks, row_bytes, offsets, 1, P, V, seeds)
    for d in range(n_decks):
        _native.shuffle_device(single[d], row_bytes, offsets, 1, P, V, want_seeds[d])
    torch.cuda.synchronize()
    povs.check_device_status(0)
    assert torch.equal(decks, single)


def test_batch_matches_oracle(oracle_api):
    n_decks, n_rows, row_bytes, P, V, offsets, iterations = 4, 3001, 32, 16, 4, [0, 1, 2, 7], 3
    decks = _bytes_deck(n_decks, n_rows, row_bytes, seed=3)
    host = decks.cpu().numpy().copy()
    povs.shuffle_batch(decks, iterations, povs.Options(V, P, offsets, 32), seeds=[5, 6, 7, 8])
    got = decks.cpu().numpy()
    for d in range(n_decks):
        want = host[d].copy()
        oracle_api.shuffle(want, iterations, P, V, offsets, 5 + d)
        assert np.array_equal(got[d], want)


def test_batch_seed_forms():
    decks = _bytes_deck(6, 500, 16, seed=1)
    a, b, c = decks.clone(), decks.clone(), decks.clone()
    opts = povs.Options(2, 16, [0, 1, 2], 32)
    povs.shuffle_batch(a, 2, opts, seeds=np.random.default_rng(9))
    rng = np.random.default_rng(9)
    for d in range(6):
        povs.shuffle(b[d], 2, opts, seed=rng)
    povs.shuffle_batch(c, 2, opts, seeds=40)
    for d in range(6):
        povs.shuffle(decks[d], 2, opts, seed=40 + d)
    torch.cuda.synchronize()
    assert torch.equal(a, b) and torch.equal(c, decks)


@pytest.mark.parametrize("entry", GOLD, ids=lambda e: f"deck{e['deck']}")
@pytest.mark.parametrize("dtype", [torch.int64, torch.int32])
def test_gpu_metrics_match_reference_values(entry, dtype):
    eps = torch.from_numpy(episodes_for(entry["case"], entry["deck"], entry["episodes"])).to(DEV, dtype)
    assert abs(povs.eval.get_tvd(eps) - entry["positional"]) < 1e-12
    for g in entry["ngram"]:
        assert abs(povs.eval.get_ngram_tvd(eps, g["n"], skip=g["skip"]) - g["tvd"]) < 1e-12, g


def test_gpu_metrics_on_strided_views_and_host_arrays():
    """Column 0 of a (episodes, deck, 16) int32 tensor: element stride 16."""
    eps = episodes_for(2, 50, 40)
    wide = torch.from_numpy(np.repeat(eps[:, :, None], 16, axis=2).astype(np.int32)).to(DEV)
    view = wide[:, :, 0]
    assert view.stride(1) == 16
    assert abs(povs.eval.get_tvd(view) - oracle_metrics.positional_tvd(eps)) < 1e-12
    assert abs(povs.eval.get_ngram_tvd(view, 3, skip=1) - oracle_metrics.ngram_tvd(eps, 3, 1)) < 1e-12
    assert abs(povs.eval.get_tvd(eps) - oracle_metrics.positional_tvd(eps)) < 1e-12  # NumPy input


@pytest.mark.parametrize(
    "samples,n,expected",
    [
        (np.array(list(permutations(range(3)))), 1, 0.0),
        (np.tile(np.arange(3), 3).reshape(3, 3), 1, 2 / 3),
        (np.array([[0, 1, 2], [1, 2, 0], [2, 0, 1]]), 1, 0.0),
        (np.array([[0, 1, 2]] * 3 + [[2, 1, 0]] * 3), 1, 1 / 3),
        (np.array(list(permutations(range(3)))), 2, 0.0),
        (np.array(list(permutations(range(3)))), 3, 0.0),
        (np.tile(np.arange(3), 3).reshape(3, 3), 2, 1 / 2),
        (np.tile(np.arange(3), 3).reshape(3, 3), 3, 1 / 2),
    ],
)
def test_gpu_metric_known_answers(samples, n, expected):
    """The reference's known-answer cases (src/tests/eval/test_metrics.py:19-98); n = 1 is get_tvd."""
    got = povs.eval.get_tvd(samples) if n == 1 else povs.eval.get_ngram_tvd(samples, n)
    assert np.isclose(got, expected, atol=0)


def test_ngram_subsampling_matches_oracle(monkeypatch):
    """Past the key budget both sides draw the same anchors from NumPy's global generator."""
    from povs.eval import metrics as gm

    eps = episodes_for(3, 101, 30)
    monkeypatch.setattr(gm, "_MAX_KEYS_BYTES", 8 * 700)
    np.random.seed(11)
    got = povs.eval.get_ngram_tvd(eps, 3, skip=2)
    np.random.seed(11)
    want = oracle_metrics.ngram_tvd(eps, 3, 2, max_keys=700)
    assert abs(got - want) < 1e-12


def test_bias_per_iteration_reproduces_the_episode_loop():
    deck_size, samples, iters = 200, 64, 3
    res = povs.eval.bias_per_iteration(deck_size, samples, iters, povs.Options(2, 8), np.random.default_rng(4),
                                       [povs.eval.NgramSpec(2), (3, 1)], torch.int64, DEV)
    # The same seeds drawn in the same order, one povs.shuffle call per episode.
    rng = np.random.default_rng(4)
    deck = torch.arange(deck_size, dtype=torch.int64, device=DEV)
    opts = povs.optim_options_for_dataset(deck, povs.Options(2, 8))
    eps = deck.unsqueeze(0).expand(samples, -1).clone()
    for i in range(iters):
        for s in range(samples):
            povs.shuffle(eps[s], iterations=1, options=opts, seed=rng)
        host = eps.cpu().numpy()
        assert abs(res.pos_tvds[i] - oracle_metrics.positional_tvd(host)) < 1e-12
        assert abs(res.ngram_tvds[i, 0] - oracle_metrics.ngram_tvd(host, 2, 0)) < 1e-12
        assert abs(res.ngram_tvds[i, 1] - oracle_metrics.ngram_tvd(host, 3, 1)) < 1e-12
    base = np.tile(np.arange(deck_size), (samples, 1))
    for s in range(samples):
        rng.shuffle(base[s])
    assert abs(res.baseline_pos_tvd - oracle_metrics.positional_tvd(base)) < 1e-12
    assert res.sample_deficits["positional"] == deck_size - samples * deck_size
    assert res.pos_tvds[-1] < res.pos_tvds[0]


def test_breaking_point_with_checkpoints(tmp_path):
    kw = dict(deck_sizes=[64, 128], num_episodes=256, ngram_specs=[povs.eval.NgramSpec(2)],
              positional_tolerance=0.02, ngram_tolerances={}, default_ngram_tolerance=0.02,
              max_iterations_per_deck_size={128: 6}, default_max_iterations=8, povs_options_per_deck_size={},
              default_options=povs.Options(2, 8), dtype=torch.int32, device=DEV, checkpoint_dir=tmp_path)
    first = povs.eval.breaking_point_per_deck_size(rng=np.random.default_rng(1), **kw)
    again = povs.eval.breaking_point_per_deck_size(rng=np.random.default_rng(999), **kw)  # from checkpoints
    for size in (64, 128):
        a, b = first.deck_sizes[size], again.deck_sizes[size]
        assert a.positional_breaking_point == b.positional_breaking_point
        assert a.ngram_breaking_points == b.ngram_breaking_points
        assert a.positional_breaking_point is None or 1 <= a.positional_breaking_point <= kw["default_max_iterations"]
    assert (tmp_path / "64" / "baseline" / "episodes.npy").exists()
    assert (tmp_path / "64" / "pov_1" / "metrics.json").exists()


def test_shuffle_time_per_deck_size_report(monkeypatch, tmp_path):
    """The timing exercise (reference eval/exercises.py:29-107) on a few deck sizes: one timing list per
    deck size, the reference's timings.csv columns, and every timed deck still a permutation of its rows
    (the exercise allocates zero decks, as the reference does; here they carry row ids)."""
    import pandas as pd

    from povs.eval import exercises

    timed = []
    real_shuffle = exercises.shuffle

    def recording_shuffle(data, *args, **kwargs):
        timed.append(data)
        return real_shuffle(data, *args, **kwargs)

    real_zeros = torch.zeros

    def id_rows(*shape, dtype=None, device=None, **kw):
        t = real_zeros(*shape, dtype=dtype, device=device, **kw)
        if t.is_cuda and t.dim() == 2:
            t.copy_(torch.arange(t.shape[0], device=t.device, dtype=torch.int64)[:, None].expand_as(t).to(t.dtype))
        return t

    monkeypatch.setattr(exercises, "shuffle", recording_shuffle)
    monkeypatch.setattr(exercises.torch, "zeros", id_rows)
    sizes = [1000, 4096, 65_536]
    res = exercises.shuffle_time_per_deck_size(
        deck_sizes=sizes, iterations=3, instance_size=16, num_runs=3, num_warmup_runs=1,
        povs_options_per_deck_size={4096: povs.Options(virtual_block_size=4)}, default_options=None,
        dtype=torch.int32, seed=11, tolerate_errors=False)
    monkeypatch.undo()
    assert [len(t) for t in res.pov_times_ms] == [3, 3, 3] and all(x > 0 for t in res.pov_times_ms for x in t)
    assert [len(t) for t in res.baseline_times_ms] == [3, 3, 3]
    assert res.option_sets[1].virtual_block_size == 4 and res.option_sets[0].virtual_block_size == 2
    assert res.pov_errors == [None] * 3 and res.baseline_errors == [None] * 3
    table = exercises.timings_table(sizes, res)
    assert list(table.columns) == ["deck_size", "pov_mean_ms", "pov_std_ms", "baseline_mean_ms", "baseline_std_ms",
                                   "speedup"]
    table.to_csv(tmp_path / "timings.csv", index=False)
    back = pd.read_csv(tmp_path / "timings.csv")
    assert back["deck_size"].tolist() == sizes and (back["speedup"] > 0).all()
    seen = {}
    for d in timed:
        seen[id(d)] = d
    assert len(seen) == len(sizes)
    torch.cuda.synchronize()
    for d in seen.values():
        ids = d[:, 0].to(torch.int64)
        assert torch.equal(d.to(torch.int64), ids[:, None].expand_as(d)), "a row was torn"
        assert torch.equal(torch.sort(ids).values, torch.arange(d.shape[0], device=d.device))
        assert not torch.equal(ids, torch.arange(d.shape[0], device=d.device))


@pytest.mark.parametrize("n,skip", [(3, 0), (4, 1)])
def test_ngram_counts_hash_table_against_sorting(n, skip):
    """The hash-table counts (povs_ngram_count_v1) against sorting the same keys (torch.unique): the
    same multiplicities, also when every count goes through the overflow list (mult_bins = 2)."""
    from povs import _native

    ids = torch.from_numpy(episodes_for(3, 1000, 300)).to(DEV)
    keys = _native.ngram_keys(ids, n, skip + 1)
    _, counts = torch.unique(keys, return_counts=True)
    c = counts.cpu().numpy()
    mult, big = _native.ngram_count(ids, n, skip + 1)
    # Keys seen 65,536 times or more (half the episodes are near-identity here) come back one by one.
    assert int(mult[0]) == len(big) == int((c >= len(mult)).sum())
    want = np.bincount(c[c < len(mult)], minlength=len(mult))
    want[0] = 0
    got = mult.astype(np.int64)
    got[0] = 0
    assert np.array_equal(got, want)
    assert np.array_equal(np.sort(big.astype(np.int64)), np.sort(c[c >= len(mult)]))
    mult2, big2 = _native.ngram_count(ids, n, skip + 1, mult_bins=2, overflow_cap=1)
    assert int(mult2[1]) == int((c == 1).sum()) and int(mult2[0]) == int((c >= 2).sum())
    assert np.array_equal(np.sort(big2.astype(np.int64)), np.sort(c[c >= 2]))
