"""Generate the bias-suite reference statistics (tests/golden/bias_suite.json).

Workload: int32 deck of 1000 rows x 16, row i filled with i; 3000 episodes seeded 0..2999; for
every iteration count it = 1..8 each episode shuffles a fresh deck with ``iterations=it`` and
``seed=episode`` (V = 2, P = 8, offsets from the reference's chooser: 0..7).  Column 0 of the
shuffled deck is the episode.  Statistics (positional TVD, bigram TVD) for:

* ``reference_numpy``  - the reference's own NumPy path (``povs.shuffle`` imported from the reference
                         checkout, src/povs/numpy.py), P = 8 allowed by lowering its MIN_PBLOCK_SIZE;
* ``reference_cuda``   - the reference CUDA path's randomness (oracle/ref_cuda_rng.cpp: std::mt19937
                         host draws + the kernel's xorshift32 Fisher-Yates) applied by the C oracle;
* ``numpy_shuffle``    - ``numpy.random.default_rng(episode).shuffle`` (the reference's baseline);
* ``library``       - the library's device randomness through the oracle port; the GPU run must
                         reproduce these episodes exactly;
* ``library_reference_cuda`` - the same with ``randomness="reference_cuda"`` (the reference CUDA
                         path's distribution drawn on the device);
* ``library_reference_numpy`` - the same with ``randomness="reference_numpy"`` (the reference NumPy
                         path's distribution: its 999 seeded RandomState permutations).

Pass ``--reuse`` to keep the ``reference_numpy`` statistics already in the file (they take minutes).

Usage: python tests/golden/make_bias_golden.py <reference_root> [episodes] [--reuse]
"""

from __future__ import annotations

import json
import multiprocessing as mp
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
REPO = HERE.parent.parent
OUT = HERE / "bias_suite.json"

N_ROWS, WIDTH, V, P = 1000, 16, 2, 8
OFFSETS = list(range(8))
ITERATIONS = list(range(1, 9))


def fresh_deck() -> np.ndarray:
    return np.repeat(np.arange(N_ROWS, dtype=np.int32)[:, None], WIDTH, axis=1)


def _ref_numpy_chunk(args):
    reference_root, seeds = args
    sys.path.insert(0, str(Path(reference_root) / "src"))
    import povs as ref_povs
    import povs.common as ref_common
    from povs import Options

    ref_common.MIN_PBLOCK_SIZE = 8
    opts = Options(virtual_block_size=V, physical_block_size=P, offsets=OFFSETS)
    out = np.zeros((len(ITERATIONS), len(seeds), N_ROWS), dtype=np.int32)
    for i, it in enumerate(ITERATIONS):
        for e, s in enumerate(seeds):
            d = fresh_deck()
            ref_povs.shuffle(d, iterations=it, options=opts, seed=int(s))
            out[i, e] = d[:, 0]
    return out


def reference_numpy_episodes(reference_root: str, n_episodes: int) -> np.ndarray:
    chunks = np.array_split(np.arange(n_episodes), 16)
    ctx = mp.get_context("spawn")
    with ctx.Pool(min(8, mp.cpu_count())) as pool:
        parts = pool.map(_ref_numpy_chunk, [(reference_root, c.tolist()) for c in chunks])
    return np.concatenate(parts, axis=1)


def oracle_episodes(n_episodes: int, kind: str, mode: str = "uniform") -> np.ndarray:
    sys.path.insert(0, str(REPO))
    from oracle import api

    out = np.zeros((len(ITERATIONS), n_episodes, N_ROWS), dtype=np.int32)
    for i, it in enumerate(ITERATIONS):
        for s in range(n_episodes):
            d = fresh_deck()
            if kind == "library":
                api.shuffle(d, it, P, V, OFFSETS, s, mode)
            else:
                offs, assign, perms = api.refcuda_randomness(s, N_ROWS, P, V, OFFSETS, it)
                for t in range(it):
                    api.apply_iteration(d, P, V, int(offs[t]), assign[t], perms[t], sort_members=True)
            out[i, s] = d[:, 0]
    return out


def main(reference_root: str, n_episodes: int = 3000, reuse: bool = False) -> None:
    sys.path.insert(0, str(REPO))
    from oracle import metrics

    result: dict = {
        "workload": f"int32 deck {N_ROWS} x {WIDTH}, row i = i, V={V}, P={P}, offsets {OFFSETS}, "
        f"{n_episodes} episodes seeded 0..{n_episodes - 1}, iterations=it per episode",
        "iterations": ITERATIONS,
        "episodes": n_episodes,
    }
    sets = {
        "library": oracle_episodes(n_episodes, "library"),
        "library_reference_cuda": oracle_episodes(n_episodes, "library", "reference_cuda"),
        "library_reference_numpy": oracle_episodes(n_episodes, "library", "reference_numpy"),
        "reference_cuda": oracle_episodes(n_episodes, "reference_cuda"),
    }
    previous = json.loads(OUT.read_text()) if (reuse and OUT.exists()) else {}
    if "reference_numpy" in previous and previous.get("episodes") == n_episodes:
        result["reference_numpy"] = previous["reference_numpy"]
    elif (Path(reference_root) / "src" / "povs").exists():
        sets["reference_numpy"] = reference_numpy_episodes(reference_root, n_episodes)
    for name, eps in sets.items():
        result[name] = {
            "positional_tvd": [metrics.positional_tvd(eps[i]) for i in range(len(ITERATIONS))],
            "bigram_tvd": [metrics.bigram_tvd(eps[i]) for i in range(len(ITERATIONS))],
        }
    base = np.zeros((n_episodes, N_ROWS), dtype=np.int64)
    for s in range(n_episodes):
        a = np.arange(N_ROWS)
        np.random.default_rng(s).shuffle(a)
        base[s] = a
    result["numpy_shuffle"] = {"positional_tvd": metrics.positional_tvd(base), "bigram_tvd": metrics.bigram_tvd(base)}
    # Checksums of the library's episodes, so the GPU run can be compared exactly.
    for key in ("library", "library_reference_cuda", "library_reference_numpy"):
        tb = sets[key].astype(np.int64)
        result[f"{key}_checksums"] = [
            int((tb[i] * np.arange(1, N_ROWS + 1)).sum() % (2**61 - 1)) for i in range(len(ITERATIONS))
        ]
    OUT.write_text(json.dumps(result, indent=1) + "\n")
    print(json.dumps({k: v for k, v in result.items() if not k.endswith("_checksums")}, indent=1))


if __name__ == "__main__":
    flags = [a for a in sys.argv[1:] if a.startswith("--")]
    args = [a for a in sys.argv[1:] if not a.startswith("--")]
    if not args:
        sys.exit(__doc__.strip().splitlines()[-1])
    main(args[0], int(args[1]) if len(args) > 1 else 3000, reuse="--reuse" in flags)
