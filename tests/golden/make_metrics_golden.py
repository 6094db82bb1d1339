"""Generate known answers of the reference's bias metrics (tests/golden/metrics_golden.json).

Seeded episode sets (``numpy.random.default_rng(case)`` permutations, plus partially shuffled
ones so that the TVDs are far from zero) and the TVDs the reference's own metric module computes
for them: ``get_tvd`` and ``get_ngram_tvd`` for n = 2, 3, 4 and skip = 0, 1, 2
(src/povs/eval/metrics.py, imported from the reference checkout; it needs only NumPy).  Every
case stays below the reference's 512 MiB key budget, so no anchor subsampling is involved.

Usage: python tests/golden/make_metrics_golden.py <reference_root>   (the checkout holding src/povs)
"""

from __future__ import annotations

import importlib.util
import json
import sys
from pathlib import Path

import numpy as np

OUT = Path(__file__).resolve().parent / "metrics_golden.json"
CASES = [(3, 6), (7, 40), (50, 40), (101, 30), (256, 12)]  # (deck, episodes)


def episodes_for(case: int, deck: int, n_ep: int) -> np.ndarray:
    rng = np.random.default_rng(case)
    eps = np.tile(np.arange(deck, dtype=np.int64), (n_ep, 1))
    for e in range(n_ep):
        if e % 2 == 0:
            eps[e] = rng.permutation(deck)
        else:  # a few random transpositions: a visibly biased shuffle
            for _ in range(max(1, deck // 8)):
                i, j = rng.integers(0, deck, 2)
                eps[e, [i, j]] = eps[e, [j, i]]
    return eps


def main() -> None:
    if len(sys.argv) != 2:
        sys.exit(__doc__.strip().splitlines()[-1])
    root = Path(sys.argv[1])
    spec = importlib.util.spec_from_file_location("ref_metrics", root / "src/povs/eval/metrics.py")
    ref = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(ref)
    cases = []
    for case, (deck, n_ep) in enumerate(CASES):
        eps = episodes_for(case, deck, n_ep)
        entry = {"case": case, "deck": deck, "episodes": n_ep, "positional": ref.get_tvd(eps), "ngram": []}
        for n in (2, 3, 4):
            if deck - 1 < n - 1:
                continue
            for skip in (0, 1, 2):
                entry["ngram"].append({"n": n, "skip": skip, "tvd": ref.get_ngram_tvd(eps, n, skip=skip)})
        cases.append(entry)
    OUT.write_text(json.dumps({"generator": "tests/golden/make_metrics_golden.py", "cases": cases}, indent=1) + "\n")
    print(f"wrote {OUT} ({len(cases)} cases)")


if __name__ == "__main__":
    main()
