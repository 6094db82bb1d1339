"""Generate the bias statistics of the reference's own CUDA kernel (tests/golden/bias_refcuda_kernel.json).

Needs a B200 and ``oracle/_ref/libref_povs_cuda.so`` (the reference's src/povs/__cuda/lib/povs.cu
compiled by oracle/build.py).  The reference's kernel cannot run the bias suite's P = 8 (its thread
block must hold 32 to P * V threads), so this suite uses the nearest shape it instantiates:

Workload: a deck of 1000 rows x 64 bytes (16 int32 values, row i filled with i; moved by the
reference as 32 two-byte values), V = 2, P = 16 (63 pblocks, the last one 8 rows, one padding
slot), offsets from the reference's chooser (0..15); 3000 episodes seeded 0..2999; for every
it = 1..8 each episode shuffles a fresh deck with ``iterations=it``, ``seed=episode``.  Column 0 of
the shuffled deck is the episode.

Recorded, per iteration count:
* ``reference_cuda_kernel``  - positional and bigram TVD of the reference's CUDA path (its host
                               loop and kernel, povs.cu:356-467), with checksums of its episodes;
* ``restatement_checksums``  - the same episodes from the oracle's restatement (oracle/ref_cuda_rng.cpp
                               randomness applied by the C oracle): equal to the kernel's;
* ``library_reference_cuda`` / ``library`` - this library's ``randomness="reference_cuda"`` and
                               default modes on the same workload (batched launches);
* ``subset_checksums``       - checksums of the first 200 episodes at it = 1..3, for a CPU check.

Usage: python tests/golden/make_refcuda_kernel_bias.py [episodes]
"""

from __future__ import annotations

import json
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
REPO = HERE.parent.parent
for _p in (REPO, REPO / "pov-shuffle_b200"):
    if str(_p) not in sys.path:
        sys.path.insert(0, str(_p))
OUT = HERE / "bias_refcuda_kernel.json"

N_ROWS, WIDTH, V, P = 1000, 16, 2, 16
ROW_BYTES = WIDTH * 4
ITERATIONS = list(range(1, 9))
SUBSET = 200


def offsets() -> list[int]:
    from povs.common import choose_offsets

    return choose_offsets(N_ROWS, WIDTH, 4, P)


def checksum(col0: np.ndarray) -> int:
    """Position-weighted sum of the episodes' ids, mod 2^61 - 1 (order sensitive)."""
    c = np.asarray(col0, dtype=np.int64)
    return int((c * np.arange(1, c.shape[-1] + 1)).sum() % (2**61 - 1))


def fresh_deck() -> np.ndarray:
    return np.repeat(np.arange(N_ROWS, dtype=np.int32)[:, None], WIDTH, axis=1)


def reference_kernel_episodes(it: int, n_episodes: int) -> np.ndarray:
    """Episodes of the reference's CUDA path: one povs_cuda call per episode on its own deck."""
    import torch

    from oracle import api

    shape = api.ref_cuda_shape(V, P, ROW_BYTES)
    assert shape is not None and api.ref_cuda_lib().ref_povs_layout_check(shape) == 0
    decks = torch.from_numpy(fresh_deck()).to("cuda:0")[None].repeat(n_episodes, 1, 1).contiguous()
    torch.cuda.synchronize()
    offs = offsets()
    for s in range(n_episodes):
        api.ref_povs_cuda(shape, decks[s].data_ptr(), N_ROWS, offs, it, s)
    flat = decks.cpu().numpy()
    assert (flat == flat[:, :, :1]).all(), "rows were torn"
    return flat[:, :, 0].astype(np.int64)


def restated_episodes(it: int, seeds) -> np.ndarray:
    """The same episodes from the oracle's restatement, on the CPU."""
    from oracle import api

    seeds = list(seeds)
    out = np.zeros((len(seeds), N_ROWS), dtype=np.int64)
    for k, s in enumerate(seeds):
        d = fresh_deck()
        offs, assign, perms = api.refcuda_randomness(s, N_ROWS, P, V, offsets(), it)
        for t in range(it):
            api.apply_iteration(d, P, V, int(offs[t]), assign[t], perms[t], sort_members=True)
        out[k] = d[:, 0]
    return out


def library_episodes(it: int, n_episodes: int, randomness: str) -> np.ndarray:
    import torch

    import povs
    from povs import _native

    decks = torch.from_numpy(fresh_deck()).to("cuda:0")[None].repeat(n_episodes, 1, 1).contiguous()
    seeds = torch.arange(n_episodes, dtype=torch.int64, device="cuda:0")
    flags = _native.FLAG_REFERENCE_RNG if randomness == "reference_cuda" else 0
    _native.shuffle_batch(decks, ROW_BYTES, offsets(), it, P, V, seeds, flags)
    torch.cuda.synchronize()
    povs.check_device_status(0)
    return decks.cpu().numpy()[:, :, 0].astype(np.int64)


def main(n_episodes: int = 3000) -> None:
    from oracle import metrics

    result: dict = {
        "workload": f"deck {N_ROWS} x {ROW_BYTES} B (int32 x {WIDTH}, row i = i), V={V}, P={P}, offsets {offsets()}, "
        f"{n_episodes} episodes seeded 0..{n_episodes - 1}, iterations=it per episode",
        "iterations": ITERATIONS,
        "episodes": n_episodes,
        "subset_episodes": SUBSET,
    }
    stats = {name: {"positional_tvd": [], "bigram_tvd": []} for name in
             ("reference_cuda_kernel", "library_reference_cuda", "library")}
    kernel_sums, restated_sums, subset_sums = [], [], []
    for it in ITERATIONS:
        eps = reference_kernel_episodes(it, n_episodes)
        kernel_sums.append(checksum(eps))
        restated = restated_episodes(it, range(n_episodes))
        restated_sums.append(checksum(restated))
        if it <= 3:
            subset_sums.append(checksum(eps[:SUBSET]))
        sets = {"reference_cuda_kernel": eps, "library_reference_cuda": library_episodes(it, n_episodes, "reference_cuda"),
                "library": library_episodes(it, n_episodes, "uniform")}
        for name, e in sets.items():
            assert (np.sort(e, axis=1) == np.arange(N_ROWS)).all(), f"{name}: not a permutation"
            stats[name]["positional_tvd"].append(metrics.positional_tvd(e))
            stats[name]["bigram_tvd"].append(metrics.bigram_tvd(e))
        print(f"it={it}: " + ", ".join(f"{k} {v['positional_tvd'][-1]:.5f}" for k, v in stats.items()), flush=True)
    result.update(stats)
    result["reference_cuda_kernel_checksums"] = kernel_sums
    result["restatement_checksums"] = restated_sums
    result["subset_checksums"] = subset_sums
    OUT.write_text(json.dumps(result, indent=1) + "\n")
    print(f"wrote {OUT}; restatement == kernel: {kernel_sums == restated_sums}")


if __name__ == "__main__":
    main(int(sys.argv[1]) if len(sys.argv) > 1 else 3000)
