"""ORACLE - test infrastructure only.

Replay of the randomness of the reference's NumPy path (src/povs/numpy.py:43-61 and
:120-136), producing the offsets, assignments and per-vblock permutations that the reference
draws, in the form the B200 kernels accept for injection (``povs_apply_v1`` with
``sort_members = 0``):

  rng = numpy.random.default_rng(seed)                       numpy.py:43
  per iteration:
    ids = arange(n_v * V); rng.shuffle(ids)                    numpy.py:53-55 (ids >= n_p are padding)
    seeds = rng.integers(1, 1000, size=n_v)                    numpy.py:57
    offset = offsets[rng.integers(0, len(offsets))]            numpy.py:58
    vblock v: valid members in ``ids`` order, rows concatenated; the rows are permuted by
    RandomState(seeds[v]).shuffle, i.e. new[k] = old[p[k]] with p = arange(n) shuffled by
    the same RandomState                                       numpy.py:125-136
    vblock 0 is processed twice: ``np.vectorize`` without ``otypes`` calls the worker on the
    first element once more to infer the output type (numpy.py:61), so vblock 0 receives p[p].

The NumPy generators are called directly (they are the third-party arithmetic of this path).
Valid only when every pblock is full (N % P == 0): the reference's NumPy path misplaces rows
when a truncated pblock is not the last member of its vblock.
"""

from __future__ import annotations

import numpy as np


class CorruptingDraw(ValueError):
    """The reference's NumPy path loses or duplicates rows for this draw (not a permutation)."""


def _effective_vblock_perm(members: list[int], n_rows: int, pblock: int, p: np.ndarray) -> np.ndarray:
    """Source slot of every destination slot, in the slot layout of ``sort_members = 0``.

    ``members`` are the vblock's ids in ``bids`` order, padding included (ids < 0 or >= n_p are
    padding).  The reference writes chunk ``local[i*P:(i+1)*P]`` to the member at position ``i``
    of ``bids`` (padding counted), capped at the member's row count (numpy.py:133-136,
    _safe_set_arr numpy.py:158-172); rows past the chunk keep their content.
    """
    n_p = -(-n_rows // pblock)
    valid = [(i, b) for i, b in enumerate(members) if 0 <= b < n_p]
    rows = {b: min(pblock, n_rows - b * pblock) for _, b in valid}
    # Slot layout of the injected mode: full members in given order, then the truncated one.
    order = sorted(valid, key=lambda ib: (rows[ib[1]] < pblock, ib[0]))
    slot_of = {b: r * pblock for r, (_, b) in enumerate(order)}
    # local index -> slot (local = valid members' rows concatenated in bids order)
    local_slot = [slot_of[b] + j for _, b in valid for j in range(rows[b])]
    n_valid = len(local_slot)
    src = np.empty(n_valid, dtype=np.int64)
    for i, b in valid:
        chunk_len = max(0, min(pblock, n_valid - i * pblock))
        write_len = min(chunk_len, rows[b])
        for j in range(rows[b]):
            dst = slot_of[b] + j
            src[dst] = local_slot[p[i * pblock + j]] if j < write_len else dst
    if not np.array_equal(np.sort(src), np.arange(n_valid)):
        raise CorruptingDraw("the reference's NumPy path does not permute this vblock")
    return src


def numpy_path_randomness(seed: int, n_rows: int, pblock: int, vblock: int, offsets: list[int],
                          iterations: int) -> tuple[np.ndarray, np.ndarray, np.ndarray]:
    """(offsets [it], assign [it, n_v, V], perms [it, n_v, V*P]) of the reference's NumPy path.

    Raises ``CorruptingDraw`` when the reference itself would lose rows for this seed.
    """
    n_p = -(-n_rows // pblock)
    n_v = -(-n_p // vblock)
    vp = vblock * pblock
    rng = np.random.default_rng(seed)
    out_off = np.zeros(iterations, dtype=np.int64)
    out_assign = np.zeros((iterations, n_v, vblock), dtype=np.int64)
    out_perms = np.full((iterations, n_v, vp), -1, dtype=np.int32)
    for it in range(iterations):
        ids = np.arange(n_v * vblock)
        rng.shuffle(ids)
        ids = ids.reshape(n_v, vblock)
        seeds = rng.integers(1, 1000, size=n_v)
        out_off[it] = offsets[rng.integers(0, len(offsets))]
        out_assign[it] = ids
        for v in range(n_v):
            members = [int(b) for b in ids[v]]
            n_valid = sum(min(pblock, n_rows - b * pblock) for b in members if b < n_p)
            p = np.arange(n_valid)
            np.random.RandomState(seed=seeds[v]).shuffle(p)
            m = _effective_vblock_perm(members, n_rows, pblock, p)
            if v == 0:
                m = m[m]
            out_perms[it, v, :n_valid] = m
    return out_off, out_assign, out_perms
