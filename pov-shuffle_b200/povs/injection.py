"""Injected randomness: run the B200 kernels with offsets, assignments and permutations chosen
by the caller instead of the device RNG.

This is the hook that makes the GPU path comparable bit for bit with any other implementation
of the algorithm (the reference's CUDA path draws them on the host with std::mt19937,
src/povs/__cuda/lib/povs.cu:396-430; its NumPy path with numpy generators,
src/povs/numpy.py:43-58).
"""

from __future__ import annotations

import numpy as np
import torch

from . import _native
from .common import get_block_counts, get_dtype_bytes, get_instance_size


def _as_int_array(x, dtype) -> np.ndarray:
    if isinstance(x, torch.Tensor):
        x = x.detach().cpu().numpy()
    return np.ascontiguousarray(np.asarray(x), dtype=dtype)


def _validate(n_rows: int, pblock: int, vblock: int, assign: np.ndarray, perms: np.ndarray, sort_members: bool) -> None:
    n_p, n_v = get_block_counts(n_rows, pblock, vblock)
    for t in range(assign.shape[0]):
        ids = assign[t].reshape(-1)
        valid = ids[(ids >= 0) & (ids < n_p)]
        if valid.size != n_p or not np.array_equal(np.sort(valid), np.arange(n_p)):
            raise ValueError(f"iteration {t}: the assignment must place every pblock 0..{n_p - 1} exactly once")
        for v in range(n_v):
            members = assign[t, v]
            rows = [min(pblock, n_rows - b * pblock) for b in members if 0 <= b < n_p]
            n_valid = int(sum(rows))
            pv = perms[t, v, :n_valid]
            if not np.array_equal(np.sort(pv), np.arange(n_valid)):
                raise ValueError(f"iteration {t}, vblock {v}: perms[:{n_valid}] must be a permutation of 0..{n_valid - 1}")


def apply_randomness(
    data: torch.Tensor,
    offsets: list[int] | np.ndarray,
    assign,
    perms,
    physical_block_size: int,
    virtual_block_size: int,
    sort_members: bool = True,
    validate: bool = True,
) -> None:
    """Run ``len(offsets)`` POV iterations on a CUDA tensor with the given randomness.

    :param data: Contiguous CUDA tensor (rows along axis 0, any dtype).
    :param offsets: Row offset of each iteration.
    :param assign: int array [iterations, n_v, V] of pblock ids per vblock slot; ids < 0 or >= n_p are padding.
    :param perms: int array [iterations, n_v, V*P]; destination slot f of a vblock receives source slot perms[f].
    :param sort_members: True orders each vblock's members ascending with padding last (the reference's
                         CUDA path); False keeps the given order (its NumPy path), placing padding last and a
                         truncated last pblock after the full ones.
    :param validate: Check on the host that assignments are partitions and permutations are permutations.
    """
    assert isinstance(data, torch.Tensor) and data.is_cuda, "data must be a CUDA tensor"
    assert data.is_contiguous(), "Tensor must be contiguous"
    n_rows = data.shape[0]
    pblock, vblock = int(physical_block_size), int(virtual_block_size)
    n_p, n_v = get_block_counts(n_rows, pblock, vblock)
    offs = [int(o) for o in offsets]
    iters = len(offs)
    a = _as_int_array(assign, np.int64).reshape(iters, n_v, vblock)
    p = _as_int_array(perms, np.int32).reshape(iters, n_v, vblock * pblock)
    if validate:
        _validate(n_rows, pblock, vblock, a, p, sort_members)
    row_bytes = get_instance_size(data) * get_dtype_bytes(data)
    if iters == 0 or row_bytes == 0:
        return
    dev = data.device
    a_dev = torch.from_numpy(a).to(dev)
    p_dev = torch.from_numpy(p).to(dev)
    _native.apply(data, row_bytes, pblock, vblock, offs, a_dev, p_dev, sort_members)
    # Keep the injected buffers alive until the kernels that read them have run.
    torch.cuda.current_stream(dev).synchronize()
