"""ORACLE - test infrastructure only.  ctypes wrappers of liboracle.so and of the
reference-compiled helper (oracle/_ref).  Only the tests, ``__graft_entry__.smoke`` and the
CPU-baseline leg of ``bench.py`` use this module; the product never does.
"""

from __future__ import annotations

import ctypes
import threading

import numpy as np

from . import build as _build

_lock = threading.Lock()
_lib: ctypes.CDLL | None = None
_ref: ctypes.CDLL | None = None
_ref_cuda: ctypes.CDLL | None = None

_P = ctypes.c_void_p


def lib() -> ctypes.CDLL:
    global _lib
    with _lock:
        if _lib is None:
            path = _build.ORACLE_LIB
            if not path.exists() or _build._stale(path, _build.C_SOURCES + _build.CXX_SOURCES):
                _build.build_oracle()
            L = ctypes.CDLL(str(path))
            L.oracle_philox4x32_10.argtypes = [_P, _P, _P]
            L.oracle_philox4x32_10.restype = None
            L.oracle_apply_iteration.argtypes = [_P, ctypes.c_int64, ctypes.c_int64, ctypes.c_int, ctypes.c_int,
                                                 ctypes.c_int64, _P, _P, ctypes.c_int]
            L.oracle_apply_iteration.restype = ctypes.c_int
            L.oracle_device_randomness.argtypes = [ctypes.c_uint64, ctypes.c_uint32, ctypes.c_int64, ctypes.c_int,
                                                   ctypes.c_int, _P, ctypes.c_int, _P, _P, _P, ctypes.c_int]
            L.oracle_device_randomness.restype = ctypes.c_int
            L.oracle_shuffle.argtypes = [_P, ctypes.c_int64, ctypes.c_int64, ctypes.c_int, ctypes.c_int, _P,
                                         ctypes.c_int, ctypes.c_int, ctypes.c_uint64, ctypes.c_int]
            L.oracle_shuffle.restype = ctypes.c_int
            L.oracle_shuffle_threads.argtypes = [_P, ctypes.c_int64, ctypes.c_int64, ctypes.c_int, ctypes.c_int, _P,
                                                 ctypes.c_int, ctypes.c_int, ctypes.c_uint64, ctypes.c_int]
            L.oracle_shuffle_threads.restype = ctypes.c_int
            L.oracle_assignment.argtypes = [ctypes.c_uint64, ctypes.c_uint32, ctypes.c_int64, _P]
            L.oracle_assignment.restype = None
            L.oracle_refcuda_randomness.argtypes = [ctypes.c_int32, ctypes.c_int64, ctypes.c_int32, ctypes.c_int32, _P,
                                                    ctypes.c_int32, ctypes.c_int32, _P, _P, _P]
            L.oracle_refcuda_randomness.restype = ctypes.c_int
            L.oracle_refcuda_perms.argtypes = [ctypes.c_int64, ctypes.c_int32, ctypes.c_int32, _P, _P, _P]
            L.oracle_refcuda_perms.restype = ctypes.c_int
            L.oracle_set_numpy_table.argtypes = [_P, _P, ctypes.c_int, ctypes.c_int, ctypes.c_int64]
            L.oracle_set_numpy_table.restype = None
            _lib = L
        return _lib


def ref_lib() -> ctypes.CDLL | None:
    """The reference-header helper, or None when it could not be built (no reference checkout)."""
    global _ref
    with _lock:
        if _ref is None:
            path = _build.build_ref()
            if path is None or not path.exists():
                return None
            R = ctypes.CDLL(str(path))
            R.ref_assign_sequence.argtypes = [ctypes.c_int32, ctypes.c_int64, ctypes.c_int32, ctypes.c_int32,
                                              ctypes.c_int32, ctypes.c_int32, _P, _P]
            R.ref_assign_sequence.restype = ctypes.c_int
            _ref = R
        return _ref


def ref_cuda_lib() -> ctypes.CDLL | None:
    """The reference's own CUDA path compiled for sm_100a (oracle/_ref/libref_povs_cuda.so), or None.

    Loading it needs no GPU; running it does.
    """
    global _ref_cuda
    with _lock:
        if _ref_cuda is None:
            path = _build.build_ref_cuda()
            if path is None or not path.exists():
                return None
            R = ctypes.CDLL(str(path))
            R.ref_povs_shapes.argtypes = [_P, ctypes.c_int32]
            R.ref_povs_shapes.restype = ctypes.c_int
            R.ref_povs_layout_check.argtypes = [ctypes.c_int32]
            R.ref_povs_layout_check.restype = ctypes.c_int
            R.ref_povs_layout_check_small_rows.argtypes = []
            R.ref_povs_layout_check_small_rows.restype = ctypes.c_int
            R.ref_povs_cuda.argtypes = [ctypes.c_int32, _P, ctypes.c_int64, _P, ctypes.c_int64, ctypes.c_int32,
                                        ctypes.c_int32, ctypes.c_int32]
            R.ref_povs_cuda.restype = ctypes.c_int
            R.ref_povs_kernel.argtypes = [ctypes.c_int32, _P, ctypes.c_int64, _P, _P, ctypes.c_int64, _P]
            R.ref_povs_kernel.restype = ctypes.c_int
            _ref_cuda = R
        return _ref_cuda


def ref_cuda_shapes() -> list[dict]:
    """Shapes the reference-built CUDA library instantiates: V, P, instance size, element bytes, block size."""
    R = ref_cuda_lib()
    if R is None:
        return []
    out = np.zeros(5 * 64, dtype=np.int32)
    n = R.ref_povs_shapes(out.ctypes.data, 64)
    keys = ("V", "P", "inst", "elem_bytes", "block")
    return [dict(zip(keys, (int(x) for x in out[5 * i:5 * i + 5])), index=i,
                 row_bytes=int(out[5 * i + 2] * out[5 * i + 3])) for i in range(n)]


def ref_cuda_shape(V: int, P: int, row_bytes: int) -> int | None:
    for sh in ref_cuda_shapes():
        if (sh["V"], sh["P"], sh["row_bytes"]) == (V, P, row_bytes):
            return sh["index"]
    return None


def ref_povs_cuda(shape: int, data_ptr: int, n_rows: int, offsets: list[int], iterations: int, seed: int,
                  device: int = 0) -> None:
    """The reference's CUDA host loop and kernel (povs.cu:356-467) on a device deck; synchronizes."""
    offs = np.array(offsets, dtype=np.int64)
    rc = ref_cuda_lib().ref_povs_cuda(shape, data_ptr, n_rows, offs.ctypes.data, len(offs), iterations, int(seed),
                                      device)
    if rc != 0:
        raise RuntimeError(f"ref_povs_cuda failed ({rc})")


def ref_povs_kernel(shape: int, data_ptr: int, n_rows: int, assign_ptr: int, seeds_ptr: int, offset: int,
                    stream: int = 0) -> None:
    """One launch of the reference kernel (povs.cu:116-349) with device assignments and seeds."""
    rc = ref_cuda_lib().ref_povs_kernel(shape, data_ptr, n_rows, assign_ptr, seeds_ptr, int(offset), stream or None)
    if rc != 0:
        raise RuntimeError(f"ref_povs_kernel failed ({rc})")


def _ptr(a: np.ndarray) -> int:
    assert a.flags.c_contiguous
    return a.ctypes.data


def block_counts(n_rows: int, pblock: int, vblock: int) -> tuple[int, int]:
    n_p = -(-n_rows // pblock)
    return n_p, -(-n_p // vblock)


def philox(ctr: tuple[int, int, int, int], key: tuple[int, int]) -> tuple[int, int, int, int]:
    c = np.array(ctr, dtype=np.uint32)
    k = np.array(key, dtype=np.uint32)
    out = np.zeros(4, dtype=np.uint32)
    lib().oracle_philox4x32_10(_ptr(c), _ptr(k), _ptr(out))
    return tuple(int(x) for x in out)


def as_rows(deck: np.ndarray) -> np.ndarray:
    """View a C-contiguous deck as (N, row_bytes) uint8."""
    assert deck.flags.c_contiguous
    return deck.reshape(deck.shape[0], -1).view(np.uint8).reshape(deck.shape[0], -1)


def apply_iteration(deck: np.ndarray, pblock: int, vblock: int, offset: int, assign: np.ndarray, perms: np.ndarray,
                    sort_members: bool) -> None:
    """One iteration with given randomness, in place on a C-contiguous host deck."""
    rows = as_rows(deck)
    n, r = rows.shape
    a = np.ascontiguousarray(assign, dtype=np.int64)
    p = np.ascontiguousarray(perms, dtype=np.int32)
    rc = lib().oracle_apply_iteration(_ptr(rows), n, r, pblock, vblock, int(offset), _ptr(a), _ptr(p),
                                      1 if sort_members else 0)
    if rc != 0:
        raise ValueError(f"oracle_apply_iteration failed ({rc})")


MODES = {"uniform": 0, "reference_cuda": 1, "reference_numpy": 2}

_np_tables: dict = {}


def _use_numpy_table(n_rows: int, pblock: int, vblock: int) -> None:
    """Hand the C oracle the NumPy path's per-vblock permutations for this geometry, built with NumPy
    itself: numpy.random.RandomState(s).shuffle(arange(n)) for s = 1..999 and every valid-row count n."""
    trunc = n_rows % pblock
    key = (pblock, vblock, trunc)
    if key not in _np_tables:
        sizes = [m * pblock for m in range(1, vblock + 1)]
        sizes += [(m - 1) * pblock + trunc if trunc else 0 for m in range(1, vblock + 1)]
        off = np.full(64, -1, dtype=np.int64)
        parts, at = [], 0
        for c, n in enumerate(sizes):
            if n <= 0:
                continue
            off[c] = at
            for s in range(1, 1000):
                a = np.arange(n, dtype=np.int32)
                np.random.RandomState(s).shuffle(a)
                parts.append(a)
            at += 999 * n
        _np_tables[key] = (np.ascontiguousarray(np.concatenate(parts)), off)
    table, off = _np_tables[key]
    lib().oracle_set_numpy_table(_ptr(table), _ptr(off), pblock, vblock, trunc)


def device_randomness(seed: int, iteration: int, n_rows: int, pblock: int, vblock: int,
                      offsets: list[int], mode: str = "uniform") -> tuple[int, np.ndarray, np.ndarray]:
    """The library's device randomness for one iteration: (offset, assign [n_v,V], perms [n_v,V*P])."""
    n_p, n_v = block_counts(n_rows, pblock, vblock)
    if mode == "reference_numpy":
        _use_numpy_table(n_rows, pblock, vblock)
    offs = np.array(offsets, dtype=np.int64)
    off = np.zeros(1, dtype=np.int64)
    assign = np.zeros((n_v, vblock), dtype=np.int64)
    perms = np.zeros((n_v, vblock * pblock), dtype=np.int32)
    rc = lib().oracle_device_randomness(seed & (2**64 - 1), iteration, n_rows, pblock, vblock, _ptr(offs), len(offs),
                                        _ptr(off), _ptr(assign), _ptr(perms), MODES[mode])
    if rc != 0:
        raise ValueError(f"oracle_device_randomness failed ({rc})")
    return int(off[0]), assign, perms


def shuffle(deck: np.ndarray, iterations: int, pblock: int, vblock: int, offsets: list[int], seed: int,
            mode: str = "uniform") -> None:
    """The library's full shuffle (device randomness of ``seed``), in place on a host deck."""
    rows = as_rows(deck)
    n, r = rows.shape
    if mode == "reference_numpy":
        _use_numpy_table(n, pblock, vblock)
    offs = np.array(offsets, dtype=np.int64)
    rc = lib().oracle_shuffle(_ptr(rows), n, r, pblock, vblock, _ptr(offs), len(offs), iterations,
                              seed & (2**64 - 1), MODES[mode])
    if rc != 0:
        raise ValueError(f"oracle_shuffle failed ({rc})")


def shuffle_threads(deck: np.ndarray, iterations: int, pblock: int, vblock: int, offsets: list[int], seed: int,
                    threads: int) -> None:
    """Same result as ``shuffle``, vblocks split over ``threads`` host threads (CPU baseline)."""
    rows = as_rows(deck)
    n, r = rows.shape
    offs = np.array(offsets, dtype=np.int64)
    rc = lib().oracle_shuffle_threads(_ptr(rows), n, r, pblock, vblock, _ptr(offs), len(offs), iterations,
                                      seed & (2**64 - 1), threads)
    if rc != 0:
        raise ValueError(f"oracle_shuffle_threads failed ({rc})")


def assignment(seed: int, iteration: int, n_slots: int) -> np.ndarray:
    out = np.zeros(n_slots, dtype=np.int64)
    lib().oracle_assignment(seed & (2**64 - 1), iteration, n_slots, _ptr(out))
    return out


def refcuda_randomness(seed: int, n_rows: int, pblock: int, vblock: int, offsets: list[int],
                       iterations: int) -> tuple[np.ndarray, np.ndarray, np.ndarray]:
    """Randomness of the reference's CUDA path: (offsets [it], assign [it,n_v,V], perms [it,n_v,V*P])."""
    n_p, n_v = block_counts(n_rows, pblock, vblock)
    offs = np.array(offsets, dtype=np.int64)
    out_off = np.zeros(iterations, dtype=np.int64)
    out_assign = np.zeros((iterations, n_v, vblock), dtype=np.int64)
    out_perms = np.zeros((iterations, n_v, vblock * pblock), dtype=np.int32)
    rc = lib().oracle_refcuda_randomness(int(seed), n_rows, pblock, vblock, _ptr(offs), len(offs), iterations,
                                         _ptr(out_off), _ptr(out_assign), _ptr(out_perms))
    if rc != 0:
        raise ValueError(f"oracle_refcuda_randomness failed ({rc})")
    return out_off, out_assign, out_perms


def refcuda_perms(n_rows: int, pblock: int, vblock: int, assign: np.ndarray, seeds: np.ndarray) -> np.ndarray:
    """The reference kernel's Stage 0 + Stage 2 for given members [n_v,V] and seeds [n_v]: perms [n_v,V*P]."""
    n_p, n_v = block_counts(n_rows, pblock, vblock)
    a = np.ascontiguousarray(assign, dtype=np.int64).reshape(n_v, vblock)
    s = np.ascontiguousarray(seeds, dtype=np.int32).reshape(n_v)
    out = np.zeros((n_v, vblock * pblock), dtype=np.int32)
    rc = lib().oracle_refcuda_perms(n_rows, pblock, vblock, _ptr(a), _ptr(s), _ptr(out))
    if rc != 0:
        raise ValueError(f"oracle_refcuda_perms failed ({rc})")
    return out


def ref_assign_sequence(seed: int, n_rows: int, pblock: int, vblock: int, n_offsets: int,
                        iterations: int) -> tuple[np.ndarray, np.ndarray] | None:
    """Assignment sequence and offset indices from the reference's compiled shuffle_array (None if unavailable)."""
    R = ref_lib()
    if R is None:
        return None
    n_p, n_v = block_counts(n_rows, pblock, vblock)
    out = np.zeros((iterations, n_v, vblock), dtype=np.int64)
    idx = np.zeros(iterations, dtype=np.int64)
    R.ref_assign_sequence(int(seed), n_rows, pblock, vblock, n_offsets, iterations, _ptr(out), _ptr(idx))
    return out, idx
