"""ctypes binding of the C ABI in include/povs.h (libpovs_sm100.so, built in tree).

This module is the only path to the GPU: if the library is missing or fails to load, every
call raises instead of falling back to another implementation.
"""

from __future__ import annotations

import ctypes
import os
import threading
from pathlib import Path

import torch

from . import _build

_LIB: ctypes.CDLL | None = None
_LOCK = threading.Lock()

POVS_OK = 0
ERRORS = {-1: "invalid argument", -2: "unsupported", -3: "CUDA error", -4: "device status"}

FLAG_NO_GRAPH = 1
FLAG_SYNC = 2
FLAG_REFERENCE_RNG = 4
FLAG_NO_PDL = 8
FLAG_REFERENCE_NUMPY = 16

# (name, restype, argtypes) of every exported symbol declared in include/povs.h.
_c_i32, _c_i64, _c_u32, _c_u64, _c_vp = ctypes.c_int32, ctypes.c_int64, ctypes.c_uint32, ctypes.c_uint64, ctypes.c_void_p
_P_I64 = ctypes.POINTER(ctypes.c_int64)
_P_I32 = ctypes.POINTER(ctypes.c_int32)
SIGNATURES: dict[str, tuple] = {
    "povs_shuffle_v1": (ctypes.c_int, [_c_vp, _c_i64, _c_i64, _P_I64, _c_i32, _c_i32, _c_i32, _c_i32, _c_u64, _c_i32, _c_vp, _c_u32]),
    "povs_shuffle_host_v1": (
        ctypes.c_int,
        [_c_vp, _c_vp, _c_i64, _c_i64, _P_I64, _c_i32, _c_i32, _c_i32, _c_i32, _c_u64, _c_i32, _c_vp, _c_u32],
    ),
    "povs_shuffle_host_batch_v1": (
        ctypes.c_int,
        [_c_vp, _c_i32, _c_vp, _c_i32, _c_i64, _c_i64, _P_I64, _c_i32, _c_i32, _c_i32, _c_i32,
         ctypes.POINTER(ctypes.c_uint64), _c_i32, _c_vp, _c_u32],
    ),
    "povs_apply_v1": (ctypes.c_int, [_c_vp, _c_i64, _c_i64, _c_i32, _c_i32, _c_i32, _P_I64, _c_vp, _c_vp, _c_i32, _c_i32, _c_vp]),
    "povs_device_status_v1": (ctypes.c_int, [_c_i32, _P_I32]),
    "povs_release_v1": (ctypes.c_int, []),
    "povs_last_error_string": (ctypes.c_char_p, []),
    "povs_version": (ctypes.c_int32, []),
    "povs_set_tuning_v1": (ctypes.c_int, [_c_i32, _c_i32, _c_i32, _c_i32, _c_i32, _c_i32]),
    "povs_set_pack_bytes_v1": (ctypes.c_int, [_c_i32]),
    "povs_enable_peer_access_v1": (ctypes.c_int, [_c_i32, _c_i32]),
    "povs_describe_plan_v1": (ctypes.c_int, [_c_vp, _c_i64, _c_i64, _c_i32, _c_i32, _c_i32, _P_I64, _c_i32]),
    "povs_plan_for_resources_v1": (
        ctypes.c_int,
        [_c_u64, _c_i64, _c_i64, _c_i32, _c_i32, _c_i32, _c_i32, _c_i32, _c_i32, _P_I64, _c_i32],
    ),
    "povs_shuffle_shards_v1": (
        ctypes.c_int,
        [_c_vp, _c_vp, _P_I64, _c_i32, _c_i64, _P_I64, _c_i32, _c_i32, _c_i32, _c_i32, _c_u64, _c_i32, _c_vp, _c_u32],
    ),
    "povs_shuffle_sharded_v1": (
        ctypes.c_int,
        [_c_vp, _c_vp, _P_I64, _c_i32, _c_i32, _c_i64, _P_I64, _c_i32, _c_i32, _c_i32, _c_i32, _c_u64, _c_vp, _c_u32,
         _c_i32, _c_vp, _c_u32],
    ),
    "povs_ipc_export_v1": (ctypes.c_int, [_c_vp, _c_i32, _c_vp, _P_I64]),
    "povs_ipc_import_v1": (ctypes.c_int, [_c_vp, _c_i64, _c_i32, ctypes.POINTER(_c_vp), ctypes.POINTER(_c_vp)]),
    "povs_ipc_close_v1": (ctypes.c_int, [_c_vp, _c_i32]),
    "povs_shuffle_mapped_v1": (
        ctypes.c_int,
        [_c_vp, _c_i64, _c_i64, _P_I64, _c_i32, _c_i32, _c_i32, _c_i32, _c_u64, _c_i32, _c_vp, _c_u32],
    ),
    "povs_shuffle_batch_v1": (
        ctypes.c_int,
        [_c_vp, _c_i64, _c_i64, _c_i64, _c_i64, _P_I64, _c_i32, _c_i32, _c_i32, _c_i32, _c_vp, _c_i32, _c_vp, _c_u32],
    ),
    "povs_travel_histogram_v1": (
        ctypes.c_int,
        [_c_vp, _c_i32, _c_i64, _c_i64, _c_i64, _c_i64, _c_i32, _c_i64, _c_vp, _c_i32, _c_vp],
    ),
    "povs_ngram_keys_v1": (
        ctypes.c_int,
        [_c_vp, _c_i32, _c_i64, _c_i64, _c_i64, _c_i64, _c_i32, _c_i64, _c_vp, _c_i64, _c_vp, _c_i32, _c_vp],
    ),
    "povs_ngram_count_v1": (
        ctypes.c_int,
        [_c_vp, _c_i32, _c_i64, _c_i64, _c_i64, _c_i64, _c_i32, _c_i64, _c_vp, _c_i64, _c_vp, _c_i64, _c_vp, _c_i64,
         _c_vp, _c_i64, _c_i32, _c_vp],
    ),
    "povs_numpy_path_perm_v1": (ctypes.c_int, [_c_u32, _c_i32, _c_vp]),
    "povs_set_peer_wait_limit_v1": (ctypes.c_int, [_c_u64]),
    "povs_apply_static_v1": (
        ctypes.c_int,
        [_c_vp, _c_i64, _c_i64, _c_i32, _c_i32, _c_i32, _P_I64, _c_vp, _c_vp, _c_i32, _c_i32, _c_vp, _c_u32],
    ),
}


def library_path() -> Path:
    return Path(os.environ.get("POVS_LIBRARY", str(_build.LIB_PATH)))


def load(build_if_missing: bool = False) -> ctypes.CDLL:
    """Load (once) the native library; optionally build it first if it is absent or stale."""
    global _LIB
    with _LOCK:
        if _LIB is not None:
            return _LIB
        path = library_path()
        if build_if_missing and "POVS_LIBRARY" not in os.environ and _build.is_stale():
            _build.build()
        if not path.exists():
            raise RuntimeError(
                f"povs native library not found at {path}; build it with `python -m povs._build` "
                "(requires nvcc with sm_100a support)"
            )
        lib = ctypes.CDLL(str(path))
        for name, (restype, argtypes) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = restype
            fn.argtypes = argtypes
        _LIB = lib
        return lib


def last_error() -> str:
    return load().povs_last_error_string().decode(errors="replace")


def check(code: int, what: str) -> None:
    if code < 0:
        raise RuntimeError(f"{what} failed ({ERRORS.get(code, code)}): {last_error()}")


def _i64_array(values) -> ctypes.Array:
    vals = [int(v) for v in values]
    return (ctypes.c_int64 * max(1, len(vals)))(*vals)


def current_stream_handle(device: torch.device) -> int:
    return int(torch.cuda.current_stream(device).cuda_stream)


def shuffle_device(
    data: torch.Tensor,
    row_bytes: int,
    offsets: list[int],
    iterations: int,
    pblock: int,
    vblock: int,
    seed: int,
    flags: int = 0,
) -> None:
    """Shuffle a contiguous CUDA tensor in place on its device's current stream."""
    lib = load()
    dev = data.device
    offs = _i64_array(offsets)
    code = lib.povs_shuffle_v1(
        ctypes.c_void_p(data.data_ptr()),
        data.shape[0],
        row_bytes,
        offs,
        len(offsets),
        iterations,
        pblock,
        vblock,
        seed,
        dev.index,
        ctypes.c_void_p(current_stream_handle(dev)),
        flags,
    )
    check(code, "povs_shuffle_v1")


def shuffle_batch(
    decks: torch.Tensor,
    row_bytes: int,
    offsets: list[int],
    iterations: int,
    pblock: int,
    vblock: int,
    seeds: torch.Tensor,
    flags: int = 0,
) -> None:
    """Shuffle every deck ``decks[d]`` (a contiguous CUDA tensor of shape (n_decks, rows, ...)) with
    seed ``seeds[d]`` (int64 CUDA tensor holding the 64-bit seeds), one launch per iteration."""
    lib = load()
    dev = decks.device
    assert seeds.is_cuda and seeds.dtype == torch.int64 and seeds.is_contiguous() and seeds.numel() == decks.shape[0]
    code = lib.povs_shuffle_batch_v1(
        ctypes.c_void_p(decks.data_ptr()), decks.shape[0], decks.stride(0) * decks.element_size(), decks.shape[1],
        row_bytes, _i64_array(offsets), len(offsets), iterations, pblock, vblock, ctypes.c_void_p(seeds.data_ptr()),
        dev.index, ctypes.c_void_p(current_stream_handle(dev)), flags,
    )
    check(code, "povs_shuffle_batch_v1")


def _episode_layout(ids: torch.Tensor) -> tuple[int, int, int, int]:
    assert ids.is_cuda and ids.dim() == 2 and ids.dtype in (torch.int32, torch.int64), \
        "episodes must be a 2-D int32/int64 CUDA tensor"
    return ids.element_size(), ids.shape[0], ids.shape[1], ids.stride(0)


def travel_histogram(ids: torch.Tensor, kind: int, step: int, counts: torch.Tensor) -> None:
    """Add the travel-distance histogram of the episodes ``ids`` (n_episodes, deck) to ``counts``
    (int64 CUDA tensor of ``deck`` bins): kind 0 positional, kind 1 2-gram with ``step``."""
    lib = load()
    id_bytes, n_ep, deck, ep_stride = _episode_layout(ids)
    assert counts.is_cuda and counts.dtype == torch.int64 and counts.numel() == deck and counts.is_contiguous()
    dev = ids.device
    code = lib.povs_travel_histogram_v1(
        ctypes.c_void_p(ids.data_ptr()), id_bytes, n_ep, deck, ep_stride, ids.stride(1), kind, step,
        ctypes.c_void_p(counts.data_ptr()), dev.index, ctypes.c_void_p(current_stream_handle(dev)),
    )
    check(code, "povs_travel_histogram_v1")


def ngram_keys(ids: torch.Tensor, n: int, step: int, positions: torch.Tensor | None = None) -> torch.Tensor:
    """int64 keys of every n-gram (anchored at ``positions`` or at every position) of every episode."""
    lib = load()
    id_bytes, n_ep, deck, ep_stride = _episode_layout(ids)
    dev = ids.device
    count = deck if positions is None else positions.numel()
    keys = torch.empty(n_ep * count, dtype=torch.int64, device=dev)
    if positions is not None:
        assert positions.is_cuda and positions.dtype == torch.int64 and positions.is_contiguous()
    code = lib.povs_ngram_keys_v1(
        ctypes.c_void_p(ids.data_ptr()), id_bytes, n_ep, deck, ep_stride, ids.stride(1), n, step,
        ctypes.c_void_p(positions.data_ptr()) if positions is not None else None, count if positions is not None else 0,
        ctypes.c_void_p(keys.data_ptr()), dev.index, ctypes.c_void_p(current_stream_handle(dev)),
    )
    check(code, "povs_ngram_keys_v1")
    return keys


def ngram_count(ids: torch.Tensor, n: int, step: int, positions: torch.Tensor | None = None,
                mult_bins: int = 1 << 16, overflow_cap: int = 1 << 20) -> tuple[np.ndarray, np.ndarray]:
    """Multiplicities of the distinct n-gram keys (``povs_ngram_count_v1``): ``mult`` (mult[c] =
    keys seen exactly c times, mult[0] = keys seen ``mult_bins`` times or more) and the counts of the
    latter, as NumPy arrays.  Raises if a key found no room in the table."""
    import numpy as np

    lib = load()
    id_bytes, n_ep, deck, ep_stride = _episode_layout(ids)
    dev = ids.device
    count = deck if positions is None else positions.numel()
    total = n_ep * count
    slots = 1
    while slots < 2 * total:
        slots <<= 1
    if positions is not None:
        assert positions.is_cuda and positions.dtype == torch.int64 and positions.is_contiguous()
    while True:
        table = torch.empty(2 * slots + 1, dtype=torch.int64, device=dev)
        mult = torch.empty(mult_bins, dtype=torch.int64, device=dev)
        overflow = torch.empty(max(1, overflow_cap), dtype=torch.int64, device=dev)
        code = lib.povs_ngram_count_v1(
            ctypes.c_void_p(ids.data_ptr()), id_bytes, n_ep, deck, ep_stride, ids.stride(1), n, step,
            ctypes.c_void_p(positions.data_ptr()) if positions is not None else None,
            count if positions is not None else 0, ctypes.c_void_p(table.data_ptr()), slots,
            ctypes.c_void_p(mult.data_ptr()), mult_bins, ctypes.c_void_p(overflow.data_ptr()), overflow_cap,
            dev.index, ctypes.c_void_p(current_stream_handle(dev)),
        )
        check(code, "povs_ngram_count_v1")
        del table
        m = mult.cpu().numpy().astype(np.uint64)
        if int(m[0]) <= overflow_cap:
            break
        overflow_cap = int(m[0])  # more keys above mult_bins than room: once more with room for all
    status = device_status(dev.index)
    if status:
        raise RuntimeError(f"device status 0x{status:x} after povs_ngram_count_v1 (8: the hash table was full)")
    return m, overflow[: int(m[0])].cpu().numpy().astype(np.uint64)


def shuffle_host(
    host_ptr: int,
    device_buffer: torch.Tensor,
    n_rows: int,
    row_bytes: int,
    offsets: list[int],
    iterations: int,
    pblock: int,
    vblock: int,
    seed: int,
    flags: int = 0,
) -> None:
    """Shuffle rows in host memory through ``device_buffer`` (blocks until the copy back is done)."""
    lib = load()
    dev = device_buffer.device
    offs = _i64_array(offsets)
    code = lib.povs_shuffle_host_v1(
        ctypes.c_void_p(host_ptr),
        ctypes.c_void_p(device_buffer.data_ptr()),
        n_rows,
        row_bytes,
        offs,
        len(offsets),
        iterations,
        pblock,
        vblock,
        seed,
        dev.index,
        ctypes.c_void_p(current_stream_handle(dev)),
        flags,
    )
    check(code, "povs_shuffle_host_v1")


def shuffle_mapped(
    host_ptr: int,
    n_rows: int,
    row_bytes: int,
    offsets: list[int],
    iterations: int,
    pblock: int,
    vblock: int,
    seed: int,
    device: int,
    flags: int = 0,
) -> None:
    """Shuffle rows that stay in host memory, through mapped page-locked memory (blocks until done)."""
    lib = load()
    dev = torch.device("cuda", device)
    code = lib.povs_shuffle_mapped_v1(
        ctypes.c_void_p(host_ptr), n_rows, row_bytes, _i64_array(offsets), len(offsets), iterations, pblock, vblock,
        seed, device, ctypes.c_void_p(current_stream_handle(dev)), flags,
    )
    check(code, "povs_shuffle_mapped_v1")


def shuffle_host_batch(
    host_ptrs: list[int],
    device_buffers: list[torch.Tensor],
    n_rows: int,
    row_bytes: int,
    offsets: list[int],
    iterations: int,
    pblock: int,
    vblock: int,
    seeds: list[int],
    flags: int = 0,
) -> None:
    """Pipelined shuffle of several host decks of one shape (blocks until all are back)."""
    lib = load()
    dev = device_buffers[0].device
    hp = (ctypes.c_void_p * len(host_ptrs))(*[ctypes.c_void_p(p) for p in host_ptrs])
    bp = (ctypes.c_void_p * len(device_buffers))(*[ctypes.c_void_p(b.data_ptr()) for b in device_buffers])
    sd = (ctypes.c_uint64 * max(1, len(seeds)))(*[int(x) & 0xFFFF_FFFF_FFFF_FFFF for x in seeds])
    code = lib.povs_shuffle_host_batch_v1(
        hp, len(host_ptrs), bp, len(device_buffers), n_rows, row_bytes, _i64_array(offsets), len(offsets),
        iterations, pblock, vblock, sd, dev.index, ctypes.c_void_p(current_stream_handle(dev)), flags,
    )
    check(code, "povs_shuffle_host_batch_v1")


def apply(
    data: torch.Tensor,
    row_bytes: int,
    pblock: int,
    vblock: int,
    offsets_per_iter: list[int],
    assign: torch.Tensor,
    perms: torch.Tensor,
    sort_members: bool,
) -> None:
    """Apply injected randomness (device int64 assign, device int32 perms) to a CUDA tensor."""
    lib = load()
    dev = data.device
    assert assign.dtype == torch.int64 and assign.is_cuda and assign.is_contiguous()
    assert perms.dtype == torch.int32 and perms.is_cuda and perms.is_contiguous()
    offs = _i64_array(offsets_per_iter)
    code = lib.povs_apply_v1(
        ctypes.c_void_p(data.data_ptr()),
        data.shape[0],
        row_bytes,
        pblock,
        vblock,
        len(offsets_per_iter),
        offs,
        ctypes.c_void_p(assign.data_ptr()),
        ctypes.c_void_p(perms.data_ptr()),
        1 if sort_members else 0,
        dev.index,
        ctypes.c_void_p(current_stream_handle(dev)),
    )
    check(code, "povs_apply_v1")


def apply_static(
    data: torch.Tensor,
    row_bytes: int,
    pblock: int,
    vblock: int,
    offsets_per_iter: list[int],
    assign_host,
    perms_host,
    sort_members: bool,
    flags: int = FLAG_SYNC,
) -> None:
    """Allocation-free injection: host int64 assign / int32 perms staged in the library's fixed scratch.

    For callers that may not allocate device memory (see include/povs.h); by default the call
    synchronizes the stream, so the host arrays may be reused as soon as it returns.
    """
    import numpy as np

    lib = load()
    dev = data.device
    a = np.ascontiguousarray(assign_host, dtype=np.int64)
    p = np.ascontiguousarray(perms_host, dtype=np.int32)
    offs = _i64_array(offsets_per_iter)
    code = lib.povs_apply_static_v1(
        ctypes.c_void_p(data.data_ptr()),
        data.shape[0],
        row_bytes,
        pblock,
        vblock,
        len(offsets_per_iter),
        offs,
        ctypes.c_void_p(a.ctypes.data),
        ctypes.c_void_p(p.ctypes.data),
        1 if sort_members else 0,
        dev.index,
        ctypes.c_void_p(current_stream_handle(dev)),
        flags,
    )
    check(code, "povs_apply_static_v1")


def _ptr_array(ptrs) -> ctypes.Array:
    return (ctypes.c_void_p * len(ptrs))(*[ctypes.c_void_p(int(p)) for p in ptrs])


def shuffle_shards(
    shard_ptrs: list[int],
    shard_rows: list[int],
    row_bytes: int,
    offsets: list[int],
    iterations: int,
    pblock: int,
    vblock: int,
    seed: int,
    device: int,
    flags: int = 0,
    scratch_ptrs: list[int] | None = None,
) -> None:
    """Shuffle a deck held in several shards addressable from ``device`` (one process).

    ``scratch_ptrs``: None (in place) or one buffer per shard of the same size (double-buffered).
    """
    lib = load()
    rows = _i64_array(shard_rows)
    code = lib.povs_shuffle_shards_v1(
        _ptr_array(shard_ptrs), _ptr_array(scratch_ptrs) if scratch_ptrs else None, rows, len(shard_ptrs), row_bytes, _i64_array(offsets), len(offsets), iterations,
        pblock, vblock, seed, device, ctypes.c_void_p(current_stream_handle(torch.device("cuda", device))), flags,
    )
    check(code, "povs_shuffle_shards_v1")


def shuffle_sharded(
    shard_ptrs: list[int],
    shard_rows: list[int],
    rank: int,
    row_bytes: int,
    offsets: list[int],
    iterations: int,
    pblock: int,
    vblock: int,
    seed: int,
    flag_ptrs: list[int],
    epoch_base: int,
    device: int,
    flags: int = 0,
    scratch_ptrs: list[int] | None = None,
) -> None:
    """This rank's part of a sharded shuffle (one process per GPU; see include/povs.h).

    ``scratch_ptrs``: None (in place) or one buffer per shard, mapped like the shards (double-buffered).
    """
    lib = load()
    code = lib.povs_shuffle_sharded_v1(
        _ptr_array(shard_ptrs), _ptr_array(scratch_ptrs) if scratch_ptrs else None, _i64_array(shard_rows), len(shard_ptrs), rank, row_bytes, _i64_array(offsets),
        len(offsets), iterations, pblock, vblock, seed, _ptr_array(flag_ptrs), epoch_base & 0xFFFFFFFF, device,
        ctypes.c_void_p(current_stream_handle(torch.device("cuda", device))), flags,
    )
    check(code, "povs_shuffle_sharded_v1")


def set_peer_wait_limit(seconds: float | None) -> None:
    """Time limit of the cross-GPU barrier of sharded shuffles (None: the default, 20 s)."""
    check(load().povs_set_peer_wait_limit_v1(0 if seconds is None else max(1, int(seconds * 1e9))),
          "povs_set_peer_wait_limit_v1")


def ipc_export(ptr: int, device: int) -> tuple[bytes, int]:
    """(64-byte IPC handle of the allocation holding ``ptr``, offset of ``ptr`` in it)."""
    lib = load()
    handle = (ctypes.c_uint8 * 64)()
    offset = ctypes.c_int64(0)
    check(lib.povs_ipc_export_v1(ctypes.c_void_p(ptr), device, handle, ctypes.byref(offset)), "povs_ipc_export_v1")
    return bytes(handle), int(offset.value)


def ipc_import(handle: bytes, offset: int, device: int) -> tuple[int, int]:
    """Map a peer's exported allocation; returns (pointer at offset, mapping base to close)."""
    lib = load()
    h = (ctypes.c_uint8 * 64).from_buffer_copy(handle)
    ptr, base = ctypes.c_void_p(), ctypes.c_void_p()
    check(lib.povs_ipc_import_v1(h, offset, device, ctypes.byref(ptr), ctypes.byref(base)), "povs_ipc_import_v1")
    return int(ptr.value), int(base.value)


def ipc_close(base: int, device: int) -> None:
    check(load().povs_ipc_close_v1(ctypes.c_void_p(base), device), "povs_ipc_close_v1")


def device_status(device: int) -> int:
    """Read and clear the sticky device status word (synchronizes the device)."""
    lib = load()
    out = ctypes.c_int32(0)
    check(lib.povs_device_status_v1(device, ctypes.byref(out)), "povs_device_status_v1")
    return int(out.value)


def set_tuning(
    stage_cap: int = 32 * 1024,
    n_stages: int = 8,
    movers: int = 4,
    permuters: int = 4,
    force_plain: bool = False,
    copy_bytes: int = 8192,
) -> None:
    """Process-wide launch tuning (see include/povs.h); the defaults restore the built-in plan."""
    check(
        load().povs_set_tuning_v1(stage_cap, n_stages, movers, permuters, int(force_plain), copy_bytes),
        "povs_set_tuning_v1",
    )


def enable_peer_access(device: int, peer: int) -> None:
    """Let kernels on ``device`` access ``peer``'s memory (idempotent)."""
    check(load().povs_enable_peer_access_v1(device, peer), "povs_enable_peer_access_v1")


def set_pack_bytes(pack_bytes: int = 16 * 1024) -> None:
    """Largest packed unit in bytes (0 = one vblock per unit); the default restores the built-in plan."""
    check(load().povs_set_pack_bytes_v1(pack_bytes), "povs_set_pack_bytes_v1")


PLAN_FIELDS = (
    "grid",
    "block",
    "smem",
    "sort_elems_per_lane",
    "bulk",
    "slab_bytes",
    "n_slabs",
    "stages_per_cta",
    "stage_bytes",
    "vec_bytes",
    "n_vblocks",
    "sm_count",
    "copy_rows",
    "perm_slots",
    "movers",
    "permuters",
    "vblocks_per_unit",
    "rows_per_unit",
    "wide_kernel",
    "chunked_kernel",
)

# B200 (sm_100a) resources for plan_for_resources: SMs, opt-in dynamic shared memory per block,
# shared memory per SM, threads per SM.
B200_RESOURCES = (148, 232448, 233472, 2048)


def describe_plan(data: torch.Tensor, row_bytes: int, pblock: int, vblock: int) -> dict[str, int]:
    lib = load()
    out = (ctypes.c_int64 * len(PLAN_FIELDS))()
    n = lib.povs_describe_plan_v1(
        ctypes.c_void_p(data.data_ptr()), data.shape[0], row_bytes, pblock, vblock, data.device.index, out, len(PLAN_FIELDS)
    )
    check(n, "povs_describe_plan_v1")
    return {k: int(out[i]) for i, k in enumerate(PLAN_FIELDS[:n])}


def plan_for_resources(n_rows: int, row_bytes: int, pblock: int, vblock: int,
                       resources: tuple[int, int, int, int] = B200_RESOURCES, address: int = 1 << 20) -> dict[str, int]:
    """The launch plan for a deck of n_rows x row_bytes at ``address`` on a device with ``resources``,
    computed on the host (no GPU needed)."""
    lib = load()
    out = (ctypes.c_int64 * len(PLAN_FIELDS))()
    n = lib.povs_plan_for_resources_v1(address, n_rows, row_bytes, pblock, vblock, *resources, out, len(PLAN_FIELDS))
    check(n, "povs_plan_for_resources_v1")
    return {k: int(out[i]) for i, k in enumerate(PLAN_FIELDS[:n])}


def release() -> None:
    if _LIB is not None:
        check(_LIB.povs_release_v1(), "povs_release_v1")
