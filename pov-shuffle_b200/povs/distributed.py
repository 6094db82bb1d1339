"""Decks split along axis 0 into shards: several tensors in one process, or one shard per GPU
process (torch.distributed, one process per GPU of a node).

The result is the same permutation as ``povs.shuffle`` on the concatenated deck with the same
seed: offsets, assignments and per-vblock permutations are functions of the seed and the global
indices only.  Options are resolved and validated against the whole deck.

One process per GPU (``ShardedDeck``): every rank maps the other ranks' shards with CUDA IPC at
construction, with a device barrier between iterations.  Two orders give the same result:

* double-buffered (default when every GPU has room for a scratch copy of its shard): every rank
  moves the pblocks stored in its own shard, reading them locally and storing each row straight
  into its destination slot in the other buffer (local or a peer's), so a row crosses NVLink at
  most once per iteration;
* in place (``double_buffer=False``, no extra memory): every rank runs the vblocks
  ``rank, rank + world, ...``, reading member rows from local or peer memory (bulk copies, no
  multicast) and writing them back with peer stores, so a remote row crosses twice.

The only collective on the data path is the broadcast of the seed from rank 0 (NCCL when the
group's backend is NCCL).
No reference counterpart: the reference has no multi-GPU code.
"""

from __future__ import annotations

import math
from typing import Any

import torch
import torch.distributed as dist

from . import _native
from .common import (
    _validate_offsets,
    _validate_pblock_size,
    _validate_vblock_size,
    choose_offsets,
    get_int_seed,
    randomness_flags,
    seed_to_u64,
)
from .constants import MIN_VBLOCK_SIZE
from .torch import _choose_pblock_size, _choose_thr_block_size, _validate_thr_block_size, options_is_complete
from .types import Options

MAX_SHARDS = 8
# Free device memory to leave next to a shard's scratch copy when double-buffering is automatic.
SCRATCH_HEADROOM_BYTES = 2 << 30


def _row_layout(t: torch.Tensor) -> tuple[tuple[int, ...], torch.dtype]:
    return tuple(t.shape[1:]), t.dtype


def resolve_options(
    n_rows: int, instance_size: int, dtype_bytes: int, device_id: int, options: Options | None
) -> Options:
    """Complete ``options`` for a deck of ``n_rows`` rows (same rules as ``optim_options_for_dataset``)."""
    options = options or Options()
    if options_is_complete(options):
        return options
    vblk = options.virtual_block_size or MIN_VBLOCK_SIZE
    pblk = options.physical_block_size or _choose_pblock_size(instance_size, dtype_bytes, vblk, device_id)
    return Options(
        virtual_block_size=vblk,
        physical_block_size=pblk,
        offsets=choose_offsets(n_rows, instance_size, dtype_bytes, pblk),
        gpu_thread_block_size=_choose_thr_block_size(instance_size, dtype_bytes, vblk, pblk, device_id),
        randomness=options.randomness,
    )


def validate(n_rows: int, instance_size: int, dtype_bytes: int, iterations: int, options: Options,
             shard_rows: list[int]) -> None:
    """Preflight of a sharded deck (``AssertionError`` like the single-tensor path)."""
    assert n_rows >= 2, f"dataset must have at least 2 instances, but has {n_rows}"
    assert iterations >= 1, f"iterations ({iterations}) must be at least 1"
    _validate_vblock_size(options.virtual_block_size)
    pblock = _validate_pblock_size(options.physical_block_size)
    _validate_offsets(options.offsets, n_rows, instance_size, dtype_bytes, pblock)
    _validate_thr_block_size(options.gpu_thread_block_size, options.physical_block_size, options.virtual_block_size)
    assert 1 <= len(shard_rows) <= MAX_SHARDS, f"between 1 and {MAX_SHARDS} shards are supported"
    assert min(shard_rows) >= pblock, f"every shard needs at least physical_block_size ({pblock}) rows"


def shuffle_shards(
    shards: list[torch.Tensor],
    iterations: int = 1,
    options: Options | None = None,
    seed: int | Any | None = None,
    scratch: list[torch.Tensor] | None = None,
) -> None:
    """Shuffle, in place, the deck formed by concatenating ``shards`` along axis 0 (one process).

    All shards must be contiguous and share the row layout and dtype; shards on other GPUs of the
    node are reached from the first shard's GPU over NVLink (peer access is enabled here).
    ``scratch``: optional buffers shaped like the shards, used for the double-buffered order
    (contents are overwritten).
    """
    assert shards, "at least one shard is required"
    layout = _row_layout(shards[0])
    for s in shards:
        assert isinstance(s, torch.Tensor) and s.is_cuda and s.is_contiguous(), "shards must be contiguous CUDA tensors"
        assert _row_layout(s) == layout, "shards must share the row shape and dtype"
    dev = shards[0].device
    instance_size = math.prod(layout[0]) if layout[0] else 1
    dtype_bytes = shards[0].element_size()
    rows = [int(s.shape[0]) for s in shards]
    n_rows = sum(rows)
    opts = resolve_options(n_rows, instance_size, dtype_bytes, dev.index, options)
    validate(n_rows, instance_size, dtype_bytes, iterations, opts, rows)
    row_bytes = instance_size * dtype_bytes
    if scratch is not None:
        assert len(scratch) == len(shards), "one scratch buffer per shard"
        for b, s in zip(scratch, shards):
            assert b.is_cuda and b.is_contiguous() and b.shape == s.shape and b.dtype == s.dtype, \
                "scratch buffers must be contiguous CUDA tensors shaped like their shards"
    if row_bytes == 0:
        return
    # Shards (and scratch buffers) on other GPUs of the node are reached over NVLink by the kernels
    # running on the first shard's GPU.
    for t in [*shards, *(scratch or [])]:
        if t.device.index != dev.index:
            _native.enable_peer_access(dev.index, t.device.index)
    _native.shuffle_shards(
        [s.data_ptr() for s in shards], rows, row_bytes, list(opts.offsets), iterations, opts.physical_block_size,
        opts.virtual_block_size, seed_to_u64(get_int_seed(seed, opts)), dev.index, randomness_flags(opts),
        scratch_ptrs=[b.data_ptr() for b in scratch] if scratch is not None else None,
    )


class ShardedDeck:
    """This rank's shard of a deck split across the GPUs of one node (one process per GPU).

    :param shard: this rank's rows, a contiguous CUDA tensor on this rank's GPU; every rank's shard
                  has the same row shape and dtype, and at least ``physical_block_size`` rows.
    :param group: process group (default: the world).  Construction is collective.
    :param double_buffer: allocate a scratch buffer the size of the shard and shuffle in the
                          double-buffered order (half the NVLink traffic of the in-place order);
                          None (default) does so when every rank's GPU has room for it.
    """

    def __init__(self, shard: torch.Tensor, group: dist.ProcessGroup | None = None, native: Any = None,
                 double_buffer: bool | None = None):
        self.native = native if native is not None else _native
        self.group = group
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        assert self.world <= MAX_SHARDS, f"at most {MAX_SHARDS} ranks are supported"
        assert shard.is_contiguous(), "Tensor must be contiguous"
        self.shard = shard
        self.device = shard.device
        if double_buffer is None:
            # Double-buffer when a scratch copy of the shard fits next to it (every rank must agree).
            room = True
            if shard.is_cuda:
                free, _ = torch.cuda.mem_get_info(shard.device)
                room = free >= shard.numel() * shard.element_size() + SCRATCH_HEADROOM_BYTES
        else:
            room = bool(double_buffer)
        meta = [None] * self.world
        dist.all_gather_object(meta, (int(shard.shape[0]), tuple(shard.shape[1:]), str(shard.dtype), room),
                               group=group)
        assert all(m[1:3] == meta[0][1:3] for m in meta), f"shards differ in row shape or dtype: {meta}"
        if double_buffer is None:
            double_buffer = all(m[3] for m in meta)
        else:
            assert all(m[3] == double_buffer for m in meta), "every rank must pass the same double_buffer"
        self.double_buffer = double_buffer
        self.shard_rows = [m[0] for m in meta]
        self.n_rows = sum(self.shard_rows)
        self.instance_size = math.prod(shard.shape[1:]) if shard.ndim > 1 else 1
        self.dtype_bytes = shard.element_size()
        self.row_bytes = self.instance_size * self.dtype_bytes
        # One uint32 barrier word per rank, zeroed; epochs only grow.
        self.flags = torch.zeros(self.world, dtype=torch.int32, device=self.device)
        self.scratch = torch.empty_like(shard) if double_buffer else None
        self.epoch = 0
        dev_index = self.device.index if self.device.type == "cuda" else -1
        mine = [self.native.ipc_export(shard.data_ptr(), dev_index),
                self.native.ipc_export(self.flags.data_ptr(), dev_index)]
        if self.scratch is not None:
            mine.append(self.native.ipc_export(self.scratch.data_ptr(), dev_index))
        handles = [None] * self.world
        dist.all_gather_object(handles, mine, group=group)
        self._mapped: list[int] = []
        self.shard_ptrs: list[int] = []
        self.flag_ptrs: list[int] = []
        self.scratch_ptrs: list[int] | None = [] if self.scratch is not None else None
        local = [shard.data_ptr(), self.flags.data_ptr()] + ([self.scratch.data_ptr()] if self.scratch is not None else [])
        for r, exported in enumerate(handles):
            if r == self.rank:
                ptrs = local
            else:
                ptrs = []
                for handle, offset in exported:
                    ptr, base = self.native.ipc_import(handle, offset, dev_index)
                    self._mapped.append(base)
                    ptrs.append(ptr)
            self.shard_ptrs.append(ptrs[0])
            self.flag_ptrs.append(ptrs[1])
            if self.scratch_ptrs is not None:
                self.scratch_ptrs.append(ptrs[2])
        dist.barrier(group=group)

    def options(self, options: Options | None = None) -> Options:
        """Options resolved against the whole deck."""
        return resolve_options(self.n_rows, self.instance_size, self.dtype_bytes, self.device.index or 0, options)

    def broadcast_seed(self, seed: int | Any | None, options: Options | None = None) -> int:
        """Rank 0's seed, on every rank (the one collective of a shuffle)."""
        value = get_int_seed(seed, options) if self.rank == 0 else 0
        t = torch.tensor([seed_to_u64(value) - (1 << 64) if seed_to_u64(value) >= (1 << 63) else seed_to_u64(value)],
                         dtype=torch.int64, device=self.device)
        dist.broadcast(t, src=dist.get_global_rank(self.group, 0) if self.group is not None else 0, group=self.group)
        return int(t.item()) & 0xFFFF_FFFF_FFFF_FFFF

    def shuffle(self, iterations: int = 1, options: Options | None = None, seed: int | Any | None = None,
                flags: int = 0) -> None:
        """Collective: every rank calls with the same iterations and options."""
        opts = self.options(options)
        validate(self.n_rows, self.instance_size, self.dtype_bytes, iterations, opts, self.shard_rows)
        seed_u64 = self.broadcast_seed(seed, opts)
        self.run(seed_u64, iterations, opts, flags)

    def run(self, seed_u64: int, iterations: int, opts: Options, flags: int = 0) -> None:
        """The iterations with a seed every rank already holds (no collective; every rank must call with
        the same arguments), on the current stream."""
        if self.row_bytes == 0:
            return
        self.native.shuffle_sharded(
            self.shard_ptrs, self.shard_rows, self.rank, self.row_bytes, list(opts.offsets), iterations,
            opts.physical_block_size, opts.virtual_block_size, seed_u64, self.flag_ptrs, self.epoch,
            self.device.index if self.device.type == "cuda" else -1, flags | randomness_flags(opts),
            scratch_ptrs=self.scratch_ptrs,
        )
        self.epoch += iterations + 1

    def close(self) -> None:
        """Unmap the peers' memory (collective: no rank may still be using this rank's mappings)."""
        if self.device.type == "cuda":
            torch.cuda.synchronize(self.device)
        dist.barrier(group=self.group)
        for base in self._mapped:
            self.native.ipc_close(base, self.device.index if self.device.type == "cuda" else -1)
        self._mapped = []


def shuffle_host_shards(decks: list[ShardedDeck], host_shards: list[torch.Tensor], iterations: int = 1,
                        options: Options | None = None, seed: int | Any | None = None) -> None:
    """Collective: stream this rank's host shards of several decks through sharded GPU buffers.

    Host shard ``k`` (a CPU tensor shaped like the decks' shards; pin it for overlap) is copied into
    ``decks[k % len(decks)]``, shuffled as that deck with seed ``s + k`` (``s`` is rank 0's seed), and
    copied back in place, on three streams ordered by events: deck k+1's copy in overlaps deck k's
    iterations and copy out, so each GPU's PCIe link carries both directions at once.  A host shard
    listed twice is shuffled twice in order.  Every rank calls with the same number of host shards,
    iterations and options; the seed is broadcast once (the only collective), and each deck's first
    device barrier orders a shuffle after every rank's copy in, which itself waits for that buffer's
    previous copy out.  Returns when every host shard is back.  Addition to the reference API (the
    sharded counterpart of ``povs.shuffle_many``).
    """
    assert decks and host_shards is not None, "at least one deck is required"
    d0 = decks[0]
    for d in decks:
        assert d.shard.shape == d0.shard.shape and d.shard.dtype == d0.shard.dtype and d.device == d0.device, \
            "the decks must have the same shard shape, dtype and device"
        assert d.shard_rows == d0.shard_rows, "the decks must be split the same way"
    for h in host_shards:
        assert isinstance(h, torch.Tensor) and not h.is_cuda and h.is_contiguous(), "host shards must be contiguous CPU tensors"
        assert h.shape == d0.shard.shape and h.dtype == d0.shard.dtype, "host shards must be shaped like the decks' shards"
    opts = d0.options(options)
    validate(d0.n_rows, d0.instance_size, d0.dtype_bytes, iterations, opts, d0.shard_rows)
    base = d0.broadcast_seed(seed, opts)
    if not host_shards:
        return
    nd = len(decks)
    dev = d0.device
    if dev.type != "cuda":
        # Decks in host memory (the native layer's own checks then decide): one step after another.
        for k, h in enumerate(host_shards):
            deck = decks[k % nd]
            deck.shard.copy_(h)
            deck.run((base + k) & 0xFFFF_FFFF_FFFF_FFFF, iterations, opts)
            h.copy_(deck.shard)
        return
    caller = torch.cuda.current_stream(dev)
    s_in, s_cmp, s_out = (torch.cuda.Stream(dev) for _ in range(3))
    for st in (s_in, s_cmp, s_out):
        st.wait_stream(caller)
    out_done: list[torch.cuda.Event] = []
    last_use: dict[int, int] = {}
    for k, h in enumerate(host_shards):
        deck = decks[k % nd]
        with torch.cuda.stream(s_in):
            if k >= nd:
                s_in.wait_event(out_done[k - nd])
            prev = last_use.get(h.data_ptr())
            if prev is not None:
                s_in.wait_event(out_done[prev])
            last_use[h.data_ptr()] = k
            deck.shard.copy_(h, non_blocking=True)
            in_done = torch.cuda.Event()
            in_done.record(s_in)
        with torch.cuda.stream(s_cmp):
            s_cmp.wait_event(in_done)
            deck.run((base + k) & 0xFFFF_FFFF_FFFF_FFFF, iterations, opts)
            cmp_done = torch.cuda.Event()
            cmp_done.record(s_cmp)
        with torch.cuda.stream(s_out):
            s_out.wait_event(cmp_done)
            h.copy_(deck.shard, non_blocking=True)
            done = torch.cuda.Event()
            done.record(s_out)
            out_done.append(done)
    for st in (s_in, s_cmp, s_out):
        caller.wait_stream(st)
    caller.synchronize()
