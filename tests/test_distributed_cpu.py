"""Host-side logic of the one-process-per-GPU sharded mode, with two gloo ranks on CPU.

The native layer is replaced by a recorder, so no GPU is touched: the test checks the collective
set-up (row table, handle exchange), that every rank uses rank 0's seed, the epoch bookkeeping of
the device barrier, option resolution against the whole deck, and the preflight errors.
"""

from __future__ import annotations

import os
import sys
from pathlib import Path

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

REPO = Path(__file__).resolve().parent.parent


class RecordingNative:
    def __init__(self):
        self.calls = []

    def ipc_export(self, ptr, device):
        return (bytes([dist.get_rank()]) * 64, 0)

    def ipc_import(self, handle, offset, device):
        return (1000 + handle[0], 2000 + handle[0])

    def ipc_close(self, base, device):
        self.calls.append(("close", base))

    def shuffle_sharded(self, *args, scratch_ptrs=None):
        self.calls.append(("shuffle", args, scratch_ptrs))


def _worker(rank: int, world: int, port: int, out_dir: str):
    sys.path[:0] = [str(REPO), str(REPO / "pov-shuffle_b200")]
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    import povs
    from povs.distributed import ShardedDeck

    rows = [40, 56][rank]
    shard = torch.zeros((rows, 4), dtype=torch.float32)
    native = RecordingNative()
    deck = ShardedDeck(shard, native=native)
    opts = povs.Options(virtual_block_size=2, physical_block_size=16, offsets=[0, 4, 8], gpu_thread_block_size=32)
    deck.shuffle(iterations=3, options=opts, seed=11 if rank == 0 else 999)
    deck.shuffle(iterations=2, options=opts, seed=12 if rank == 0 else 5)
    errors = []
    try:
        deck.shuffle(iterations=1, options=opts._replace(physical_block_size=64), seed=1)
    except AssertionError as e:
        errors.append(str(e))
    deck.close()
    # Ranks that disagree on double_buffer are told so on every rank (collective check).
    try:
        ShardedDeck(shard, native=RecordingNative(), double_buffer=(rank == 0))
    except AssertionError as e:
        errors.append(str(e))
    in_place = ShardedDeck(shard, native=RecordingNative(), double_buffer=False)
    errors.append(f"in_place scratch={in_place.scratch_ptrs}")
    # Host shards through two decks: one seed broadcast, step k uses rank 0's seed + k on deck k % 2.
    streamed = [ShardedDeck(torch.zeros_like(shard), native=RecordingNative(), double_buffer=False) for _ in range(2)]
    hosts = [torch.full_like(shard, float(d)) for d in range(3)]
    povs.shuffle_host_shards(streamed, hosts, iterations=2, options=opts, seed=40 if rank == 0 else 1)
    host_calls = [[(c[1][8], c[1][10]) for c in d.native.calls if c[0] == "shuffle"] for d in streamed]
    calls = [c for c in native.calls if c[0] == "shuffle"]
    result = {
        "shard_rows": deck.shard_rows,
        "n_rows": deck.n_rows,
        "shard_ptrs": deck.shard_ptrs,
        "seeds": [c[1][8] for c in calls],
        "epochs": [c[1][10] for c in calls],
        "ranks": [c[1][2] for c in calls],
        "scratch": [c[2] for c in calls],
        "errors": errors,
        "closed": len([c for c in native.calls if c[0] == "close"]),
        "host_calls": host_calls,
    }
    torch.save(result, os.path.join(out_dir, f"rank{rank}.pt"))
    dist.destroy_process_group()


def test_two_rank_control_plane(tmp_path):
    port = 29500 + (os.getpid() % 2000)
    mp.start_processes(_worker, args=(2, port, str(tmp_path)), nprocs=2, start_method="spawn", join=True)
    r0 = torch.load(tmp_path / "rank0.pt")
    r1 = torch.load(tmp_path / "rank1.pt")
    for r, res in enumerate((r0, r1)):
        assert res["shard_rows"] == [40, 56] and res["n_rows"] == 96
        assert res["ranks"] == [r, r]
        assert res["epochs"] == [0, 4], "epoch base advances by iterations + 1 per shuffle"
        assert res["seeds"] == [11, 12], "every rank uses rank 0's seed"
        assert res["errors"] and "at least physical_block_size" in res["errors"][0]
        assert "same double_buffer" in res["errors"][1] and res["errors"][2] == "in_place scratch=None"
        assert res["closed"] == 3, "shard, barrier flags and scratch of the one peer are unmapped"
        assert len(res["scratch"]) == 2 and all(len(p) == 2 for p in res["scratch"])
        assert res["host_calls"] == [[(40, 0), (42, 3)], [(41, 0)]], \
            "host shard k: rank 0's seed + k on deck k % 2, each deck's epochs advancing on their own"
    assert r0["shard_ptrs"][1] == 1000 + 1 and r1["shard_ptrs"][0] == 1000 + 0
