"""Sharded mode across GPUs (one process per GPU, NCCL for the seed broadcast only).

Runs when at least two GPUs are visible: each rank holds a shard of one deck, and the
concatenation of the shuffled shards must equal the oracle's shuffle of the whole deck.
NVLS is switched off for these child processes.
"""

from __future__ import annotations

import os
import sys
from datetime import timedelta
from pathlib import Path

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

REPO = Path(__file__).resolve().parent.parent
pytestmark = pytest.mark.gpu

N_ROWS, ROW_BYTES, P, V, OFFSETS, ITERATIONS, SEED = 200_003, 128, 64, 4, [0, 1, 2, 3, 5, 63], 3, 7


def _deck() -> np.ndarray:
    return np.random.default_rng(5).integers(0, 256, size=(N_ROWS, ROW_BYTES), dtype=np.uint8)


def _split(world: int) -> list[int]:
    base = N_ROWS // world
    rows = [base + (17 * r if r < world - 1 else 0) for r in range(world)]
    rows[-1] = N_ROWS - sum(rows[:-1])
    return rows


def _worker(rank: int, world: int, port: int, out_dir: str, randomness: str, double_buffer: bool | None):
    sys.path[:0] = [str(REPO), str(REPO / "pov-shuffle_b200")]
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=120),
                            device_id=torch.device("cuda", rank))
    import povs

    rows = _split(world)
    start = sum(rows[:rank])
    shard = torch.from_numpy(_deck()[start:start + rows[rank]].copy()).to(f"cuda:{rank}")
    deck = povs.ShardedDeck(shard, double_buffer=double_buffer)
    opts = povs.Options(V, P, OFFSETS, 64, randomness)
    deck.shuffle(iterations=ITERATIONS, options=opts, seed=SEED if rank == 0 else 12345)
    deck.shuffle(iterations=2, options=opts, seed=SEED + 1)
    torch.cuda.synchronize()
    povs.check_device_status(rank)
    np.save(os.path.join(out_dir, f"rank{rank}.npy"), shard.cpu().numpy())
    deck.close()
    dist.destroy_process_group()


CASES = [("uniform", False), ("uniform", True), ("reference_cuda", False), ("reference_cuda", True),
         ("uniform", None), ("reference_numpy", True)]


@pytest.mark.parametrize("randomness,double_buffer", CASES)
def test_sharded_deck_matches_oracle(oracle_api, tmp_path, randomness, double_buffer):
    """Odd (3) then even (2) iteration counts: the double-buffered order ends in the shard both ways.
    double_buffer=None lets the ranks choose together (double-buffered when every GPU has room)."""
    world = min(torch.cuda.device_count(), 8)
    if world < 2:
        pytest.skip("needs at least two GPUs")
    port = 31000 + (os.getpid() % 2000) + 11 * CASES.index((randomness, double_buffer))
    mp.start_processes(_worker, args=(world, port, str(tmp_path), randomness, double_buffer), nprocs=world,
                       start_method="spawn", join=True)
    got = np.concatenate([np.load(tmp_path / f"rank{r}.npy") for r in range(world)])
    want = _deck()
    oracle_api.shuffle(want, ITERATIONS, P, V, OFFSETS, SEED, randomness)
    oracle_api.shuffle(want, 2, P, V, OFFSETS, SEED + 1, randomness)
    assert np.array_equal(got, want)


@pytest.mark.parametrize("double_buffer", [False, True])
def test_one_process_shards_on_two_gpus(oracle_api, double_buffer):
    """One process, shards on GPUs 0 and 1 (and their scratch buffers): the kernels on GPU 0 reach GPU 1's
    shard over NVLink; the result is the oracle's shuffle of the concatenated deck."""
    if torch.cuda.device_count() < 2:
        pytest.skip("needs at least two GPUs")
    sys.path[:0] = [str(REPO), str(REPO / "pov-shuffle_b200")]
    import povs

    rows = _split(2)
    host = _deck()
    shards = [torch.from_numpy(host[:rows[0]].copy()).to("cuda:0"),
              torch.from_numpy(host[rows[0]:].copy()).to("cuda:1")]
    scratch = [torch.empty_like(s) for s in shards] if double_buffer else None
    opts = povs.Options(V, P, OFFSETS, 64)
    povs.shuffle_shards(shards, iterations=ITERATIONS, options=opts, seed=SEED, scratch=scratch)
    torch.cuda.synchronize(0)
    povs.check_device_status(0)
    got = np.concatenate([s.cpu().numpy() for s in shards])
    want = host.copy()
    oracle_api.shuffle(want, ITERATIONS, P, V, OFFSETS, SEED)
    assert np.array_equal(got, want)
