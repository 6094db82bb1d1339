"""Sharded mode across GPUs (one process per GPU, NCCL for the seed broadcast only).

Each rank holds a shard of one deck, and the concatenation of the shuffled shards must equal the
oracle's shuffle of the whole deck.  Most cases need at least two GPUs; the one-rank cases (the
whole deck as one shard) run on any machine with a GPU.
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


@pytest.mark.parametrize("randomness,double_buffer", [("uniform", True), ("reference_numpy", False)])
def test_one_rank_sharded_deck_matches_oracle(oracle_api, tmp_path, randomness, double_buffer):
    """A ShardedDeck of one rank (the whole deck is its shard): the sharded entry's barrier kernels
    and, double-buffered, the push order against its own scratch buffer, on any machine with a GPU."""
    port = 32800 + (os.getpid() % 2000) + (7 if double_buffer else 0)
    mp.start_processes(_worker, args=(1, port, str(tmp_path), randomness, double_buffer), nprocs=1,
                       start_method="spawn", join=True)
    want = _deck()
    oracle_api.shuffle(want, ITERATIONS, P, V, OFFSETS, SEED, randomness)
    oracle_api.shuffle(want, 2, P, V, OFFSETS, SEED + 1, randomness)
    assert np.array_equal(np.load(tmp_path / "rank0.npy"), want)


def _host_worker(rank: int, world: int, port: int, out_dir: str, randomness: str, double_buffer: bool):
    sys.path[:0] = [str(REPO), str(REPO / "pov-shuffle_b200")]
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=120),
                            device_id=torch.device("cuda", rank))
    import povs

    rows = _split(world)
    start = sum(rows[:rank])
    decks = [povs.ShardedDeck(torch.empty((rows[rank], ROW_BYTES), dtype=torch.uint8, device=f"cuda:{rank}"),
                              double_buffer=double_buffer) for _ in range(2)]
    hosts = [torch.from_numpy(_host_deck(d)[start:start + rows[rank]].copy()).pin_memory() for d in range(3)]
    opts = povs.Options(V, P, OFFSETS, 64, randomness)
    # Host shard 0 goes through twice (steps 0 and 3), the others once; three steps share two decks.
    povs.shuffle_host_shards(decks, [hosts[0], hosts[1], hosts[2], hosts[0]], iterations=ITERATIONS,
                             options=opts, seed=SEED if rank == 0 else 999)
    povs.check_device_status(rank)
    for d in range(3):
        np.save(os.path.join(out_dir, f"host{d}_rank{rank}.npy"), hosts[d].numpy())
    for deck in decks:
        deck.close()
    dist.destroy_process_group()


def _host_deck(d: int) -> np.ndarray:
    return np.random.default_rng(100 + d).integers(0, 256, size=(N_ROWS, ROW_BYTES), dtype=np.uint8)


@pytest.mark.parametrize("one_rank", [False, True])
@pytest.mark.parametrize("randomness,double_buffer", [("uniform", True), ("reference_cuda", False)])
def test_host_shards_streamed_through_two_sharded_decks(oracle_api, tmp_path, randomness, double_buffer, one_rank):
    """povs.shuffle_host_shards: step k shuffles its host shard with seed SEED + k; a host shard listed
    twice is shuffled twice in order; every host deck ends as the oracle's shuffle of it.  With one
    rank (any machine with a GPU) the whole deck is one shard and the streams and events still
    order every copy against the shuffles."""
    world = 1 if one_rank else min(torch.cuda.device_count(), 8)
    if world < 1 or (not one_rank and world < 2):
        pytest.skip("needs at least two GPUs")
    port = 33500 + (os.getpid() % 2000) + (11 if double_buffer else 0) + (5 if one_rank else 0)
    mp.start_processes(_host_worker, args=(world, port, str(tmp_path), randomness, double_buffer), nprocs=world,
                       start_method="spawn", join=True)
    steps = {0: [0, 3], 1: [1], 2: [2]}
    for d, ks in steps.items():
        got = np.concatenate([np.load(tmp_path / f"host{d}_rank{r}.npy") for r in range(world)])
        want = _host_deck(d)
        for k in ks:
            oracle_api.shuffle(want, ITERATIONS, P, V, OFFSETS, SEED + k, randomness)
        assert np.array_equal(got, want), f"host deck {d}"


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
