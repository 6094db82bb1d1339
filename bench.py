"""Benchmark of the POV-shuffle hot path on B200.

Metric: effective shuffle GB/s = 2 x deck bytes x iterations / time (each iteration reads and
writes every byte once), with the fraction of the measured HBM copy bandwidth.

One step = one ``povs.shuffle`` call of ITERATIONS iterations over the whole deck, which stays
resident in HBM (``value``).  ``e2e`` runs the same call through the C ABI with the deck in
pinned host memory (``povs_shuffle_host_v1``): host->device copy, the iterations, device->host
copy and a stream sync, every step.

Workloads (synthetic data with the shapes and value distributions of the named configs):
  bf16_32GiB   134,217,728 x 128 bf16 (32 GiB), uniform [-1, 1) from seed 1, 4 iterations, V=4, P=32  [default]
  fp16_256MiB  1,048,576 x 128 fp16 (256 MiB), standard normal from seed 0, 4 iterations, V=2, P=64
  u8_12KiB     1,000,000 x 3x64x64 uint8 (12.3 GB), uniform 0..255 from seed 2, 3 iterations, V=2, P=16
  f32_128GiB   1,073,741,824 x 32 fp32 (128 GiB), standard normal from seed 3, 4 iterations, V=4, P=64
  i32x16_2GiB  33,554,432 x 16 int32 (2 GiB), the bias suite's 64-byte rows, V=2, P=8, 4 iterations
With --gpus N > 1 (torchrun, one process per GPU) the workload's deck is split along axis 0 into N
shards, one per GPU, and shuffled as one deck (povs.ShardedDeck: member rows move over NVLink):
the total work is fixed, so the scaling is strong.

``--impl reference`` times the CPU implementation of the same path (the oracle's C restatement,
all host threads) on a bounded sample of the workload and prints the same JSON line.  Its line also
carries ``reference_cuda_path``: the reference's own CUDA path (src/povs/__cuda/lib/povs.cu, its
host loop and kernel, compiled into oracle/_ref) timed on this GPU on the full workload deck, when
the reference instantiates that shape.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time
from datetime import timedelta
from pathlib import Path

REPO = Path(__file__).resolve().parent
for _p in (REPO, REPO / "pov-shuffle_b200"):
    if str(_p) not in sys.path:
        sys.path.insert(0, str(_p))

METRIC = "effective shuffle GB/s (2×bytes×iters/time), % HBM peak, 1/2/4/8×B200"
FALLBACK_HBM_GBS = 6650.0
# NVLink 5 per direction per GPU (18 links through NVSwitch): the denominator of the sharded mode's
# roofline.  The bandwidth a peer copy reaches in the same run is measured and reported beside it.
NVLINK_NOMINAL_GBS = 900.0
DTYPE_NAMES = {"bfloat16": "bf16", "float16": "fp16", "float32": "fp32", "uint8": "u8", "int32": "i32"}

WORKLOADS = {
    "bf16_32GiB": dict(
        rows=134_217_728, shape=(128,), dtype="bfloat16", iterations=4, V=4, P=32, seed=1, init="uniform",
        desc="bf16 deck 134,217,728 x 128 (32 GiB), uniform [-1,1) from seed 1, iterations=4, V=4, P=32",
    ),
    "fp16_256MiB": dict(
        rows=1_048_576, shape=(128,), dtype="float16", iterations=4, V=2, P=64, seed=0, init="normal",
        desc="fp16 deck 1,048,576 x 128 (256 MiB), standard normal from seed 0, iterations=4, V=2, P=64",
    ),
    "f32_128GiB": dict(
        rows=1_073_741_824, shape=(32,), dtype="float32", iterations=4, V=4, P=64, seed=3, init="normal",
        desc="fp32 deck 1,073,741,824 x 32 (128 GiB), standard normal from seed 3, iterations=4, V=4, P=64",
    ),
    "i32x16_2GiB": dict(
        rows=33_554_432, shape=(16,), dtype="int32", iterations=4, V=2, P=8, seed=4, init="bytes",
        desc="int32 deck 33,554,432 x 16 (64-byte rows and V=2, P=8 of the bias suite, 2 GiB), uniform bytes "
        "from seed 4, iterations=4",
    ),
    "f32x4_2GiB": dict(
        rows=134_217_728, shape=(4,), dtype="float32", iterations=4, V=2, P=64, seed=5, init="bytes",
        desc="fp32 deck 134,217,728 x 4 (16-byte rows with the reference chooser's V=2, P=64, 2 GiB), uniform "
        "bytes from seed 5, iterations=4",
    ),
    "f32x6_2GiB": dict(
        rows=89_478_485, shape=(6,), dtype="float32", iterations=4, V=2, P=64, seed=6, init="bytes",
        desc="fp32 deck 89,478,485 x 6 (24-byte rows, not a multiple of 16 bytes: plain loads and chunked "
        "stores, with the reference chooser's V=2, P=64, 2 GiB), uniform bytes from seed 6, iterations=4",
    ),
    "u8_12KiB": dict(
        rows=1_000_000, shape=(3, 64, 64), dtype="uint8", iterations=3, V=2, P=16, seed=2, init="bytes",
        desc="uint8 deck 1,000,000 x 3x64x64 (12,288 B rows, 12.3 GB), uniform 0..255 from seed 2, iterations=3, V=2, P=16",
    ),
}


ELEM_BYTES = {"bfloat16": 2, "float16": 2, "uint8": 1, "float32": 4, "int32": 4}


def measured_peaks() -> tuple[float, str]:
    path = REPO / "MEASURED_PEAKS.json"
    try:
        data = json.loads(path.read_text())
        return float(data["hbm_gbs"]), "measured"
    except Exception:
        return FALLBACK_HBM_GBS, "fallback"


def row_bytes_of(w: dict) -> int:
    import numpy as np

    elem = ELEM_BYTES[w["dtype"]]
    return int(np.prod(w["shape"])) * elem


def traffic_per_launch(kernel: str, workload: str) -> int | None:
    """DRAM bytes per launch of ``kernel`` from the committed ncu summary, if one exists."""
    path = REPO / "profiles" / f"{kernel}__{workload}.md"
    if not path.exists():
        return None
    for line in path.read_text().splitlines():
        if line.strip().startswith("traffic_bytes_per_launch:"):
            return int(line.split(":", 1)[1].strip().replace(",", ""))
    return None


class ClockSampler:
    """nvidia-smi clock / throttle sampling during the timed region."""

    FIELDS = (
        "index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
        "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
        "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap"
    )

    def __init__(self, gpu_index: int):
        self.gpu_index = gpu_index
        self.proc = None
        self.file = None

    def start(self):
        try:
            self.file = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits", "-lms", "200",
                 "-i", str(self.gpu_index)],
                stdout=self.file, stderr=subprocess.DEVNULL,
            )
        except Exception:
            self.proc = None

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        self.file.flush()
        self.file.seek(0)
        sms, maxes, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in self.file.read().splitlines():
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                sms.append(float(parts[1]))
                maxes.append(float(parts[2]))
            except ValueError:
                continue
            for name, val in zip(names, parts[5:9]):
                if val.lower().startswith("active"):
                    reasons.add(name)
        os.unlink(self.file.name)
        return {
            "sm_mhz": statistics.median(sms) if sms else None,
            "sm_max_mhz": max(maxes) if maxes else None,
            "reasons": sorted(reasons),
            "samples": len(sms),
        }


def make_deck(w: dict, device, rows: int | None = None, seed_offset: int = 0):
    import torch

    dtype = getattr(torch, w["dtype"])
    shape = (w["rows"] if rows is None else rows, *w["shape"])
    g = torch.Generator(device=device).manual_seed(w["seed"] + seed_offset)
    if w["init"] == "uniform":
        return torch.rand(shape, generator=g, device=device, dtype=dtype) * 2 - 1
    if w["init"] == "normal":
        return torch.randn(shape, generator=g, device=device, dtype=dtype)
    raw = torch.randint(0, 256, (shape[0], row_bytes_of(w)), generator=g, device=device, dtype=torch.uint8)
    return raw.view(dtype).reshape(shape)


def run_ours(args, w: dict, wname: str) -> None:
    import torch
    import torch.distributed as dist

    import povs
    from povs import _native
    from povs.common import choose_offsets

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        # The group only broadcasts seeds; NVLink multicast (NVLS) is not needed for that.
        os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", device_id=torch.device("cuda", local), timeout=timedelta(seconds=300))
    device = torch.device("cuda", local)
    torch.cuda.set_device(device)

    R = row_bytes_of(w)
    N, P, V, iters = w["rows"], w["P"], w["V"], w["iterations"]
    elem = ELEM_BYTES[w["dtype"]]
    offsets = choose_offsets(N, R // elem, elem, P)
    opts = povs.Options(virtual_block_size=V, physical_block_size=P, offsets=offsets,
                        gpu_thread_block_size=max(32, min(64, V * P)))
    stream = torch.cuda.current_stream(device)
    if world > 1:
        # One deck of N rows split into `world` shards; every rank times the same collective steps.
        rows = [N // world] * world
        rows[-1] += N - sum(rows)
        deck = make_deck(w, device, rows=rows[rank], seed_offset=rank)
        push = args.sharded_order == "push"
        sharded = povs.ShardedDeck(deck, double_buffer=push)
        plan = {"shard_rows": rows, "order": "double-buffered push" if push else "in place"}

        def step(seed: int) -> None:
            sharded.shuffle(iterations=iters, options=opts, seed=seed)
    else:
        deck = make_deck(w, device)
        plan = _native.describe_plan(deck, R, P, V)

        def step(seed: int) -> None:
            povs.shuffle(deck, iterations=iters, options=opts, seed=seed)

    def barrier():
        if world > 1:
            dist.barrier(device_ids=[local])

    sampler = ClockSampler(local)
    sampler.start()
    time.sleep(0.5)  # let nvidia-smi start sampling before the timed region
    # Warm-up right before the timed region, so that its first step does not start on a GPU that
    # idled through the pause above (on the 256 MiB deck that cost 4 % over 20 steps).
    for s in range(args.warmup):
        step(1000 + s)
    torch.cuda.synchronize(device)
    povs.check_device_status(device)
    barrier()
    torch.cuda.synchronize(device)
    start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record(stream)
    for s in range(args.steps):
        step(s)
    stop.record(stream)
    torch.cuda.synchronize(device)
    barrier()
    clocks = sampler.stop()
    ms = start.elapsed_time(stop)
    povs.check_device_status(device)
    if world > 1:
        t = torch.tensor([ms], device=device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())

    deck_bytes = N * R  # the whole deck (all shards)
    alg_bytes_per_step = 2 * deck_bytes * iters
    ms_per_step = ms / args.steps
    value = alg_bytes_per_step / (ms_per_step / 1e3) / 1e9
    per_launch_s = (ms / 1e3) / (args.steps * iters)
    peak, peak_kind = measured_peaks()
    peer_copy = None
    if world == 1:
        bound, achieved, roof_peak, roof_kind = "hbm", 2 * deck_bytes / per_launch_s / 1e9, peak, peak_kind
    else:
        # Per GPU and iteration, bytes crossing NVLink in each direction.  Push order: (world-1)/world
        # of the rows of its shard go to peers and as many arrive from them, once each.  In place:
        # every remote member row is read and written back, twice that.
        crossings = 1 if args.sharded_order == "push" else 2
        link_bytes = crossings * (world - 1) / world * (deck_bytes / world)
        bound, achieved, roof_peak, roof_kind = "nvlink", link_bytes / per_launch_s / 1e9, NVLINK_NOMINAL_GBS, (
            "nominal NVLink 5 bandwidth per direction per GPU")
        peer_copy = measure_peer_copy(device, rank, world, local, dist)

    # End to end: the same work with the deck in pinned host memory, copies inside the timed region.
    e2e = None
    if not args.no_e2e:
        e2e = run_e2e(args, w, deck, opts, offsets, iters, world, rank, local, stream,
                      sharded if world > 1 else None, dist)

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cpu = cpu_baseline(w, threads=1, target_s=args.cpu_seconds)
        cpu["reference_povs_shuffle"] = reference_cpu_path(wname)

    if rank == 0:
        line = {
            "metric": METRIC,
            "value": round(value, 3),
            "unit": "GB/s",
            "n_gpus": world,
            "steps": args.steps,
            "warmup": args.warmup,
            "ms_per_step": round(ms_per_step, 4),
            "higher_is_better": True,
            "scaling": "strong",
            "vs_baseline": None,
            "dtype": DTYPE_NAMES[w["dtype"]],
            "data": "synthetic",
            "config": {
                "workload": w["desc"],
                "name": wname,
                "rows": N,
                "row_bytes": R,
                "deck_dtype": w["dtype"],
                "iterations": iters,
                "virtual_block_size": V,
                "physical_block_size": P,
                "offsets": offsets,
                "instances_per_s": round(N * iters / (ms_per_step / 1e3)),
                "l2": "inputs larger than L2 (deck > 126 MB)" if deck_bytes > 126e6 else "deck fits L2",
                "parallelism": f"sharded x{world} (NVLink P2P, one process per GPU)" if world > 1 else "single GPU",
                "plan": plan,
            },
            "roofline": {
                "bound": bound,
                "kernel": "povs_iteration_kernel",
                "achieved": round(achieved, 1),
                "peak": roof_peak,
                "peak_kind": roof_kind,
                "unit": "GB/s",
                "frac": round(achieved / roof_peak, 4),
                "traffic": traffic_per_launch("povs_iteration_kernel", wname) if world == 1 and not (args.rows or args.vblock or args.pblock) else None,
                "alg_bytes_per_launch": 2 * deck_bytes // world,
                "hbm_frac_per_gpu": round(2 * deck_bytes / world / per_launch_s / 1e9 / peak, 4),
                **({"peer_copy_gbs_measured": peer_copy,
                    "frac_of_measured_peer_copy": round(achieved / peer_copy, 4) if peer_copy else None}
                   if world > 1 else {}),
            },
            "gpu_launches": args.steps * iters if world == 1 else args.steps * (2 * iters + 1),
            "clocks": clocks,
            "e2e": e2e,
            "cpu_baseline": cpu,
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        sharded.close()
        dist.destroy_process_group()


def measure_peer_copy(device, rank: int, world: int, local: int, dist, nbytes: int = 1 << 30, reps: int = 5) -> float:
    """GB/s per direction per GPU of a ring exchange (every rank sends 1 GiB to the next rank and
    receives 1 GiB from the previous one at the same time), after the timed region; max time over ranks."""
    import torch

    send = torch.empty(nbytes, dtype=torch.uint8, device=device)
    recv = torch.empty_like(send)
    nxt, prv = (rank + 1) % world, (rank - 1) % world

    def exchange() -> None:
        reqs = dist.batch_isend_irecv([dist.P2POp(dist.isend, send, nxt), dist.P2POp(dist.irecv, recv, prv)])
        for r in reqs:
            r.wait()

    exchange()
    torch.cuda.synchronize(device)
    dist.barrier(device_ids=[local])
    stream = torch.cuda.current_stream(device)
    start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record(stream)
    for _ in range(reps):
        exchange()
    stop.record(stream)
    torch.cuda.synchronize(device)
    t = torch.tensor([start.elapsed_time(stop)], device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    del send, recv
    torch.cuda.empty_cache()
    return round(nbytes * reps / (float(t.item()) / 1e3) / 1e9, 1)


def run_e2e(args, w, deck, opts, offsets, iters, world, rank, local, stream, sharded, dist) -> dict | None:
    """Same metric with the deck (or this rank's shard) in pinned host memory, copies timed."""
    import ctypes

    import psutil
    import torch

    import povs
    from povs import _native

    shard_bytes = deck.numel() * deck.element_size()
    total_bytes = w["rows"] * row_bytes_of(w)
    # One GPU: three host decks in rotation through three device buffers keep both PCIe directions
    # busy (a deck's copy in never waits for its own previous copy out); two when host memory is short.
    # Several ranks: two sharded decks per rank (the resident one and a second of the same split),
    # so that one deck's copies in overlap the other's shuffle and copy out.
    avail = psutil.virtual_memory().available
    n_host = 3 if world == 1 and avail >= 3.5 * total_bytes else 2
    free_dev, _ = torch.cuda.mem_get_info(deck.device)
    # The extra device buffers must fit next to the resident deck (and its scratch buffer).
    per_buffer = shard_bytes * (2 if world > 1 and sharded.double_buffer else 1)
    while n_host > 1 and (n_host - 1) * per_buffer + (2 << 30) > free_dev:
        n_host -= 1
    # Decide together, before anything is pinned, so that every rank takes the same steps.
    ok = torch.tensor([1 if avail >= (n_host + 0.5) * total_bytes else 0, n_host], device=deck.device)
    if world > 1:
        dist.all_reduce(ok, op=dist.ReduceOp.MIN)
    if not int(ok[0].item()):
        return {"value": None, "unit": "GB/s", "skipped": "not enough host memory for pinned copies of the deck"}
    n_host = int(ok[1].item())
    flat = deck.view(torch.uint8).reshape(-1)
    hosts = []
    for _ in range(n_host):
        h = torch.empty(shard_bytes, dtype=torch.uint8, pin_memory=True)
        h.copy_(flat)
        hosts.append(h)
    R = row_bytes_of(w)
    P, V = w["P"], w["V"]
    e2e_steps = max(2, args.e2e_steps)
    if world == 1:
        # povs.shuffle_many's native call: deck k of the timed steps is host deck k % 2, staged through
        # the resident deck buffer and a second device buffer; copies in and out overlap the work.
        buffers = [flat] + [torch.empty_like(flat) for _ in range(n_host - 1)]

        def run_steps(n: int, seed: int) -> None:
            _native.shuffle_host_batch([hosts[k % n_host].data_ptr() for k in range(n)], buffers, deck.shape[0], R,
                                       offsets, iters, P, V, [seed + k for k in range(n)])
        path = (f"povs_shuffle_host_batch_v1 (povs.shuffle_many): {n_host} pinned host decks in rotation, "
                f"{n_host} device buffers")
    else:
        decks = [sharded] + [povs.ShardedDeck(torch.empty_like(deck), double_buffer=sharded.double_buffer)
                             for _ in range(n_host - 1)]
        host_shards = [h.view(deck.dtype).view(deck.shape) for h in hosts]

        def run_steps(n: int, seed: int) -> None:
            povs.shuffle_host_shards(decks, [host_shards[k % n_host] for k in range(n)], iterations=iters,
                                     options=opts, seed=seed)
        path = (f"povs.shuffle_host_shards per rank: {n_host} pinned host shards in rotation through {n_host} "
                f"sharded decks, copies on their own streams")

    run_steps(2, 7)
    if world > 1:
        dist.barrier(device_ids=[local])
    e_start, e_stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e_start.record(stream)
    run_steps(e2e_steps, 100)
    e_stop.record(stream)
    torch.cuda.synchronize()
    e_ms = e_start.elapsed_time(e_stop)
    if world > 1:
        t = torch.tensor([e_ms], device=deck.device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e_ms = float(t.item())
    povs.check_device_status(deck.device)
    if world > 1:
        for d in decks[1:]:
            d.close()
    return {
        "value": round(2 * total_bytes * iters / (e_ms / e2e_steps / 1e3) / 1e9, 3),
        "unit": "GB/s",
        "h2d_bytes_per_step": total_bytes,
        "d2h_bytes_per_step": total_bytes,
        "steps": e2e_steps,
        "ms_per_step": round(e_ms / e2e_steps, 3),
        "path": path,
    }


def cpu_baseline(w: dict, threads: int, target_s: float) -> dict:
    """Times the oracle's C restatement of the path on a bounded sample of the workload."""
    import numpy as np

    from oracle import api as oracle
    from povs.common import choose_offsets

    R = row_bytes_of(w)
    elem = ELEM_BYTES[w["dtype"]]
    P, V, iters = w["P"], w["V"], w["iterations"]

    def run(rows: int) -> float:
        deck = np.random.default_rng(w["seed"]).integers(0, 256, size=(rows, R), dtype=np.uint8)
        offs = choose_offsets(rows, R // elem, elem, P)
        t0 = time.perf_counter()
        if threads == 1:
            oracle.shuffle(deck, iters, P, V, offs, 11)
        else:
            oracle.shuffle_threads(deck, iters, P, V, offs, 11, threads)
        return time.perf_counter() - t0

    probe_rows = min(w["rows"], max(4096, (64 << 20) // R))
    t_probe = run(probe_rows)
    rows = int(min(w["rows"], max(probe_rows, probe_rows * target_s / max(t_probe, 1e-3))))
    rows = min(rows, max(probe_rows, (8 << 30) // R))  # at most 8 GiB of host memory
    t = run(rows) if rows != probe_rows else t_probe
    gbs = 2 * rows * R * iters / t / 1e9
    out = {
        "value": round(gbs, 3),
        "unit": "GB/s",
        "cores": threads,
        "host_cpus": os.cpu_count(),
        "kind": "port",
        "sample": f"{rows:,} of {w['rows']:,} rows x {R} B, {iters} iterations, {t:.2f} s",
    }
    if threads == 1:
        # The reference's uniform baseline: numpy.random.Generator.shuffle of the rows (one full
        # shuffle moves every byte once: 2 x bytes / time, the same unit as one POV iteration).
        base = np.random.default_rng(w["seed"]).integers(0, 256, size=(rows, R), dtype=np.uint8)
        t0 = time.perf_counter()
        np.random.default_rng(w["seed"]).shuffle(base)
        tn = time.perf_counter() - t0
        out["numpy_shuffle"] = {"value": round(2 * rows * R / tn / 1e9, 3), "unit": "GB/s", "cores": 1,
                                "sample": f"numpy Generator.shuffle of {rows:,} rows x {R} B, {tn:.2f} s"}
    return out


REFERENCE_CPU_UNAVAILABLE = (
    "the reference's Python package is not on this host: its setup.py imports cutlass_library at "
    "line 9, which this image lacks, so it cannot be installed, and its sources do not ship with "
    "this repository"
)


def reference_cpu_path(wname: str) -> dict:
    """The reference's own povs.shuffle on a NumPy deck: unavailable here; the figure recorded where
    the reference checkout is (tests/golden/reference_cpu_timing.json) is reported with its machine."""
    out = {"value": None, "unit": "GB/s", "unavailable": REFERENCE_CPU_UNAVAILABLE}
    fixture = REPO / "tests" / "golden" / "reference_cpu_timing.json"
    if fixture.exists():
        rec = json.loads(fixture.read_text())
        sample = rec.get("samples", {}).get(wname)
        if sample:
            out["recorded_elsewhere"] = dict(sample, cores=rec.get("cores_used"), host_cpus=rec.get("host_cpus"),
                                             cpu_model=rec.get("cpu_model"),
                                             where="the build machine (no GPU), not this host")
    return out


def reference_cuda_path(w: dict, wname: str, steps: int) -> dict:
    """The reference's own CUDA path on this GPU over the full workload deck (oracle/_ref):
    ``path`` = whole povs_cuda calls (its host randomness, blocking copies and kernels; wall clock);
    ``kernel`` = its kernel alone with device-resident assignments and seeds (CUDA events)."""
    import torch

    from oracle import api as oracle
    from povs.common import choose_offsets

    if not torch.cuda.is_available():
        return {"value": None, "unavailable": "no GPU"}
    if oracle.ref_cuda_lib() is None:
        return {"value": None, "unavailable": "oracle/_ref/libref_povs_cuda.so is not built"}
    R = row_bytes_of(w)
    elem = ELEM_BYTES[w["dtype"]]
    N, P, V, iters = w["rows"], w["P"], w["V"], w["iterations"]
    shape = oracle.ref_cuda_shape(V, P, R)
    if shape is None:
        if V * P < 32:
            why = (f"the reference kernel needs a thread block of 32 to V*P = {V * P} threads "
                   "(src/povs/__cuda/lib/povs.cu:139-142): this shape has no valid instantiation")
        elif V * P * R + 4 * V * P > 48 * 1024:
            why = (f"the reference kernel stages a whole vblock ({V * P * R:,} B) in static shared memory (48 KB "
                   "limit, src/povs/__cuda/lib/povs.cu:167): no instantiation exists for this shape")
        else:
            why = "the reference-built library has no instantiation of this shape"
        return {"value": None, "unavailable": why}
    info = next(sh for sh in oracle.ref_cuda_shapes() if sh["index"] == shape)
    device = torch.device("cuda", 0)
    torch.cuda.set_device(device)
    deck = make_deck(w, device)
    ptr = deck.data_ptr()
    offsets = choose_offsets(N, R // elem, elem, P)
    alg = 2 * N * R * iters
    oracle.ref_povs_cuda(shape, ptr, N, offsets, iters, 1)  # warm-up (module load, first allocations)
    t0 = time.perf_counter()
    for k in range(steps):
        oracle.ref_povs_cuda(shape, ptr, N, offsets, iters, 2 + k)
    t_path = (time.perf_counter() - t0) / steps
    # Kernel alone: one launch per iteration, device-resident randomness of the reference's form.
    n_p = -(-N // P)
    n_v = -(-n_p // V)
    g = torch.Generator(device=device).manual_seed(5)
    slots = torch.randperm(n_v * V, generator=g, device=device)
    assign = torch.where(slots < n_p, slots, torch.full_like(slots, -1)).to(torch.int64)
    seeds = torch.randint(1, 1000, (n_v,), generator=g, device=device, dtype=torch.int32)
    legacy = torch.cuda.default_stream(device)
    for it in range(iters):
        oracle.ref_povs_kernel(shape, ptr, N, assign.data_ptr(), seeds.data_ptr(), offsets[it % len(offsets)])
    torch.cuda.synchronize(device)
    start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record(legacy)
    for k in range(steps):
        for it in range(iters):
            oracle.ref_povs_kernel(shape, ptr, N, assign.data_ptr(), seeds.data_ptr(), offsets[it % len(offsets)])
    stop.record(legacy)
    torch.cuda.synchronize(device)
    t_kernel = start.elapsed_time(stop) / 1e3 / steps
    peak, peak_kind = measured_peaks()
    del deck, assign, seeds, slots
    torch.cuda.empty_cache()
    return {
        "value": round(alg / t_path / 1e9, 3),
        "unit": "GB/s",
        "what": "the reference's povs_cuda (src/povs/__cuda/lib/povs.cu:356-467) on the full deck, per call of "
        f"{iters} iterations, wall clock",
        "kernel": {"value": round(alg / t_kernel / 1e9, 1), "unit": "GB/s",
                   "frac_of_hbm": round(alg / t_kernel / 1e9 / peak, 4), "peak": peak, "peak_kind": peak_kind,
                   "ms_per_launch": round(t_kernel * 1e3 / iters, 3)},
        "ms_per_call": round(t_path * 1e3, 2),
        "instantiation": {k: info[k] for k in ("V", "P", "inst", "elem_bytes", "block")},
        "steps": steps,
        "deck": w["desc"],
    }


def run_reference(args, w: dict, wname: str) -> None:
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    threads = os.cpu_count() or 1
    vals = []
    cb = None
    for s in range(args.warmup + args.steps):
        cb = cpu_baseline(w, threads=threads, target_s=min(5.0, args.cpu_seconds))
        if s >= args.warmup:
            vals.append(cb["value"])
    value = statistics.median(vals) if vals else cb["value"]
    cb = dict(cb, value=round(value, 3))
    cb["reference_povs_shuffle"] = reference_cpu_path(wname)
    try:
        ref_gpu = reference_cuda_path(w, wname, steps=3)
    except Exception as exc:  # reported, not fatal: the CPU arm above is the line's value
        ref_gpu = {"value": None, "unavailable": f"{type(exc).__name__}: {exc}"}
    line = {
        "metric": METRIC,
        "impl": "reference",
        "value": round(value, 3),
        "unit": "GB/s",
        "n_gpus": int(os.environ.get("WORLD_SIZE", "1")),
        "steps": args.steps,
        "warmup": args.warmup,
        "higher_is_better": True,
        "scaling": "strong",
        "vs_baseline": None,
        "dtype": DTYPE_NAMES[w["dtype"]],
        "data": "synthetic",
        "config": {"workload": w["desc"], "name": wname},
        "cpu_baseline": cb,
        "e2e": {"value": round(value, 3), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "reference_cuda_path": ref_gpu,
        "note": "value: the CPU implementation of the path on this host's cores, the oracle's C restatement of the "
        "POV iteration on all threads (the reference's own CPU path is Python/NumPy and cannot be installed here: "
        "see cpu_baseline.reference_povs_shuffle); reference_cuda_path: the reference's own CUDA path compiled "
        "from its sources, timed on this GPU",
    }
    print(json.dumps(line), flush=True)


def run_one_process_shards(args, w: dict, wname: str) -> None:
    """Profiling mode (not the benchmark line): the workload deck split into K equal shards on GPUs
    0..K-1 of this one process and shuffled by povs.shuffle_shards in the double-buffered push order.
    One kernel per iteration on GPU 0 moves every pblock: it reads the rows of the K-1 remote shards
    over NVLink (bulk copies, no multicast) and stores the rows whose destination slot is remote
    over NVLink, so per iteration (K-1)/K of the deck enters GPU 0 over NVLink and as much leaves it."""
    import torch

    import povs
    from povs.common import choose_offsets

    K = args.shards_on_gpus
    assert torch.cuda.device_count() >= K, f"needs {K} GPUs"
    R = row_bytes_of(w)
    N, P, V, iters = w["rows"], w["P"], w["V"], w["iterations"]
    elem = ELEM_BYTES[w["dtype"]]
    offsets = choose_offsets(N, R // elem, elem, P)
    opts = povs.Options(virtual_block_size=V, physical_block_size=P, offsets=offsets,
                        gpu_thread_block_size=max(32, min(64, V * P)))
    rows = [N // K] * K
    rows[-1] += N - sum(rows)
    shards = [make_deck(w, torch.device("cuda", i), rows=rows[i], seed_offset=i) for i in range(K)]
    scratch = [torch.empty_like(s) for s in shards]
    dev0 = torch.device("cuda", 0)
    for s in range(args.warmup):
        povs.shuffle_shards(shards, iterations=iters, options=opts, seed=1000 + s, scratch=scratch)
    for i in range(K):
        torch.cuda.synchronize(i)
    stream = torch.cuda.current_stream(dev0)
    start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record(stream)
    for s in range(args.steps):
        povs.shuffle_shards(shards, iterations=iters, options=opts, seed=s, scratch=scratch)
    stop.record(stream)
    torch.cuda.synchronize(dev0)
    povs.check_device_status(0)
    ms = start.elapsed_time(stop)
    deck_bytes = N * R
    per_launch_s = ms / 1e3 / (args.steps * iters)
    link = (K - 1) / K * deck_bytes
    print(json.dumps({
        "mode": f"one process, deck split over GPUs 0..{K - 1}, double-buffered push order, kernels on GPU 0",
        "workload": w["desc"], "shard_rows": rows,
        "value": round(2 * deck_bytes / per_launch_s / 1e9, 1), "unit": "GB/s",
        "ms_per_launch": round(per_launch_s * 1e3, 3),
        "nvlink_rx_bytes_per_launch": int(link), "nvlink_tx_bytes_per_launch": int(link),
        "nvlink_gbs_per_direction": round(link / per_launch_s / 1e9, 1),
        "frac_of_nominal_nvlink": round(link / per_launch_s / 1e9 / NVLINK_NOMINAL_GBS, 4),
    }), flush=True)


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--workload", default="bf16_32GiB", choices=sorted(WORKLOADS))
    ap.add_argument("--e2e-steps", type=int, default=16)
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--cpu-seconds", type=float, default=10.0)
    ap.add_argument("--sharded-order", default="push", choices=["push", "inplace"],
                    help="with --gpus N > 1: double-buffered push order (default) or in place")
    ap.add_argument("--rows", type=int, default=None, help="override the workload's row count (profiling captures)")
    ap.add_argument("--vblock", type=int, default=None, help="override the workload's V (profiling captures)")
    ap.add_argument("--pblock", type=int, default=None, help="override the workload's P (profiling captures)")
    ap.add_argument("--pack-bytes", type=int, default=None,
                    help="largest packed unit in bytes (0 = one vblock per unit; profiling captures)")
    ap.add_argument("--shards-on-gpus", type=int, default=None,
                    help="profiling mode: split the deck over this many GPUs of one process (povs.shuffle_shards)")
    args = ap.parse_args()
    if args.warmup < 3:
        print("warning: fewer than 3 warm-up steps", file=sys.stderr)
    w = dict(WORKLOADS[args.workload])
    if args.rows:
        w["desc"] = w["desc"] + f" [rows overridden: {args.rows:,}]"
        w["rows"] = args.rows
    for key, val in (("V", args.vblock), ("P", args.pblock)):
        if val:
            w["desc"] = w["desc"] + f" [{key} overridden: {val}]"
            w[key] = val
    if args.pack_bytes is not None:
        from povs import _native

        _native.set_pack_bytes(args.pack_bytes)
        w["desc"] = w["desc"] + f" [pack_bytes {args.pack_bytes}]"
    if args.impl == "reference":
        run_reference(args, w, args.workload)
    elif args.shards_on_gpus:
        run_one_process_shards(args, w, args.workload)
    else:
        run_ours(args, w, args.workload)


if __name__ == "__main__":
    main()
