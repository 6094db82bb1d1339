"""Timing helpers of the evaluation exercises (reference: src/povs/eval/utils.py:9-55)."""

from __future__ import annotations

import time
from collections.abc import Callable


def time_cuda_op(op: Callable, num_warmup: int, num_runs: int) -> list[float]:
    """Per-run device time in milliseconds of ``op`` (CUDA events on the current stream)."""
    import torch

    for _ in range(num_warmup):
        op()
    torch.cuda.synchronize()
    times = []
    for _ in range(num_runs):
        begin, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        begin.record()
        op()
        end.record()
        torch.cuda.synchronize()
        times.append(begin.elapsed_time(end))
    return times


def time_cpu_op(op: Callable, num_warmup: int, num_runs: int) -> list[float]:
    """Per-run wall time in milliseconds of a host operation."""
    for _ in range(num_warmup):
        op()
    times = []
    for _ in range(num_runs):
        t0 = time.perf_counter()
        op()
        times.append((time.perf_counter() - t0) * 1e3)
    return times
