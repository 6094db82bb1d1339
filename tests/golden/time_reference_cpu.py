"""Time the reference's own CPU path (``povs.shuffle`` on a NumPy array, src/povs/numpy.py:18-61)
on samples of the benchmark workloads, and record the figures in reference_cpu_timing.json.

The reference's Python package cannot be installed on the GPU hosts (its setup.py imports
``cutlass_library`` at line 9, which the image lacks), and its sources do not ship with this
repository, so the figure is taken where the reference checkout is, on that machine's host cores,
and ``bench.py`` reports it beside its own CPU baselines with the machine it came from.

Each sample keeps the workload's row size, dtype width, V, P, iterations and the reference
chooser's offsets (bf16 rows as uint16: NumPy has no bf16; the bytes moved are the same).  The
reference runs single-threaded (NumPy, ``np.vectorize`` over vblocks).

Usage: python tests/golden/time_reference_cpu.py <reference_root>
"""

from __future__ import annotations

import json
import os
import platform
import sys
import time
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
OUT = HERE / "reference_cpu_timing.json"

# name: (sample rows, row elements, numpy dtype, V, P, iterations, workload rows)
SAMPLES = {
    "bf16_32GiB": (1_048_576, 128, np.uint16, 4, 32, 4, 134_217_728),
    "fp16_256MiB": (1_048_576, 128, np.float16, 2, 64, 4, 1_048_576),
    "u8_12KiB": (20_000, 12_288, np.uint8, 2, 16, 3, 1_000_000),
    "f32_128GiB": (1_048_576, 32, np.float32, 4, 64, 4, 1_073_741_824),
}


def cpu_model() -> str:
    try:
        for line in Path("/proc/cpuinfo").read_text().splitlines():
            if line.startswith("model name"):
                return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return platform.processor() or "unknown"


def main(reference_root: str) -> None:
    sys.path.insert(0, str(Path(reference_root) / "src"))
    import povs as ref_povs  # the reference package
    from povs import Options
    from povs.common import choose_offsets

    result = {"what": "the reference's povs.shuffle(numpy array) (src/povs/numpy.py:18-61), single-threaded",
              "host_cpus": os.cpu_count(), "cpu_model": cpu_model(), "cores_used": 1, "samples": {}}
    for name, (rows, elems, dtype, V, P, iters, full_rows) in SAMPLES.items():
        rng = np.random.default_rng(0)
        deck = rng.integers(0, 255, size=(rows, elems)).astype(dtype)
        item = deck.dtype.itemsize
        opts = Options(virtual_block_size=V, physical_block_size=P, offsets=choose_offsets(rows, elems, item, P))
        t0 = time.perf_counter()
        ref_povs.shuffle(deck, iterations=iters, options=opts, seed=7)
        t = time.perf_counter() - t0
        nbytes = rows * elems * item
        result["samples"][name] = {
            "value": round(2 * nbytes * iters / t / 1e9, 4),
            "unit": "GB/s",
            "seconds": round(t, 3),
            "sample": f"{rows:,} of {full_rows:,} rows x {elems * item} B, {iters} iterations, V={V}, P={P}",
        }
        print(name, result["samples"][name], flush=True)
    OUT.write_text(json.dumps(result, indent=1) + "\n")


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit(__doc__.strip().splitlines()[-1])
    main(sys.argv[1])
