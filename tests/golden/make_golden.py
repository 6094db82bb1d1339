"""Generate the golden fixtures of the reference's NumPy path.

Runs the reference's own ``povs.shuffle`` on NumPy decks (importing ``povs`` from the reference
checkout, src/povs/numpy.py) and stores every case's input, options, seed and output in
``numpy_path_golden.npz``.  The tests replay the same randomness (oracle/numpy_path.py), inject
it into the C oracle and into the CUDA kernels, and require both outputs to equal the stored
reference output byte for byte.

For P = 8 the reference's ``MIN_PBLOCK_SIZE`` (16) is lowered for the call; the reference's
validator reads that module global (src/povs/common.py:90).  Seeds whose draw makes the
reference lose rows (a pblock written from a misaligned chunk, numpy.py:133-136) are skipped.

Usage: python tests/golden/make_golden.py <reference_root>   (the checkout holding src/povs)
"""

from __future__ import annotations

import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
REPO = HERE.parent.parent
OUT = HERE / "numpy_path_golden.npz"

# (name, n_rows, instance shape, dtype, P, V, iterations, offsets or None for the reference's defaults, seeds)
CASES = [
    ("f32_64x4", 64, (4,), "float32", 16, 2, 1, [0, 4], [0, 1, 42]),
    ("f32_128x8_refopts", 128, (8,), "float32", 16, 2, 3, [4, 8], [42, 7]),
    ("f32_128x2x4_auto", 128, (2, 4), "float32", None, None, 3, None, [42]),
    ("i32_1000x16_bias", 1000, (16,), "int32", 8, 2, 4, list(range(8)), [0, 1, 2, 3, 2999]),
    ("f16_1024x3", 1024, (3,), "float16", 16, 4, 2, [0, 8, 12], [5, 6]),
    ("i64_4096x2x2", 4096, (2, 2), "int64", 32, 8, 3, [0, 1, 2, 3, 5], [11]),
    ("u8_128x3x16x32", 128, (3, 16, 32), "uint8", 16, 2, 3, None, [2]),
]


def make_deck(n_rows: int, shape: tuple[int, ...], dtype: str, input_seed: int) -> np.ndarray:
    rng = np.random.default_rng(input_seed)
    if np.dtype(dtype).kind == "u":
        return rng.integers(0, 256, size=(n_rows, *shape), dtype=np.uint8).astype(dtype)
    if np.dtype(dtype).kind == "i":
        return rng.integers(-(2**30), 2**30, size=(n_rows, *shape)).astype(dtype)
    return (rng.standard_normal((n_rows, *shape)) * 100).astype(dtype)


def main(reference_root: str) -> None:
    sys.path.insert(0, str(REPO))
    sys.path.insert(0, str(Path(reference_root) / "src"))
    import povs as ref_povs  # the reference package
    import povs.common as ref_common
    from povs import Options

    from oracle.numpy_path import CorruptingDraw, numpy_path_randomness

    arrays: dict[str, np.ndarray] = {}
    names = []
    for name, n_rows, shape, dtype, P, V, iters, offsets, seeds in CASES:
        for seed in seeds:
            deck = make_deck(n_rows, shape, dtype, input_seed=1000 + seed)
            if P is None:
                opts = ref_povs.optim_options_for_dataset(deck)
            else:
                if offsets is None:
                    offsets = ref_common.choose_offsets(n_rows, int(np.prod(shape)), np.dtype(dtype).itemsize, P)
                opts = Options(virtual_block_size=V, physical_block_size=P, offsets=list(offsets))
            try:
                numpy_path_randomness(seed, n_rows, opts.physical_block_size, opts.virtual_block_size,
                                      list(opts.offsets), iters)
            except CorruptingDraw:
                print(f"skip {name} seed {seed}: the reference loses rows for this draw")
                continue
            out = deck.copy()
            saved = ref_common.MIN_PBLOCK_SIZE
            ref_common.MIN_PBLOCK_SIZE = min(saved, opts.physical_block_size)
            try:
                ref_povs.shuffle(out, iterations=iters, options=opts, seed=seed)
            finally:
                ref_common.MIN_PBLOCK_SIZE = saved
            key = f"{name}_s{seed}"
            names.append(key)
            arrays[f"{key}__input"] = deck
            arrays[f"{key}__output"] = out
            arrays[f"{key}__meta"] = np.array(
                [n_rows, opts.physical_block_size, opts.virtual_block_size, iters, seed], dtype=np.int64
            )
            arrays[f"{key}__offsets"] = np.array(opts.offsets, dtype=np.int64)
            print(f"{key}: P={opts.physical_block_size} V={opts.virtual_block_size} offsets={list(opts.offsets)}")
    arrays["cases"] = np.array(names)
    np.savez_compressed(OUT, **arrays)
    print(f"wrote {OUT} ({OUT.stat().st_size} bytes, {len(names)} cases)")


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit(__doc__.strip().splitlines()[-1])
    main(sys.argv[1])
