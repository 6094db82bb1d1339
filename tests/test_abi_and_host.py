"""CPU checks of the C-ABI library (loads, exports every declared symbol) and of the host-side
API logic that runs before any device call."""

from __future__ import annotations

import ctypes
import re

import numpy as np
import pytest
import torch

import povs
from povs import _build, _native

HEADERS = sorted((_build.INCLUDE_DIR).glob("*.h"))


def _declared_functions() -> set[str]:
    names: set[str] = set()
    for h in HEADERS:
        text = re.sub(r"/\*.*?\*/", "", h.read_text(), flags=re.S)
        names.update(re.findall(r"^[A-Za-z_][\w \*]*?\b(povs_\w+)\s*\(", text, flags=re.M))
    return names


def test_headers_declare_entry_points():
    names = _declared_functions()
    for required in ("povs_shuffle_v1", "povs_apply_v1", "povs_shuffle_host_v1", "povs_last_error_string"):
        assert required in names


def test_library_loads_and_exports_every_declared_symbol():
    lib = ctypes.CDLL(str(_build.LIB_PATH))
    missing = [n for n in sorted(_declared_functions()) if not hasattr(lib, n)]
    assert not missing, missing
    assert set(_native.SIGNATURES) == _declared_functions()


C_CALLER = r"""
#include <stdio.h>
#include "povs.h"
int main(void)
{
    int64_t offsets[2] = {0, 4};
    if (povs_version() < 100) return 2;
    /* A NULL deck is rejected on the host, before any device call. */
    int rc = povs_shuffle_v1(NULL, 64, 4, offsets, 2, 1, 16, 2, 42u, 0, NULL, 0);
    if (rc != POVS_ERR_INVALID_ARGUMENT) return 3;
    printf("%s\n", povs_last_error_string());
    return 0;
}
"""


def test_header_serves_plain_c_callers(tmp_path):
    """include/povs.h compiles as C99 and a C program links and calls the library."""
    import shutil
    import subprocess

    gcc = shutil.which("gcc")
    if gcc is None:
        pytest.skip("gcc is not available")
    src = tmp_path / "caller.c"
    src.write_text(C_CALLER)
    exe = tmp_path / "caller"
    lib = _build.LIB_PATH
    subprocess.run([gcc, "-std=c99", "-Wall", "-Werror", f"-I{_build.INCLUDE_DIR}", str(src), "-o", str(exe),
                    str(lib), f"-Wl,-rpath,{lib.parent}"], check=True, capture_output=True)
    out = subprocess.run([str(exe)], capture_output=True, text=True, timeout=120)
    assert out.returncode == 0, (out.returncode, out.stderr)
    assert "NULL" in out.stdout


def test_library_is_built_for_sm100a():
    params = povs.get_build_params()
    assert params.cuda_arch == ["100a"]
    assert params.cartesian_instancing is False


def test_version_and_error_string_without_gpu():
    lib = _native.load()
    assert lib.povs_version() >= 100
    assert isinstance(lib.povs_last_error_string(), bytes)


def test_invalid_arguments_are_rejected_before_any_device_call():
    lib = _native.load()
    offs = (ctypes.c_int64 * 2)(0, 4)
    # NULL data, too few rows, bad block sizes, out-of-range offsets: all host-side errors.
    assert lib.povs_shuffle_v1(None, 64, 4, offs, 2, 1, 16, 2, 0, 0, None, 0) == -1
    assert b"NULL" in lib.povs_last_error_string()
    assert lib.povs_shuffle_v1(ctypes.c_void_p(16), 1, 4, offs, 2, 1, 16, 2, 0, 0, None, 0) == -1
    assert lib.povs_shuffle_v1(ctypes.c_void_p(16), 64, 4, offs, 2, 1, 12, 2, 0, 0, None, 0) == -1
    assert lib.povs_shuffle_v1(ctypes.c_void_p(16), 64, 4, offs, 2, 1, 16, 3, 0, 0, None, 0) == -1
    assert lib.povs_shuffle_v1(ctypes.c_void_p(16), 64, 4, offs, 2, 1, 16, 64, 0, 0, None, 0) == -2
    bad = (ctypes.c_int64 * 2)(0, 64)
    assert lib.povs_shuffle_v1(ctypes.c_void_p(16), 64, 4, bad, 2, 1, 16, 2, 0, 0, None, 0) == -1
    assert b"offset" in lib.povs_last_error_string()
    many = (ctypes.c_int64 * 300)(*([0] * 300))
    assert lib.povs_shuffle_v1(ctypes.c_void_p(16), 64, 4, many, 300, 1, 16, 2, 0, 0, None, 0) == -2


def test_added_entry_points_reject_invalid_arguments_before_any_device_call():
    """Batched decks, mapped host decks and the metric kernels check their arguments on the host."""
    lib = _native.load()
    offs = (ctypes.c_int64 * 2)(0, 4)
    seeds = ctypes.c_void_p(64)
    data = ctypes.c_void_p(16)
    # Batched decks: NULL seeds, no decks, overlapping decks, unknown flags.
    assert lib.povs_shuffle_batch_v1(data, 2, 256, 64, 4, offs, 2, 1, 16, 2, None, 0, None, 0) == -1
    assert b"seeds" in lib.povs_last_error_string()
    assert lib.povs_shuffle_batch_v1(data, 0, 256, 64, 4, offs, 2, 1, 16, 2, seeds, 0, None, 0) == -1
    assert lib.povs_shuffle_batch_v1(data, 2, 100, 64, 4, offs, 2, 1, 16, 2, seeds, 0, None, 0) == -1
    assert b"deck_stride" in lib.povs_last_error_string()
    assert lib.povs_shuffle_batch_v1(data, 2, 256, 64, 4, offs, 2, 1, 16, 2, seeds, 0, None, 64) == -1
    assert b"flags" in lib.povs_last_error_string()
    # Mapped host decks: NULL deck, bad pblock.
    assert lib.povs_shuffle_mapped_v1(None, 64, 4, offs, 2, 1, 16, 2, 0, 0, None, 0) == -1
    assert lib.povs_shuffle_mapped_v1(data, 64, 4, offs, 2, 1, 12, 2, 0, 0, None, 0) == -1
    # Metric kernels: NULL ids, bad id width, unknown kind, n-gram degree below 2.
    counts = ctypes.c_void_p(32)
    assert lib.povs_travel_histogram_v1(None, 4, 10, 10, 10, 1, 0, 1, counts, 0, None) == -1
    assert lib.povs_travel_histogram_v1(data, 3, 10, 10, 10, 1, 0, 1, counts, 0, None) == -1
    assert b"id_bytes" in lib.povs_last_error_string()
    assert lib.povs_travel_histogram_v1(data, 4, 10, 10, 10, 1, 2, 1, counts, 0, None) == -1
    assert lib.povs_travel_histogram_v1(data, 4, 10, 10, 10, 1, 1, 0, counts, 0, None) == -1
    assert lib.povs_ngram_keys_v1(data, 8, 10, 10, 10, 1, 1, 1, None, 0, counts, 0, None) == -1
    assert b"degree" in lib.povs_last_error_string()
    assert lib.povs_ngram_keys_v1(data, 8, 0, 10, 10, 1, 3, 1, None, 0, counts, 0, None) == -1
    # n-gram counting: the table must be a power of two above the number of keys.
    tab = ctypes.c_void_p(128)
    assert lib.povs_ngram_count_v1(data, 8, 10, 10, 10, 1, 3, 1, None, 0, tab, 64, counts, 16, counts, 4, 0, None) == -1
    assert b"slots" in lib.povs_last_error_string()
    assert lib.povs_ngram_count_v1(data, 8, 10, 10, 10, 1, 3, 1, None, 0, tab, 256, counts, 1, counts, 4, 0, None) == -1
    assert lib.povs_ngram_count_v1(data, 8, 10, 10, 10, 1, 3, 1, None, 0, None, 256, counts, 16, counts, 4, 0, None) == -1
    # Allocation-free injection: only POVS_FLAG_SYNC is accepted.
    host = ctypes.c_void_p(64)
    for flags in (_native.FLAG_NO_GRAPH, _native.FLAG_REFERENCE_RNG, 8, 1 << 20):
        assert lib.povs_apply_static_v1(data, 64, 4, 16, 2, 1, offs, host, host, 1, 0, None, flags) == -1
        assert b"POVS_FLAG_SYNC" in lib.povs_last_error_string()


def test_unsupported_container_raises_type_error():
    with pytest.raises(TypeError):
        povs.shuffle([1, 2, 3])
    with pytest.raises(TypeError):
        povs.optim_options_for_dataset([1, 2, 3])


def test_host_options_match_reference_defaults():
    deck = np.zeros((128, 2, 4), dtype=np.float32)
    opts = povs.optim_options_for_dataset(deck)
    assert opts.virtual_block_size == 2 and opts.physical_block_size == 16
    assert opts.offsets == list(range(16))
    cpu = torch.zeros(128, 8)
    assert povs.optim_options_for_dataset(cpu) == povs.optim_options_for_dataset(cpu.numpy())


@pytest.mark.parametrize(
    "kwargs",
    [
        dict(iterations=0),
        dict(options=povs.Options(virtual_block_size=3, physical_block_size=16, offsets=[0, 4])),
        dict(options=povs.Options(virtual_block_size=2, physical_block_size=16, offsets=[0])),
        dict(options=povs.Options(virtual_block_size=2, physical_block_size=16, offsets=[0, 16])),
    ],
)
def test_host_preflight_errors(kwargs):
    deck = np.zeros((64, 4), dtype=np.float32)
    with pytest.raises(AssertionError):
        povs.shuffle(deck, seed=1, **{"iterations": 1, **kwargs})


def test_single_row_deck_rejected():
    with pytest.raises(AssertionError):
        povs.shuffle(np.zeros((1, 4), dtype=np.float32), options=povs.Options(2, 16, [0, 1]), seed=0)


@pytest.mark.skipif(torch.cuda.is_available(), reason="checks the no-GPU error path")
def test_host_route_requires_a_gpu():
    deck = np.arange(64 * 4, dtype=np.float32).reshape(64, 4)
    with pytest.raises(RuntimeError, match="CUDA device"):
        povs.shuffle(deck, seed=1)


def test_numpy_path_permutations_match_numpy():
    """The host restatement of MT19937 and NumPy's legacy shuffle (povs_mt19937.h) against
    numpy.random.RandomState itself, for the reference's seeds 1..999 and beyond."""
    lib = _native.load()
    for seed in list(range(0, 1000, 7)) + [999, 2**31, 2**32 - 1]:
        for n in (1, 2, 16, 17, 128, 1000):
            out = np.zeros(n, dtype=np.int32)
            assert lib.povs_numpy_path_perm_v1(seed, n, ctypes.c_void_p(out.ctypes.data)) == 0
            want = np.arange(n)
            np.random.RandomState(seed).shuffle(want)
            assert np.array_equal(out, want), (seed, n)
    assert lib.povs_numpy_path_perm_v1(1, -1, None) == -1
