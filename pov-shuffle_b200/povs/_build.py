"""In-tree build of the sm_100a CUDA library ``libpovs_sm100.so``.

Replaces the reference's setup.py template-instantiation build (setup.py:14-28,110-197):
the kernels here are runtime-general in (V, P, row bytes), so one library serves every
configuration and ``build_params.json`` records only the target architecture.
"""

from __future__ import annotations

import json
import os
import shutil
import subprocess
from pathlib import Path

PKG_DIR = Path(__file__).resolve().parent
CSRC_DIR = PKG_DIR.parent / "csrc"
INCLUDE_DIR = PKG_DIR.parent.parent / "include"
LIB_NAME = "libpovs_sm100.so"
LIB_PATH = PKG_DIR / LIB_NAME
BUILD_PARAMS_PATH = PKG_DIR / "build_params.json"
CUDA_ARCH = "100a"

SOURCES = [CSRC_DIR / "povs_abi.cu"]
DEPENDS = [*SOURCES, CSRC_DIR / "povs_kernel.cuh", CSRC_DIR / "povs_rng.cuh", CSRC_DIR / "povs_metrics.cuh",
           CSRC_DIR / "povs_mt19937.h", INCLUDE_DIR / "povs.h"]


def _nvcc() -> str:
    cuda_home = os.environ.get("CUDA_HOME", "/usr/local/cuda")
    cand = Path(cuda_home) / "bin" / "nvcc"
    if cand.exists():
        return str(cand)
    found = shutil.which("nvcc")
    if not found:
        raise RuntimeError("nvcc not found: set CUDA_HOME or put nvcc on PATH")
    return found


def nvcc_command(output: Path = LIB_PATH, debug: bool = False) -> list[str]:
    cmd = [
        _nvcc(),
        "-gencode",
        f"arch=compute_{CUDA_ARCH},code=sm_{CUDA_ARCH}",
        "-lineinfo",
        "-std=c++17",
        "-Xcompiler",
        "-fPIC",
        "-shared",
        "-O3",
        "-o",
        str(output),
        *(str(s) for s in SOURCES),
    ]
    if debug:
        cmd.insert(-len(SOURCES), "-DPOVS_DEBUG=1")
    return cmd


def is_stale() -> bool:
    if not LIB_PATH.exists() or not BUILD_PARAMS_PATH.exists():
        return True
    built = LIB_PATH.stat().st_mtime
    return any(dep.stat().st_mtime > built for dep in DEPENDS)


def write_build_params(debug: bool = False) -> None:
    params = {
        "debug_mode": debug,
        "cuda_arch": [CUDA_ARCH],
        "vblock_sizes": [],
        "pblock_sizes": [],
        "instance_sizes": [],
        "cartesian_instancing": False,
        "instantiations": [],
        "instantiations_all_types": [],
    }
    BUILD_PARAMS_PATH.write_text(json.dumps(params, indent=2) + "\n")


def build(force: bool = False, verbose: bool = False, debug: bool = False) -> Path:
    """Compile the library in place (next to this file) unless it is up to date."""
    if force or is_stale():
        cmd = nvcc_command(debug=debug)
        if verbose:
            print(" ".join(cmd), flush=True)
        tmp = LIB_PATH.with_suffix(".so.tmp")
        cmd[cmd.index(str(LIB_PATH))] = str(tmp)
        subprocess.run(cmd, check=True)
        os.replace(tmp, LIB_PATH)
        write_build_params(debug)
    return LIB_PATH


if __name__ == "__main__":
    import sys

    build(force="--force" in sys.argv, verbose=True, debug="--debug" in sys.argv)
    print(LIB_PATH)
