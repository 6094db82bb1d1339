"""Build recipe of the oracle (test infrastructure only).

* ``oracle/liboracle.so``           - the C/C++ restatements in this directory (gcc/g++).
* ``oracle/_ref/libref_host_rng.so`` - a driver compiled against the reference's own
  ``src/povs/__cuda/lib/utils.h`` where it lies under the reference checkout (only when that
  checkout exists; the built file then travels with the repository like the other .so files).

The reference's CUDA kernel itself (src/povs/__cuda/lib/povs.cu) is not built: it needs the
CUTLASS/CuTe headers and generated dispatch code.
"""

from __future__ import annotations

import os
import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
ORACLE_LIB = HERE / "liboracle.so"
REF_DIR = HERE / "_ref"
REF_LIB = REF_DIR / "libref_host_rng.so"
REFERENCE_ROOT = Path(os.environ.get("POVS_REFERENCE_ROOT", "/root/reference"))
REF_UTILS_DIR = REFERENCE_ROOT / "src" / "povs" / "__cuda" / "lib"
CUDA_INCLUDE = Path(os.environ.get("CUDA_HOME", "/usr/local/cuda")) / "include"

C_SOURCES = [HERE / "povs_oracle.c"]
CXX_SOURCES = [HERE / "ref_cuda_rng.cpp"]


def _stale(target: Path, deps: list[Path]) -> bool:
    return not target.exists() or any(d.stat().st_mtime > target.stat().st_mtime for d in deps)


def build_oracle(force: bool = False) -> Path:
    deps = C_SOURCES + CXX_SOURCES
    if force or _stale(ORACLE_LIB, deps):
        objs = []
        for src in C_SOURCES:
            obj = HERE / (src.stem + ".o")
            subprocess.run(["gcc", "-O2", "-fPIC", "-std=c11", "-c", str(src), "-o", str(obj)], check=True)
            objs.append(obj)
        for src in CXX_SOURCES:
            obj = HERE / (src.stem + ".o")
            subprocess.run(["g++", "-O2", "-fPIC", "-std=c++17", "-c", str(src), "-o", str(obj)], check=True)
            objs.append(obj)
        tmp = ORACLE_LIB.with_suffix(".so.tmp")
        subprocess.run(["g++", "-shared", "-o", str(tmp), *map(str, objs), "-lpthread"], check=True)
        os.replace(tmp, ORACLE_LIB)
        for obj in objs:
            obj.unlink(missing_ok=True)
    return ORACLE_LIB


def build_ref(force: bool = False) -> Path | None:
    """Compile the reference-header driver, when the reference checkout is present."""
    header = REF_UTILS_DIR / "utils.h"
    driver = HERE / "ref_host_rng_driver.cpp"
    if not header.exists():
        return REF_LIB if REF_LIB.exists() else None
    if force or _stale(REF_LIB, [driver, header]):
        REF_DIR.mkdir(exist_ok=True)
        tmp = REF_LIB.with_suffix(".so.tmp")
        subprocess.run(
            [
                "g++",
                "-O2",
                "-fPIC",
                "-shared",
                "-std=c++17",
                f"-I{REF_UTILS_DIR}",
                f"-I{CUDA_INCLUDE}",
                "-o",
                str(tmp),
                str(driver),
            ],
            check=True,
        )
        os.replace(tmp, REF_LIB)
    return REF_LIB


def build(force: bool = False) -> None:
    build_oracle(force)
    build_ref(force)


if __name__ == "__main__":
    build(force="--force" in sys.argv)
    print(ORACLE_LIB, REF_LIB if REF_LIB.exists() else "(reference helper not built)")
