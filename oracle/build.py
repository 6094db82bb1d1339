"""Build recipe of the oracle (test infrastructure only).

* ``oracle/liboracle.so``            - the C/C++ restatements in this directory (gcc/g++).
* ``oracle/_ref/libref_host_rng.so`` - a driver compiled against the reference's own
  ``src/povs/__cuda/lib/utils.h`` (the host assignment shuffle).
* ``oracle/_ref/libref_povs_cuda.so`` - the reference's own CUDA path, ``src/povs/__cuda/lib/povs.cu``
  (its kernel and its host loop), compiled for sm_100a by ``ref_povs_cuda_driver.cu`` with the
  CUTLASS/CuTe headers that ship in the Python environment and a hand-written, empty stand-in for
  the instantiation file the reference's setup.py generates (``ref_gen/``).

The two reference-built libraries are compiled from the sources where they lie in a reference
checkout named by the environment variable ``POVS_REFERENCE_ROOT`` (the directory holding
``src/povs``).  Without it nothing under ``_ref`` is rebuilt and prebuilt files are used as they
are; the built files travel with the repository like the other ``.so`` files, so machines without
the checkout use them.  The reference's own build (setup.py) is never run.
"""

from __future__ import annotations

import importlib.util
import os
import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
ORACLE_LIB = HERE / "liboracle.so"
REF_DIR = HERE / "_ref"
REF_LIB = REF_DIR / "libref_host_rng.so"
REF_CUDA_LIB = REF_DIR / "libref_povs_cuda.so"
CUDA_HOME = Path(os.environ.get("CUDA_HOME", "/usr/local/cuda"))

C_SOURCES = [HERE / "povs_oracle.c"]
CXX_SOURCES = [HERE / "ref_cuda_rng.cpp"]
REF_CUDA_DRIVER = HERE / "ref_povs_cuda_driver.cu"
REF_GEN_DIR = HERE / "ref_gen"


def reference_root() -> Path | None:
    """The reference checkout named by POVS_REFERENCE_ROOT, or None."""
    root = os.environ.get("POVS_REFERENCE_ROOT")
    return Path(root) if root else None


def _ref_lib_dir() -> Path | None:
    root = reference_root()
    if root is None:
        return None
    lib_dir = root / "src" / "povs" / "__cuda" / "lib"
    return lib_dir if lib_dir.is_dir() else None


def cute_include_dir() -> Path | None:
    """CUTLASS/CuTe headers vendored in an installed Python package (found without importing it)."""
    for pkg, rel in (("flashinfer", "data/cutlass/include"), ("tilelang", "3rdparty/cutlass/include")):
        spec = importlib.util.find_spec(pkg)
        if spec is None or not spec.submodule_search_locations:
            continue
        cand = Path(list(spec.submodule_search_locations)[0]) / rel
        if (cand / "cute" / "tensor.hpp").exists():
            return cand
    return None


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
    """Compile the driver against the reference's utils.h, when the checkout is named."""
    lib_dir = _ref_lib_dir()
    driver = HERE / "ref_host_rng_driver.cpp"
    if lib_dir is None:
        return REF_LIB if REF_LIB.exists() else None
    header = lib_dir / "utils.h"
    if force or _stale(REF_LIB, [driver, header]):
        REF_DIR.mkdir(exist_ok=True)
        tmp = REF_LIB.with_suffix(".so.tmp")
        subprocess.run(
            ["g++", "-O2", "-fPIC", "-shared", "-std=c++17", f"-I{lib_dir}", f"-I{CUDA_HOME / 'include'}",
             "-o", str(tmp), str(driver)],
            check=True,
        )
        os.replace(tmp, REF_LIB)
    return REF_LIB


def ref_cuda_command(output: Path = REF_CUDA_LIB) -> list[str] | None:
    """nvcc command that compiles the reference's povs.cu through the driver (None if inputs are missing)."""
    lib_dir = _ref_lib_dir()
    cute = cute_include_dir()
    if lib_dir is None or cute is None:
        return None
    return [
        str(CUDA_HOME / "bin" / "nvcc"),
        "-std=c++20",  # the reference's own nvcc flags (setup.py:180-184)
        "-O3",
        "--use_fast_math",
        "--expt-relaxed-constexpr",  # as torch's extension builder passes it (CuTe needs it)
        "-gencode",
        "arch=compute_100a,code=sm_100a",
        "-lineinfo",
        "-Xcompiler",
        "-fPIC",
        "-shared",
        "-DPOVS_H",  # skip povs.h: a declaration of the template plus ATen, which the driver does not use
        f"-I{REF_GEN_DIR}",
        f"-I{lib_dir}",
        f"-I{cute}",
        "-o",
        str(output),
        str(REF_CUDA_DRIVER),
    ]


def build_ref_cuda(force: bool = False) -> Path | None:
    """Compile the reference's CUDA path into oracle/_ref, when the checkout is named."""
    lib_dir = _ref_lib_dir()
    if lib_dir is None:
        return REF_CUDA_LIB if REF_CUDA_LIB.exists() else None
    deps = [REF_CUDA_DRIVER, REF_GEN_DIR / "povs_cuda_template_instances.gen.inc", lib_dir / "povs.cu",
            lib_dir / "utils.h"]
    if force or _stale(REF_CUDA_LIB, deps):
        REF_DIR.mkdir(exist_ok=True)
        tmp = REF_CUDA_LIB.with_suffix(".so.tmp")
        cmd = ref_cuda_command(tmp)
        if cmd is None:
            return REF_CUDA_LIB if REF_CUDA_LIB.exists() else None
        # CuTe's headers print pages of warnings under these flags; keep them out of the log unless it fails.
        proc = subprocess.run(cmd, capture_output=True, text=True)
        if proc.returncode != 0:
            errors = [ln for ln in proc.stderr.splitlines() if "error" in ln]
            raise RuntimeError("reference CUDA build failed:\n" + "\n".join(errors[:20] or proc.stderr.splitlines()[-20:]))
        os.replace(tmp, REF_CUDA_LIB)
    return REF_CUDA_LIB


def build(force: bool = False) -> None:
    build_oracle(force)
    build_ref(force)
    build_ref_cuda(force)


if __name__ == "__main__":
    build(force="--force" in sys.argv)
    print(ORACLE_LIB)
    print(REF_LIB if REF_LIB.exists() else "(reference utils.h helper not built: set POVS_REFERENCE_ROOT)")
    print(REF_CUDA_LIB if REF_CUDA_LIB.exists() else "(reference CUDA path not built: set POVS_REFERENCE_ROOT)")
