"""Build recipe of libkairo_spmm.so (sm_100a) with nvcc, in-tree.

Each ``csrc/*.cu`` file is compiled to an object under ``kairo_b200/_build``
and linked into ``kairo_b200/libkairo_spmm.so``.  A rebuild happens only when a
source or header is newer than the library.  The CUDA runtime is linked
statically, so the library needs only the driver at run time.
"""

from __future__ import annotations

import concurrent.futures as cf
import os
import shutil
import subprocess
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
INCLUDE = ROOT / "include"
BUILD = PKG / "_build"
LIB = PKG / "libkairo_spmm.so"

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = [
    "-O3",
    "-std=c++17",
    "-lineinfo",
    "--expt-relaxed-constexpr",
    "-Xcompiler",
    "-fPIC",
    "-Xcompiler",
    "-fvisibility=hidden",
    f"-I{INCLUDE}",
] + ARCH_FLAGS


def nvcc_path() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found: the kairo_b200 CUDA library cannot be built")


def _sources() -> list[Path]:
    return sorted(CSRC.glob("*.cu"))


def _deps() -> list[Path]:
    return _sources() + sorted(CSRC.glob("*.cuh")) + sorted(CSRC.glob("*.h")) + sorted(INCLUDE.glob("*.h"))


def needs_build() -> bool:
    if not LIB.exists():
        return True
    t = LIB.stat().st_mtime
    return any(p.stat().st_mtime > t for p in _deps())


def build(verbose: bool = False, force: bool = False, ptxas_verbose: bool = False) -> Path:
    """Compile and link the library if it is missing or stale; returns its path."""
    if not force and not needs_build():
        return LIB
    nvcc = nvcc_path()
    BUILD.mkdir(exist_ok=True)
    flags = list(NVCC_FLAGS)
    if ptxas_verbose:
        flags += ["-Xptxas", "-v"]

    def compile_one(src: Path) -> tuple[Path, str]:
        obj = BUILD / (src.stem + ".o")
        cmd = [nvcc, *flags, "-c", str(src), "-o", str(obj)]
        res = subprocess.run(cmd, capture_output=True, text=True)
        if res.returncode != 0:
            raise RuntimeError(f"nvcc failed on {src.name}:\n{res.stdout}\n{res.stderr}")
        return obj, res.stdout + res.stderr

    with cf.ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 1)) as ex:
        results = list(ex.map(compile_one, _sources()))
    logs = "".join(r[1] for r in results)
    if verbose and logs:
        print(logs)
    tmp = LIB.with_suffix(".so.tmp")
    cmd = [nvcc, *ARCH_FLAGS, "-shared", "-o", str(tmp), *[str(o) for o, _ in results]]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"link of {LIB.name} failed:\n{res.stdout}\n{res.stderr}")
    os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    import sys

    build(verbose=True, force="--force" in sys.argv, ptxas_verbose="-v" in sys.argv)
    print(LIB)
