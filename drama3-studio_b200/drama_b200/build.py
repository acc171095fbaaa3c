"""Build the sm_100a C-ABI library in-tree (``drama_b200/lib/libdrama_b200.so``).

nvcc cross-compiles without a GPU; every translation unit is compiled for
``-gencode arch=compute_100a,code=sm_100a`` only. The library links the CUDA
runtime statically and exports only the ``drama_b200_*`` symbols declared in
``include/drama_b200.h``.
"""

from __future__ import annotations

import concurrent.futures
import os
import shutil
import subprocess
from pathlib import Path

PACKAGE = Path(__file__).resolve().parent
SOURCE_ROOT = PACKAGE.parent
CSRC = SOURCE_ROOT / "csrc"
INCLUDE = SOURCE_ROOT.parent / "include"
LIB_DIR = PACKAGE / "lib"
LIB_PATH = LIB_DIR / "libdrama_b200.so"
BUILD_DIR = SOURCE_ROOT / "_build"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = [
    "-O3", "-lineinfo", "-std=c++20", "--expt-relaxed-constexpr",
    "-Xcompiler", "-fPIC,-fvisibility=hidden", "-Xptxas", "-warn-spills",
]


def cutlass_include() -> Path:
    """A CUTLASS / CuTe header tree with the sm100 UMMA headers.

    DRAMA_B200_CUTLASS_INCLUDE, else the copy that ships inside an installed
    package of this environment (flashinfer, tilelang). Only the headers are
    used (the tcgen05 descriptor unions, MMA, TMEM-allocation and commit
    wrappers); nothing is linked.
    """
    import importlib.util

    candidates = []
    if os.environ.get("DRAMA_B200_CUTLASS_INCLUDE"):
        candidates.append(Path(os.environ["DRAMA_B200_CUTLASS_INCLUDE"]))
    for package, sub in (("flashinfer", "data/cutlass/include"), ("tilelang", "3rdparty/cutlass/include")):
        spec = importlib.util.find_spec(package)
        if spec is not None and spec.submodule_search_locations:
            candidates.append(Path(list(spec.submodule_search_locations)[0]) / sub)
    for path in candidates:
        if (path / "cute" / "arch" / "mma_sm100_umma.hpp").is_file():
            return path
    raise RuntimeError("no CUTLASS header tree with cute/arch/mma_sm100_umma.hpp found; "
                       "set DRAMA_B200_CUTLASS_INCLUDE")


def nvcc() -> str:
    found = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not Path(found).exists():
        raise RuntimeError("nvcc not found; the CUDA toolkit is required to build drama_b200")
    return found


def sources() -> list[Path]:
    return sorted(CSRC.glob("*.cu"))


def _stale(target: Path, deps: list[Path]) -> bool:
    if not target.exists():
        return True
    t = target.stat().st_mtime
    return any(d.stat().st_mtime > t for d in deps)


def build(verbose: bool = False, force: bool = False, ptxas_info: bool = False) -> Path:
    """Compile every ``csrc/*.cu`` and link the shared library; returns its path."""
    BUILD_DIR.mkdir(parents=True, exist_ok=True)
    LIB_DIR.mkdir(parents=True, exist_ok=True)
    headers = sorted(CSRC.glob("*.cuh")) + sorted(CSRC.glob("*.h")) + sorted(INCLUDE.glob("*.h"))
    compiler = nvcc()
    objects = []
    jobs = []
    for src in sources():
        obj = BUILD_DIR / (src.stem + ".o")
        objects.append(obj)
        if force or _stale(obj, [src, *headers, Path(__file__)]):
            cmd = [compiler, *ARCH, *NVCC_FLAGS, f"-I{INCLUDE}", f"-I{CSRC}", "-c", str(src), "-o", str(obj)]
            if "umma.cuh" in src.read_text():
                cmd[1:1] = [f"-I{cutlass_include()}"]
            if ptxas_info:
                cmd[1:1] = ["-Xptxas", "-v"]
            jobs.append(cmd)

    def run(cmd):
        proc = subprocess.run(cmd, capture_output=True, text=True)
        if proc.returncode != 0:
            raise RuntimeError(f"nvcc failed:\n{' '.join(cmd)}\n{proc.stdout}\n{proc.stderr}")
        return proc.stdout + proc.stderr

    with concurrent.futures.ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 1)) as pool:
        for out in pool.map(run, jobs):
            if verbose and out.strip():
                print(out)
    if force or jobs or _stale(LIB_PATH, objects):
        cmd = [compiler, *ARCH, "-shared", "-o", str(LIB_PATH), *map(str, objects), "-Xcompiler", "-fPIC"]
        out = run(cmd)
        if verbose and out.strip():
            print(out)
    return LIB_PATH


if __name__ == "__main__":
    import sys

    print(build(verbose=True, force="--force" in sys.argv, ptxas_info="-v" in sys.argv))
