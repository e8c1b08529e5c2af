"""Build recipe for the kquant_b200 CUDA library (sm_100a only).

``python -m kquant_b200.build`` compiles every ``csrc/*.cu`` with nvcc into
``kquant_b200/_kq_b200.so`` in the package directory.  The shared object is
loaded with ctypes and exports exactly the C ABI of ``include/kq_b200.h``.
No torch types cross the boundary.
"""

from __future__ import annotations

import os
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
BUILD = PKG / "_build"
LIB = PKG / "_kq_b200.so"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "--expt-relaxed-constexpr",
              "-I", str(ROOT / "include")]


def nvcc() -> str:
    cand = os.environ.get("CUDA_HOME", "/usr/local/cuda") + "/bin/nvcc"
    return cand if Path(cand).exists() else "nvcc"


def sources() -> list[Path]:
    return sorted(CSRC.glob("*.cu"))


def _stale() -> bool:
    if not LIB.exists():
        return True
    t = LIB.stat().st_mtime
    deps = sources() + sorted(CSRC.glob("*.cuh")) + sorted(CSRC.glob("*.inc")) + [ROOT / "include" / "kq_b200.h", Path(__file__)]
    return any(p.stat().st_mtime > t for p in deps)


def build(force: bool = False, verbose: bool = False) -> Path:
    """Compile csrc/*.cu for sm_100a and link ``_kq_b200.so``; returns its path."""
    if not force and not _stale():
        return LIB
    BUILD.mkdir(exist_ok=True)
    objs = []
    procs = []
    for src in sources():
        obj = BUILD / (src.stem + ".o")
        cmd = [nvcc(), *ARCH, *NVCC_FLAGS, "-c", str(src), "-o", str(obj)]
        if verbose:
            cmd.insert(1, "-Xptxas=-v")
        procs.append((subprocess.Popen(cmd, stdout=subprocess.PIPE, stderr=subprocess.STDOUT, text=True), src))
        objs.append(obj)
    failed = []
    for p, src in procs:
        out, _ = p.communicate()
        if verbose or p.returncode:
            sys.stderr.write(out)
        if p.returncode:
            failed.append(src.name)
    if failed:
        raise RuntimeError(f"nvcc failed for {failed}")
    tmp = LIB.with_suffix(".so.tmp")
    subprocess.run([nvcc(), *ARCH, "-shared", "-o", str(tmp), *map(str, objs), "-cudart", "static"], check=True)
    os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose="-v" in sys.argv)
    print(LIB)
