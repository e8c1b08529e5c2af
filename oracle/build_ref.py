"""Compile the reference's own CUDA Viterbi extension into ``oracle/_ref/`` (test infrastructure).

The sources are read where they lie (``<reference>/kquant/csrc/sqg_quantize.cpp``,
``sqg_quantize.cu`` and the headers next to them).  This recipe invokes nvcc
and g++ directly with torch's include paths.  It does not use the reference's
JIT loader.  Nothing is copied into this repository.  The resulting
``oracle/_ref/kquant_ref_sqg.so`` is a Python extension module exposing the
reference binding ``quantize_tiles_sqg`` / ``quantize_tiles_procedural``
(kquant/csrc/sqg_quantize.cpp:23-33).  The GPU parity tests use it as the
bit-exact oracle; ``oracle/_ref`` is git-ignored but travels to the GPU box.

Flags follow the reference's own build (kquant/sqg_quantizer.py:15-36):
-O3 --use_fast_math -lineinfo, here for sm_100a.
"""

from __future__ import annotations

import os
import subprocess
import sys
import sysconfig
from pathlib import Path

HERE = Path(__file__).resolve().parent
OUT_DIR = HERE / "_ref"
MODULE = "kquant_ref_sqg"
OUT = OUT_DIR / f"{MODULE}.so"


def default_root() -> Path:
    """The reference checkout: $KQ_REFERENCE_ROOT, else a ``reference`` directory beside this repository."""
    env = os.environ.get("KQ_REFERENCE_ROOT")
    return Path(env) if env else HERE.parents[1] / "reference"


DEFAULT_REF = default_root()


def available(ref_root: Path = DEFAULT_REF) -> bool:
    return (ref_root / "kquant" / "csrc" / "sqg_quantize.cu").exists()


def build(ref_root: Path = DEFAULT_REF, force: bool = False) -> Path | None:
    if OUT.exists() and not force:
        return OUT
    if not available(ref_root):
        return None
    import torch
    from torch.utils import cpp_extension as ce

    csrc = ref_root / "kquant" / "csrc"
    OUT_DIR.mkdir(exist_ok=True)
    incs = [f"-I{p}" for p in ce.include_paths(device_type="cuda")] + [
        f"-I{sysconfig.get_paths()['include']}", f"-I{csrc}"]
    abi = f"-D_GLIBCXX_USE_CXX11_ABI={int(torch._C._GLIBCXX_USE_CXX11_ABI)}"
    defs = [f"-DTORCH_EXTENSION_NAME={MODULE}", "-DTORCH_API_INCLUDE_EXTENSION_H", abi]
    nvcc = os.environ.get("CUDA_HOME", "/usr/local/cuda") + "/bin/nvcc"
    cu_obj = OUT_DIR / "sqg_quantize_cu.o"
    cpp_obj = OUT_DIR / "sqg_quantize_cpp.o"
    cmds = [
        [nvcc, "-c", str(csrc / "sqg_quantize.cu"), "-o", str(cu_obj), "-Xcompiler", "-fPIC", "-std=c++17",
         "-O3", "--use_fast_math", "-lineinfo", "-gencode", "arch=compute_100a,code=sm_100a",
         "--expt-relaxed-constexpr", "-Xcudafe", "--diag_suppress=177", "-Xcudafe", "--diag_suppress=20012",
         "-D__CUDA_NO_HALF_OPERATORS__", "-D__CUDA_NO_HALF_CONVERSIONS__", "-D__CUDA_NO_HALF2_OPERATORS__",
         "-D__CUDA_NO_BFLOAT16_CONVERSIONS__", *defs, *incs],
        ["g++", "-c", str(csrc / "sqg_quantize.cpp"), "-o", str(cpp_obj), "-fPIC", "-std=c++17", "-O3",
         *defs, *incs],
    ]
    procs = [subprocess.Popen(c) for c in cmds]
    if any(p.wait() for p in procs):
        raise RuntimeError("reference extension compile failed")
    libdir = Path(torch.__file__).parent / "lib"
    link = ["g++", "-shared", "-o", str(OUT), str(cu_obj), str(cpp_obj), f"-L{libdir}",
            "-lc10", "-lc10_cuda", "-ltorch", "-ltorch_cpu", "-ltorch_cuda", "-ltorch_python",
            f"-L{os.environ.get('CUDA_HOME', '/usr/local/cuda')}/lib64", "-lcudart", f"-Wl,-rpath,{libdir}"]
    subprocess.run(link, check=True)
    for o in (cu_obj, cpp_obj):
        o.unlink(missing_ok=True)
    return OUT


HARNESS = OUT_DIR / "kquant_ref_harness.so"


def build_harness(ref_root: Path = DEFAULT_REF, force: bool = False) -> Path | None:
    """Compile oracle/ref_harness.cu (the reference's sqg_quantize.cu for every K in 1..8) into oracle/_ref."""
    if HARNESS.exists() and not force:
        return HARNESS
    if not available(ref_root):
        return None
    import torch
    from torch.utils import cpp_extension as ce

    csrc = ref_root / "kquant" / "csrc"
    OUT_DIR.mkdir(exist_ok=True)
    incs = [f"-I{p}" for p in ce.include_paths(device_type="cuda")] + [
        f"-I{sysconfig.get_paths()['include']}", f"-I{csrc}"]
    abi = f"-D_GLIBCXX_USE_CXX11_ABI={int(torch._C._GLIBCXX_USE_CXX11_ABI)}"
    nvcc = os.environ.get("CUDA_HOME", "/usr/local/cuda") + "/bin/nvcc"
    obj = OUT_DIR / "ref_harness.o"
    cmd = [nvcc, "-c", str(HERE / "ref_harness.cu"), "-o", str(obj), "-Xcompiler", "-fPIC", "-std=c++17",
           "-O3", "--use_fast_math", "-lineinfo", "-gencode", "arch=compute_100a,code=sm_100a",
           "--expt-relaxed-constexpr", "-Xcudafe", "--diag_suppress=177", "-Xcudafe", "--diag_suppress=20012",
           "-D__CUDA_NO_HALF_OPERATORS__", "-D__CUDA_NO_HALF_CONVERSIONS__", "-D__CUDA_NO_HALF2_OPERATORS__",
           "-D__CUDA_NO_BFLOAT16_CONVERSIONS__", "-DTORCH_EXTENSION_NAME=kquant_ref_harness",
           "-DTORCH_API_INCLUDE_EXTENSION_H", abi, *incs]
    subprocess.run(cmd, check=True)
    libdir = Path(torch.__file__).parent / "lib"
    link = ["g++", "-shared", "-o", str(HARNESS), str(obj), f"-L{libdir}", "-lc10", "-lc10_cuda", "-ltorch",
            "-ltorch_cpu", "-ltorch_cuda", "-ltorch_python",
            f"-L{os.environ.get('CUDA_HOME', '/usr/local/cuda')}/lib64", "-lcudart", f"-Wl,-rpath,{libdir}"]
    subprocess.run(link, check=True)
    obj.unlink(missing_ok=True)
    return HARNESS


def load_harness():
    """ctypes handle of the compiled harness (needs `import torch` first)."""
    import ctypes
    import torch  # noqa: F401
    if not HARNESS.exists():
        raise FileNotFoundError(f"{HARNESS} not built")
    lib = ctypes.CDLL(str(HARNESS))
    P, I = ctypes.c_void_p, ctypes.c_int
    lib.kqref_quantize_procedural.argtypes = [P, P, P, P, P, I, I, I, I, I, P]
    lib.kqref_quantize_procedural.restype = I
    lib.kqref_decision_bytes_per_tile.argtypes = [I]
    lib.kqref_decision_bytes_per_tile.restype = ctypes.c_longlong
    return lib


def load():
    """Import the compiled reference extension (needs `import torch` first)."""
    import importlib.util
    import torch  # noqa: F401
    if not OUT.exists():
        raise FileNotFoundError(f"{OUT} not built")
    spec = importlib.util.spec_from_file_location(MODULE, OUT)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


if __name__ == "__main__":
    args = [a for a in sys.argv[1:] if not a.startswith("--")]
    root = Path(args[0]) if args else DEFAULT_REF
    print(build(root, force="--force" in sys.argv))
    print(build_harness(root, force="--force" in sys.argv))
