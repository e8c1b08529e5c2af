"""ctypes front end of the CPU oracle (test infrastructure only).

Only ``tests/``, ``__graft_entry__.smoke()`` and the CPU-baseline legs of
``bench.py`` import this module.  It is a checker, never a product path.
The C source is ``oracle/kq_oracle.c``.  It restates the reference encoder
(``kquant/csrc/qsrt_quantize_tiles_kernel.cuh:21-471``, ``kquant/qsrt.py:811-857``,
``kquant/exl3_reference.py:37-61``).
"""

from __future__ import annotations

import ctypes
import os
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIB_PATH = HERE / "_build" / "libkq_oracle.so"

CB_3INST = 0
CB_MCG = 1
CB_MUL1 = 2
CB_SQG = 4

_lib = None


def build() -> Path:
    """Compile the oracle with its Makefile (gcc, OpenMP)."""
    subprocess.run(["make", "-s", "-C", str(HERE)], check=True)
    return LIB_PATH


def lib():
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            build()
        L = ctypes.CDLL(str(LIB_PATH))
        P = ctypes.c_void_p
        L.kqo_build_labels.argtypes = [ctypes.c_int, P, P]
        L.kqo_viterbi.argtypes = [ctypes.c_int, P, P, ctypes.c_int64, ctypes.c_int, P, P, ctypes.c_int]
        L.kqo_pack_trellis.argtypes = [P, ctypes.c_int64, ctypes.c_int, P]
        L.kqo_unpack_trellis.argtypes = [P, ctypes.c_int64, ctypes.c_int, P]
        L.kqo_reconstruct_states.argtypes = [P, ctypes.c_int64, ctypes.c_int, P]
        for name in ("kqo_hsub", "kqo_hmul"):
            getattr(L, name).argtypes = [ctypes.c_uint16, ctypes.c_uint16]
            getattr(L, name).restype = ctypes.c_uint16
        for name in ("kqo_hfma", "kqo_hfma_exact"):
            getattr(L, name).argtypes = [ctypes.c_uint16] * 3
            getattr(L, name).restype = ctypes.c_uint16
        L.kqo_f2h.argtypes = [ctypes.c_float]
        L.kqo_f2h.restype = ctypes.c_uint16
        _lib = L
    return _lib


def _ptr(a: np.ndarray):
    return a.ctypes.data_as(ctypes.c_void_p)


def labels(kind: int, lut: np.ndarray | None = None) -> np.ndarray:
    """65,536 binary16 labels (as uint16 bits) of a codebook, indexed by state."""
    out = np.empty(65536, dtype=np.uint16)
    lut_arr = None
    if kind == CB_SQG:
        lut_arr = np.ascontiguousarray(lut, dtype=np.uint8)
        assert lut_arr.size == 65536
    rc = lib().kqo_build_labels(kind, _ptr(lut_arr) if lut_arr is not None else None, _ptr(out))
    if rc != 0:
        raise ValueError(f"kqo_build_labels failed: {rc}")
    return out


def viterbi(K: int, label_bits: np.ndarray, tiles: np.ndarray, C: int = 128,
            threads: int = 0) -> tuple[np.ndarray, np.ndarray, int]:
    """Encode [n, 256] fp32 tiles; returns (states uint16, values fp32, status)."""
    tiles = np.ascontiguousarray(tiles, dtype=np.float32).reshape(-1, 256)
    label_bits = np.ascontiguousarray(label_bits, dtype=np.uint16)
    n = tiles.shape[0]
    idx = np.zeros((n, 256), dtype=np.uint16)
    val = np.zeros((n, 256), dtype=np.float32)
    rc = lib().kqo_viterbi(K, _ptr(label_bits), _ptr(tiles), n, C, _ptr(idx), _ptr(val),
                           int(threads or os.cpu_count() or 1))
    if rc not in (0, -3):
        raise ValueError(f"kqo_viterbi failed: {rc}")
    return idx, val, rc


def pack_trellis(states: np.ndarray, K: int) -> np.ndarray:
    s = np.ascontiguousarray(states, dtype=np.int16).reshape(-1, 256)
    out = np.empty((s.shape[0], 16 * K), dtype=np.int16)
    assert lib().kqo_pack_trellis(_ptr(s), s.shape[0], K, _ptr(out)) == 0
    return out.reshape(*states.shape[:-1], 16 * K)


def unpack_trellis(packed: np.ndarray, K: int) -> np.ndarray:
    p = np.ascontiguousarray(packed, dtype=np.int16).reshape(-1, 16 * K)
    out = np.empty((p.shape[0], 256), dtype=np.int16)
    assert lib().kqo_unpack_trellis(_ptr(p), p.shape[0], K, _ptr(out)) == 0
    return out.reshape(*packed.shape[:-1], 256)


def reconstruct_states(edges: np.ndarray, K: int) -> np.ndarray:
    e = np.ascontiguousarray(edges, dtype=np.int16).reshape(-1, 256)
    out = np.empty_like(e)
    assert lib().kqo_reconstruct_states(_ptr(e), e.shape[0], K, _ptr(out)) == 0
    return out.reshape(edges.shape)
