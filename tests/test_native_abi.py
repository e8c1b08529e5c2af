"""The C-ABI library loads and exports every symbol include/kq_b200.h declares (no GPU needed)."""
import ctypes
import re
from pathlib import Path

from kquant_b200 import _native, build

HEADER = Path(__file__).resolve().parents[1] / "include" / "kq_b200.h"


def _declared():
    text = re.sub(r"/\*.*?\*/", "", HEADER.read_text(), flags=re.S)
    return sorted(set(re.findall(r"\b(kq_[a-z0-9_]+)\s*\(", text)))


def test_header_declares_the_python_binding_set():
    assert set(_declared()) == set(_native.EXPORTED)


def test_library_builds_loads_and_exports_all_symbols():
    build.build()
    lib = ctypes.CDLL(str(_native.LIB_PATH))
    for name in _declared():
        assert hasattr(lib, name), name
    L = _native.load()
    assert L.kq_abi_version() == 1


def test_argument_errors_are_status_codes_not_crashes():
    L = _native.load()
    # invalid K and context are rejected before any device work
    assert L.kq_quantize_tiles_sqg(None, None, None, 4, None, 3, 128, None, 0, None) != 0
    assert L.kq_quantize_tiles_procedural(None, None, None, 1, 9, 1, 128, None, 0, None) != 0
    assert L.kq_pack_trellis(None, 1, 0, None, None) != 0
    assert L.kq_viterbi_encode(None, 1, 3, None, 0, None, None, None, 0, None) != 0
    assert b"" != L.kq_last_error()
