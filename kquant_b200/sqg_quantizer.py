"""Tile-quantizer hook of kquant's encoder (mirrors kquant/sqg_quantizer.py:59-164).

The reference patches ``module.quantize_tiles`` so that SQG LUTs reach its
CUDA extension.  ``kquant_b200.exl3_encoder_backend.quantize_tiles`` already
dispatches SQG / MCG / MUL1 / 3INST to the native sm_100a kernel, so
installing on this backend only records the flag.  Installing on any other
module routes its ``quantize_tiles`` through this backend's implementation.
"""

from __future__ import annotations

from . import exl3_encoder_backend as _backend


def install_sqg_quantizer(quantizer_module) -> None:
    if getattr(quantizer_module, "_kquant_sqg_installed", False):
        return
    if quantizer_module is not _backend:
        quantizer_module.quantize_tiles = _backend.quantize_tiles
    quantizer_module._kquant_sqg_installed = True
