"""Loader entry point with the reference's signature (mirrors kquant/exl3_loader.py:17-111).

The reference fabricates ``exllamav3.*`` package stubs and executes its
backend file from an ExLlamaV3 checkout.  This backend has no such
dependency, so ``load_qsrt_encoder`` ignores the checkout path and returns
``kquant_b200.exl3_encoder_backend``.  It also registers the module under
the name the reference uses, so code that looks it up in ``sys.modules``
finds it.
"""

from __future__ import annotations

import sys
import types
from pathlib import Path

from . import exl3_encoder_backend

_BACKEND_MODULE = "exllamav3.modules.quant.exl3_lib.kquant_qsrt_encoder"


def load_qsrt_encoder(exllamav3_root: str | Path | None = None) -> types.ModuleType:
    sys.modules.setdefault(_BACKEND_MODULE, exl3_encoder_backend)
    return exl3_encoder_backend
