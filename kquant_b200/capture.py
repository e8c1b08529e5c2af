"""Hessian accumulation H = sum_t w_t x_t x_t^T on the tensor cores.

Mirrors kquant/capture.py:713-730 (``_accumulate_hessian``): rows [T, d]
and weights [T] stream in chunks of ``chunk_rows``; returns (accumulator
[d, d] fp32, denominator = sum of weights).  Each chunk is one call of
``kq_accumulate_hessian``: an operand kernel (transpose, weighting, TF32
hi/lo split) and one tcgen05 GEMM over the upper-triangle tiles, mirrored.
Precision ``"3xtf32"`` (default) accumulates hi*hi + hi*lo + lo*hi and
drains the tensor-core accumulator into fp32 registers every 128 samples,
which matches the accuracy of the reference's FP32 addmm; ``"tf32"``
issues the single TF32 product.  The result is exactly symmetric.
"""

from __future__ import annotations

import torch

from . import _native

_SPLIT = {"3xtf32": 3, "tf32": 1}


def accumulate_hessian(rows: torch.Tensor, weights: torch.Tensor, *, device: torch.device, chunk_rows: int,
                       precision: str = "3xtf32", out: torch.Tensor | None = None) -> tuple[torch.Tensor, float]:
    if rows.ndim != 2 or weights.ndim != 1 or rows.shape[0] != weights.shape[0]:
        raise ValueError("invalid Hessian sample shapes")
    if precision not in _SPLIT:
        raise ValueError("precision must be '3xtf32' or 'tf32'")
    device = torch.device(device)
    if device.type != "cuda":
        raise ValueError("accumulate_hessian requires a CUDA device (kquant_b200 has no CPU path)")
    dim = int(rows.shape[1])
    acc = out if out is not None else torch.zeros((dim, dim), dtype=torch.float32, device=device)
    den = torch.zeros((), dtype=torch.float64, device=device)
    step = max(int(chunk_rows), 1)
    ws = None
    for start in range(0, int(rows.shape[0]), step):
        x = rows[start:start + step].to(device=device, dtype=torch.float32).contiguous()
        w = weights[start:start + step].to(device=device, dtype=torch.float32).contiguous()
        den += w.double().sum()
        ws = _native.accumulate_hessian(x, w, acc, _SPLIT[precision], ws)
    _native.check_trace_errors()
    return acc, float(den.item())


# the reference's private name, for callers that import it directly
_accumulate_hessian = accumulate_hessian
