"""Hessian accumulation H = sum_t w_t x_t x_t^T on the tensor cores.

Mirrors kquant/capture.py:713-730 (``_accumulate_hessian``): rows [T, d]
and weights [T] stream in chunks; returns (accumulator [d, d] fp32,
denominator = sum of weights).  Each chunk is X^T diag(w) X, computed by
the tcgen05 GEMM kernel (``kq_gemm_abt_tf32``) with operands X^T and
(w X)^T.  Precision ``"3xtf32"`` (default) splits every operand into a TF32
high part and its remainder and accumulates hi*hi + hi*lo + lo*hi, which
keeps the result at FP32-level accuracy (relative error ~2^-21 per
product); ``"tf32"`` issues the single product.  Shapes the kernel does not
tile (d not a multiple of 256) use FP32 addmm on the same device.
"""

from __future__ import annotations

import torch

from . import _native


def _split_tf32(t: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    hi = (t.view(torch.int32) & ~0x1FFF).view(torch.float32)
    return hi, t - hi


def accumulate_hessian(rows: torch.Tensor, weights: torch.Tensor, *, device: torch.device, chunk_rows: int,
                       precision: str = "3xtf32", out: torch.Tensor | None = None) -> tuple[torch.Tensor, float]:
    if rows.ndim != 2 or weights.ndim != 1 or rows.shape[0] != weights.shape[0]:
        raise ValueError("invalid Hessian sample shapes")
    if precision not in ("3xtf32", "tf32"):
        raise ValueError("precision must be '3xtf32' or 'tf32'")
    device = torch.device(device)
    if device.type != "cuda":
        raise ValueError("accumulate_hessian requires a CUDA device (kquant_b200 has no CPU path)")
    dim = int(rows.shape[1])
    acc = out if out is not None else torch.zeros((dim, dim), dtype=torch.float32, device=device)
    den = torch.zeros((), dtype=torch.float64, device=device)
    step = max(int(chunk_rows), 1)
    tiled = dim % 256 == 0
    for start in range(0, int(rows.shape[0]), step):
        x = rows[start:start + step].to(device=device, dtype=torch.float32)
        w = weights[start:start + step].to(device=device, dtype=torch.float32)
        den += w.double().sum()
        if not tiled:
            acc.addmm_(x.T, x * w.unsqueeze(1))
            continue
        pad = (-x.shape[0]) % 32
        a = x.T
        b = (x * w.unsqueeze(1)).T
        if pad:
            a = torch.nn.functional.pad(a, (0, pad))
            b = torch.nn.functional.pad(b, (0, pad))
        a, b = a.contiguous(), b.contiguous()
        if precision == "tf32":
            _native.gemm_abt_tf32(a, b, acc)
        else:
            ah, al = _split_tf32(a)
            bh, bl = _split_tf32(b)
            _native.gemm_abt_tf32(ah, bh, acc)
            _native.gemm_abt_tf32(ah, bl, acc)
            _native.gemm_abt_tf32(al, bh, acc)
    _native.check_trace_errors()
    return acc, float(den.item())


# the reference's private name, for callers that import it directly
_accumulate_hessian = accumulate_hessian
