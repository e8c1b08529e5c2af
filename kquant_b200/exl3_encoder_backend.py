"""EXL3/QSRT offline encoder backend for B200 (drop-in for kquant's ``exl3_encoder_backend``).

This module exposes the plugin API that kquant's encoder wrapper calls
(``kquant/pack/qsrt_encoder.py:824-832`` and ``:1193``).  Names, arguments,
return values, in-place mutations of ``H_data`` / ``quant_args`` and error
types follow ``kquant/exl3_encoder_backend.py``; each function cites the
lines it mirrors.  It imports absolutely and needs no ExLlamaV3 checkout.
It can be passed as ``quantizer_module=`` or loaded by
``kquant_b200.exl3_loader.load_qsrt_encoder``.

The hot path is native sm_100a CUDA, reached through the C ABI of
``_kq_b200.so``:
  * tile quantization (tail-biting Viterbi) -> ``kq_viterbi_encode``;
  * codebook label tables -> ``kq_build_labels``;
  * trellis packing -> ``kq_pack_trellis``.
The dense linear algebra around it (Cholesky, block-LDL, the LDLQ feedback
products, Hadamard rotations and the proxy traces) runs as PyTorch/cuBLAS
FP32 calls on the same stream.  It matches the reference's FP32 maths.
There is no CPU path: every entry point requires a CUDA device.
"""

from __future__ import annotations

import math
import threading
from collections.abc import Mapping
from functools import lru_cache

import torch

from . import _native
from .codebooks import sqg_e4m3_bytes

had_k, had_n = 128, 128
codebook_scale = 1.24371088
codebook_mcg_mult = 0xCBAC1FED
codebook_mul1_mult = 0x83DCD12D

# --------------------------------------------------------------------------
# tile order
# --------------------------------------------------------------------------


def _tc_order() -> list[int]:
    """Row-major 16x16 index visited at each trellis position (EXL tensor-core order).

    Position 8*t + s (t = MMA thread, s = fragment slot) holds row
    r = 2*(t%4) + (s&1) + 8*((s>>1)&1), column c = t//4 + 8*(s>>2)
    (kquant/exl3_encoder_backend.py:27-50, kquant/exl3_reference.py:89-108).
    """
    order = []
    for t in range(32):
        for s in range(8):
            r = 2 * (t % 4) + (s & 1) + 8 * ((s >> 1) & 1)
            c = t // 4 + 8 * (s >> 2)
            order.append(16 * r + c)
    return order


@lru_cache
def tensor_core_perm(device):
    return torch.tensor(_tc_order(), dtype=torch.int, device=device)


@lru_cache
def tensor_core_perm_i(device):
    return torch.argsort(tensor_core_perm(device))


# --------------------------------------------------------------------------
# tile quantizer (kquant/exl3_encoder_backend.py:81-111 with the SQG hook of
# kquant/sqg_quantizer.py:59-164 built in)
# --------------------------------------------------------------------------

_label_cache: dict = {}
_label_lock = threading.Lock()


def _labels_for(device: torch.device, bits: int, kind: int, lut: torch.Tensor | None) -> torch.Tensor:
    """Binary16 label table for (codebook, K) on ``device``; cached per source LUT object."""
    if kind == _native.KQ_CB_SQG:
        key = (str(device), bits, kind, lut.data_ptr() if lut.is_cuda else id(lut))
    else:
        key = (str(device), bits, kind, None)
    with _label_lock:
        hit = _label_cache.get(key)
        if hit is not None and (kind != _native.KQ_CB_SQG or hit[0] is lut):
            return hit[1]
    dev_lut = None
    if kind == _native.KQ_CB_SQG:
        dev_lut = lut.to(device=device, dtype=torch.uint8).contiguous()
        if dev_lut.numel() != 65536:
            raise ValueError("codebook must contain 65,536 uint8 E4M3 values")
    labels = _native.build_labels(kind, dev_lut, device)
    with _label_lock:
        _label_cache[key] = (lut, labels)
    return labels


def _tile_codebook(quant_args: dict, bits: int) -> tuple[int, torch.Tensor | None]:
    """Codebook selection of one quantize_tiles call (kquant/sqg_quantizer.py:78-129)."""
    codebook = quant_args.get("sqg_e4m3_lut")
    rate_codebooks = quant_args.get("sqg_e4m3_luts_by_bits")
    mode = quant_args.get("sqg_e4m3_mode")
    if codebook is None and rate_codebooks is None and mode is None:
        if "mcg" in quant_args:
            return _native.KQ_CB_MCG, None
        if "mul1" in quant_args:
            return _native.KQ_CB_MUL1, None
        return _native.KQ_CB_3INST, None
    if rate_codebooks is not None:
        if codebook is not None or mode is not None:
            raise ValueError("rate-specific SQG LUTs cannot be combined with another SQG law")
        if not isinstance(rate_codebooks, Mapping):
            raise TypeError("sqg_e4m3_luts_by_bits must be a mapping")
        if set(rate_codebooks) - {2, 3, 4}:
            raise ValueError("rate-specific SQG LUT keys must be K2, K3, or K4")
        try:
            codebook = rate_codebooks[bits]
        except KeyError as exc:
            raise ValueError(f"missing rate-specific SQG K{bits} LUT") from exc
        if codebook is None:
            return _native.KQ_CB_MCG, None
        return _native.KQ_CB_SQG, codebook
    if codebook is None:
        if mode != "normal":
            raise ValueError("the supported R44 mode is 'normal'")
        return _native.KQ_CB_SQG, sqg_e4m3_bytes(bits, mode)
    return _native.KQ_CB_SQG, codebook


def quantize_tiles(tiles: torch.Tensor, quant_args: dict):
    """Quantize [N, 256] fp32 tiles (tensor-core order) on their CUDA device.

    Returns (reconstructed fp32 tiles, int16 16-bit states).  Mirrors
    kquant/exl3_encoder_backend.py:81-111 as patched by
    kquant/sqg_quantizer.py:59-164: SQG LUTs (``sqg_e4m3_lut``,
    ``sqg_e4m3_luts_by_bits`` with ``None`` selecting MCG,
    ``sqg_e4m3_mode='normal'``), else the procedural MCG / MUL1 codebooks
    (key presence of ``mcg`` / ``mul1``), else 3INST.
    """
    if len(quant_args.get("devices", [None])) > 1 and any(
        k in quant_args for k in ("sqg_e4m3_lut", "sqg_e4m3_luts_by_bits", "sqg_e4m3_mode")
    ):
        raise ValueError("the SQG validation hook currently requires one CUDA device")
    tiles = tiles.contiguous()
    if tiles.dtype != torch.float32 or tiles.ndim != 2 or tiles.shape[1] != 256:
        raise ValueError("SQG tiles must be contiguous FP32 [N, 256]")
    if not tiles.is_cuda:
        raise ValueError("quantize_tiles requires CUDA tiles (kquant_b200 has no CPU path)")
    bits = int(quant_args["K"])
    if bits not in (2, 3, 4):
        raise ValueError("the trellis kernel supports K2--K4")
    kind, lut = _tile_codebook(quant_args, bits)
    labels = _labels_for(tiles.device, bits, kind, lut)
    ctx = int(quant_args.get("tailbite_context", 128))
    if not 1 <= ctx <= 128:
        raise ValueError("tailbite_context must be in 1..128")
    return _native.viterbi_encode(tiles, bits, labels, ctx)


@lru_cache
def get_quant_stream(device):
    return torch.cuda.Stream(device=device)


def _split_sizes(total: int, devices, ratios) -> list[int]:
    if ratios:
        s = sum(ratios)
        sizes = [round(total * r / s / 16) * 16 for r in ratios]
        sizes[-1] += total - sum(sizes)
    else:
        sizes = [total // len(devices)] * len(devices)
        sizes[-1] += total - sum(sizes)
    for i in range(len(sizes) - 2, -1, -1):
        if sizes[i + 1] < 0:
            sizes[i] += sizes[i + 1]
            sizes[i + 1] = 0
    return sizes


def quantize_tiles_multigpu(tiles, quant_args: dict):
    """Split one tile batch across ``quant_args['devices']`` and gather on the first.

    Mirrors kquant/exl3_encoder_backend.py:131-228.  Slices move device to
    device (NVLink peer copies) rather than through pinned host memory.
    """
    devices = quant_args["devices"]
    if len(devices) == 1:
        return quantize_tiles(tiles, quant_args)
    tiles = tiles.contiguous()
    sizes = _split_sizes(tiles.shape[0], devices, quant_args.get("device_ratios"))
    home = torch.device(devices[0])
    q = torch.empty_like(tiles)
    idx = torch.empty((tiles.shape[0], 256), dtype=torch.int16, device=home)
    local = dict(quant_args)
    local["devices"] = [devices[0]]
    ready = torch.cuda.current_stream(home).record_event()
    begin = 0
    done = []
    for size, dev in zip(sizes, devices):
        dev = torch.device(dev)
        if size > 0:
            stream = get_quant_stream(dev)
            stream.wait_event(ready)
            with torch.cuda.device(dev), torch.cuda.stream(stream):
                part = tiles[begin:begin + size].to(dev, non_blocking=True)
                part_q, part_i = quantize_tiles(part, local)
                q[begin:begin + size].copy_(part_q, non_blocking=True)
                idx[begin:begin + size].copy_(part_i, non_blocking=True)
                done.append(stream.record_event())
        begin += size
    for ev in done:
        torch.cuda.current_stream(home).wait_event(ev)
    return q, idx


def quantize_tiles_multigpu_sync(tiles, quant_args: dict):
    """Synchronous variant (kquant/exl3_encoder_backend.py:231-265)."""
    out = quantize_tiles_multigpu(tiles, quant_args)
    for dev in quant_args["devices"]:
        torch.cuda.synchronize(dev)
    return out


# --------------------------------------------------------------------------
# Hadamard rotations (Sylvester order, scaled 1/sqrt(128); the decoder's
# contract in kquant/exl3_reference.py:195-230)
# --------------------------------------------------------------------------


@lru_cache
def _hadamard(n: int, device, dtype) -> torch.Tensor:
    h = torch.ones((1, 1), dtype=torch.float64)
    while h.shape[0] < n:
        h = torch.cat((torch.cat((h, h), 1), torch.cat((h, -h), 1)), 0)
    return (h * (1.0 / math.sqrt(n))).to(device=device, dtype=dtype)


def preapply_had_l(x: torch.Tensor, had_dim):
    """Left block Hadamard on a copy (kquant/exl3_encoder_backend.py:268-275)."""
    k, n = x.shape
    dt = x.dtype
    xf = x.to(torch.float)
    out = torch.matmul(_hadamard(had_dim, xf.device, xf.dtype), xf.view(-1, had_dim, n)).view(k, n)
    return out.to(dt)


def preapply_had_r(x: torch.Tensor, had_dim):
    """Right block Hadamard on a copy (kquant/exl3_encoder_backend.py:278-285)."""
    k, n = x.shape
    dt = x.dtype
    xf = x.to(torch.float)
    out = torch.matmul(xf.view(k, -1, had_dim), _hadamard(had_dim, xf.device, xf.dtype)).view(k, n)
    return out.to(dt)


def blockwise_preapply_had_l_(x: torch.Tensor, had_dim):
    """In-place left block Hadamard (kquant/exl3_encoder_backend.py:288-299)."""
    k, n = x.shape
    assert k % had_dim == 0
    assert x.dtype == torch.float
    had = _hadamard(had_dim, x.device, x.dtype)
    x.copy_(torch.matmul(had, x.view(k // had_dim, had_dim, n)).view(k, n))


def blockwise_preapply_had_r_(x: torch.Tensor, had_dim):
    """In-place right block Hadamard (kquant/exl3_encoder_backend.py:302-313)."""
    k, n = x.shape
    assert n % had_dim == 0
    assert x.dtype == torch.float
    had = _hadamard(had_dim, x.device, x.dtype)
    x.copy_(torch.matmul(x.view(k, n // had_dim, had_dim), had).view(k, n))


# --------------------------------------------------------------------------
# Hessian factorisation (kquant/exl3_encoder_backend.py:316-386, 1586-1663)
# --------------------------------------------------------------------------


def _is_oom(e: Exception) -> bool:
    return e.__class__.__name__ == "OutOfMemoryError" or "out of memory" in str(e)


def block_ldl(H: torch.Tensor, b: int, quant_args: dict, verbose: bool):
    """Block LDL: H = L L^T with unit 16x16 diagonal blocks after normalisation.

    Returns (L on H's device, overwriting H's storage; H moved to CPU).
    Cholesky retries add 2*sigma_reg*mean(diag) up to ten times, then
    re-raise; an out-of-memory factorises on the CPU
    (kquant/exl3_encoder_backend.py:326-363).
    """
    n = H.shape[0]
    assert n % b == 0
    m = n // b
    retries = 0
    L = None
    while True:
        try:
            L = torch.linalg.cholesky(H)
            break
        except torch._C._LinAlgError:
            retries += 1
            if retries > 10:
                print(" ## Cholesky decomp. failed, number of retries exceeded")
                raise
            print(f" !! Cholesky decomp. failed, increasing diagonal damping, attempt {retries}/10")
            H.diagonal().add_(2.0 * quant_args.get("sigma_reg", 0.025) * H.diagonal().mean())
        except Exception as e:  # noqa: BLE001
            if not _is_oom(e):
                raise
            print(f" !! Out of memory on {H.device}, trying CPU fallback")
            L = torch.linalg.cholesky(H.cpu()).to(H.device)
            break
    H_cpu = H.cpu()
    H.copy_(L)
    del L
    L = H
    # Normalise every block column by the inverse of its diagonal block.
    Lb = L.view(n, m, b)
    DL = torch.diagonal(L.view(m, b, m, b), dim1=0, dim2=2).permute(2, 0, 1)
    DLi = torch.linalg.inv(DL)
    Lb.copy_(torch.einsum("nmb,mbc->nmc", Lb, DLi))
    L = L.view(n, n)
    blocks = L.view(m, b, m, b)
    eye = torch.eye(b, device=L.device, dtype=L.dtype)
    for i in range(m):
        blocks[i, :, i, :] = eye
    return L, H_cpu


finalize_capture_H_mutex = threading.Lock()


def finalize_capture_H(H_data: dict, quant_args: dict, verbose: bool):
    """Average, damp, sign-flip, Hadamard-rotate and block-LDL a captured H once.

    Returns (q_fallback, H, L, su, diag) and records them in ``H_data``
    (kquant/exl3_encoder_backend.py:1588-1663).
    """
    with finalize_capture_H_mutex:
        H = H_data["H"]
        if H.is_meta:
            k = H.shape[0]
            su = (torch.randn(k, device=H_data["device"]).sign() + 1e-5).sign().to(torch.float).unsqueeze(1)
            H_data.update(L=None, finalized=True, diag=None, q_fallback=True, su=su)
            return True, None, None, su, None
        if "H_swap_device" in H_data:
            H_data["H"] = H_data["H"].to(H_data.pop("H_swap_device"))
            H = H_data["H"]
        if H_data["finalized"]:
            return H_data["q_fallback"], H, H_data["L"], H_data["su"], H_data["diag"]
        count = H_data["count"]
        if count == 0:
            q_fallback = True
            diag_mean = 0.0
        else:
            H /= count
            diag_mean = torch.diag(H).mean()
            q_fallback = diag_mean.item() < 1e-20
        H.diagonal().add_(quant_args.get("sigma_reg", 0.025) * diag_mean)
        diag = H.diagonal().clone()
        if verbose:
            print(f"     - H min/max: {H.min().item():.6f}   {H.max().item():.6f}")
        k = H.shape[0]
        su = (torch.randn(k, device=H.device).sign() + 1e-5).sign().to(torch.float).unsqueeze(1)
        H_data["su"] = su
        H *= su.T
        blockwise_preapply_had_r_(H, had_k)
        H *= su
        blockwise_preapply_had_l_(H, had_k)
        if q_fallback:
            L = None
        else:
            L, H = block_ldl(H, 16, quant_args, verbose)
            idx = torch.arange(k)
            L[idx, idx] = 0
        H_data["L"] = L
        H = H.cpu()
        H_data["H"] = H
        H_data["finalized"] = True
        H_data["diag"] = diag
        H_data["q_fallback"] = q_fallback
        return q_fallback, H, L, su, diag
