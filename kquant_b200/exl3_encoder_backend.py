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


# Trellis rates the tile kernels cover: K2..K4 on the tile-pair kernel, K1 and
# K5..K8 on the wide-butterfly kernel.
TRELLIS_BITS = (1, 2, 3, 4, 5, 6, 7, 8)


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
    if bits not in TRELLIS_BITS:
        raise ValueError("the trellis kernels support K1--K8")
    kind, lut = _tile_codebook(quant_args, bits)
    labels = _labels_for(tiles.device, bits, kind, lut)
    ctx = int(quant_args.get("tailbite_context", 128))
    if not 1 <= ctx <= 128:
        raise ValueError("tailbite_context must be in 1..128")
    return _native.viterbi_encode(tiles, bits, labels, ctx)


def get_quant_stream(device):
    """The quantizer's stream of a device (one per device, however the device is named)."""
    d = torch.device(device)
    if d.index is None:
        d = torch.device(d.type, torch.cuda.current_device())
    return _quant_stream(d)


@lru_cache
def _quant_stream(device: torch.device):
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


def _host_copy(t: torch.Tensor) -> torch.Tensor:
    """Stream-ordered copy of a device tensor into pinned host memory.

    The copy completes in stream order; every public entry point of this module
    reads a proxy scalar back to the host before returning, which orders it.
    """
    if not t.is_cuda:
        return t
    out = torch.empty(t.shape, dtype=t.dtype, pin_memory=True)
    out.copy_(t, non_blocking=True)
    return out


def _device_H(H_data: dict, H: torch.Tensor, device) -> torch.Tensor:
    """The finalised H on ``device``: the resident copy kept by finalize_capture_H, else an upload."""
    dev_h = H_data.get("_H_device")
    if dev_h is not None and dev_h.device == torch.device(device):
        return dev_h
    return H.to(device)


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
    H_cpu = _host_copy(H)
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
    diag_blocks = torch.arange(m, device=L.device)
    blocks[diag_blocks, :, diag_blocks, :] = torch.eye(b, device=L.device, dtype=L.dtype)
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
            # Keep the rotated, damped H resident for the proxy (B200 has the
            # room); H_data["H"] still becomes the host copy, as the callers expect.
            H_data["_H_device"] = H.clone()
            L, H = block_ldl(H, 16, quant_args, verbose)
            idx = torch.arange(k)
            L[idx, idx] = 0
        H_data["L"] = L
        if H.is_cuda:
            H = _host_copy(H)
        H_data["H"] = H
        H_data["finalized"] = True
        H_data["diag"] = diag
        H_data["q_fallback"] = q_fallback
        return q_fallback, H, L, su, diag


# --------------------------------------------------------------------------
# LDLQ: one backward traversal engine behind every public variant
# --------------------------------------------------------------------------


def mixed_rate_spec(size_k: int, size_n: int, quant_args: dict):
    """Validate a K2/K3/K4 per-tile rate map (kquant/exl3_encoder_backend.py:508-536)."""
    rate_axis = quant_args.get("mixed_rate_axis")
    if rate_axis not in ("k", "n"):
        raise ValueError("mixed_rate_axis must be 'k' or 'n'")
    if size_k % 16 or size_n % 16:
        raise ValueError("mixed-rate LDLQ input must be 16x16 tile aligned")
    raw = quant_args.get("mixed_tile_bits")
    if raw is None:
        raise ValueError("mixed_tile_bits is required for mixed-rate LDLQ")
    tile_bits = tuple(raw)
    expected = size_k // 16 if rate_axis == "k" else size_n // 16
    if len(tile_bits) != expected:
        raise ValueError(f"mixed_tile_bits has {len(tile_bits)} entries; expected {expected}")
    if any(isinstance(b, bool) or not isinstance(b, int) or b not in (2, 3, 4) for b in tile_bits):
        raise ValueError("mixed-rate LDLQ supports only integer K2, K3, and K4")
    return rate_axis, tile_bits


def _baddbmm_ldlq(input, batch1, batch2, *, tf32, inplace=False):
    """One LDLQ feedback product at the requested FP32 policy (kquant/exl3_encoder_backend.py:725-742)."""
    previous = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = bool(tf32)
    try:
        if inplace:
            return input.baddbmm_(batch1, batch2)
        return torch.baddbmm(input, batch1, batch2)
    finally:
        torch.backends.cuda.matmul.allow_tf32 = previous


class _RatePlan:
    """Which K each tile of a 16-row LDLQ step uses, as launch groups.

    ``groups_for(step_tile)`` returns [(K, flat_tile_index or None)], where the
    flat index enumerates tiles member-major ([B, tiles_n] flattened) and
    ``None`` means all tiles.
    """

    def __init__(self, member_bits, rate_axis: str | None, batch: int, tiles_n: int, device):
        self.rate_axis = rate_axis
        self.uniform = None
        self._cache: dict = {}
        self.device = device
        self.tiles_n = tiles_n
        self.batch = batch
        if rate_axis is None:
            self.uniform = int(member_bits)
            return
        self.member_bits = member_bits
        if rate_axis == "n":
            flat = [b for bits in member_bits for b in bits]
            self._static = self._groups(flat)

    def _groups(self, flat_bits):
        widths = sorted(set(flat_bits))
        if len(widths) == 1:
            return [(widths[0], None)]
        t = torch.tensor(flat_bits, dtype=torch.int64)
        return [(w, torch.nonzero(t == w).flatten().to(self.device)) for w in widths]

    def groups_for(self, step_tile: int):
        if self.uniform is not None:
            return [(self.uniform, None)]
        if self.rate_axis == "n":
            return self._static
        key = tuple(bits[step_tile] for bits in self.member_bits)
        g = self._cache.get(key)
        if g is None:
            g = self._groups([b for b in key for _ in range(self.tiles_n)])
            self._cache[key] = g
        return g


def _quantize_step_tiles(tiles: torch.Tensor, plan: _RatePlan, step_tile: int, quant_args: dict):
    groups = plan.groups_for(step_tile)
    if len(groups) == 1:
        args = dict(quant_args)
        args["K"] = groups[0][0]
        return quantize_tiles_multigpu(tiles, args)
    q = torch.empty_like(tiles)
    idx = torch.empty((tiles.shape[0], 256), dtype=torch.int16, device=tiles.device)
    for bits, where in groups:
        args = dict(quant_args)
        args["K"] = bits
        gq, gi = quantize_tiles_multigpu(tiles.index_select(0, where), args)
        q.index_copy_(0, where, gq)
        idx.index_copy_(0, where, gi)
    return q, idx


def _drive(gen):
    while True:
        try:
            next(gen)
        except StopIteration as done:
            return done.value


def _ldlq_traverse(weights, Ls, quant_args, plan: _RatePlan, **kw):
    """Run :func:`_ldlq_traverse_steps` to completion; returns (What, enc, P)."""
    return _drive(_ldlq_traverse_steps(weights, Ls, quant_args, plan, **kw))


def _ldlq_traverse_steps(weights, Ls, quant_args, plan: _RatePlan, *, buffer_rows: int, tf32: bool,
                         process_begin: int = 0, process_end: int | None = None, state=None,
                         source_indices: torch.Tensor | None = None, pb=None):
    """Backward block-LDLQ over rows [process_begin, process_end) of a batch.

    A generator: it yields after enqueueing each 16-row step (so several
    independent traversals can be interleaved on their own streams) and
    returns (What, enc, P).

    weights [S, k, n] and Ls [S, k, k] are sources; members read source
    ``source_indices[b]`` (identity when None).  For every 16-row step
    r0:r1 inside a 128-row buffer [begin, end):

        comp  = P[r0:r1] + L[r1:end, r0:r1]^T (W - What)[r1:end]
        tiles = tensor-core-ordered 16x16 tiles of W[r0:r1] + comp
        What[r0:r1], enc[:, r0/16] = Viterbi(tiles)

    and after the buffer P[:begin] += L[begin:end, :begin]^T (W - What)[begin:end]
    (the dead-prefix trim of kquant/exl3_encoder_backend.py:968-989).
    Returns (What, enc, P).
    """
    S, size_k, size_n = weights.shape
    B = source_indices.shape[0] if source_indices is not None else S
    tiles_n = size_n // 16
    dev = weights.device
    if process_end is None:
        process_end = size_k
    if state is None:
        wq = weights.new_zeros((B, size_k, size_n))
        enc = torch.zeros((B, size_k // 16, tiles_n, 256), dtype=torch.int16, device=dev)
        P = weights.new_zeros((B, size_k, size_n))
    else:
        wq, enc, P = state
    perm = tensor_core_perm(dev)
    perm_i = tensor_core_perm_i(dev)

    def src(x, sl_rows, sl_cols=None):
        v = x[:, sl_rows] if sl_cols is None else x[:, sl_rows, sl_cols]
        return v if source_indices is None else v.index_select(0, source_indices)

    progress = 0
    fused = (state is None and source_indices is None and process_begin == 0 and process_end == size_k
             and plan.uniform in (2, 3, 4) and len(quant_args.get("devices", [dev])) == 1
             and weights.is_contiguous() and weights.dtype == torch.float32)
    if fused:
        # Fused steps: the Viterbi launch gathers W + comp into tiles and
        # scatters What, E = W - What and the states itself.
        bits = plan.uniform
        ctx = int(quant_args.get("tailbite_context", 128))
        if not 1 <= ctx <= 128:
            raise ValueError("tailbite_context must be in 1..128")
        kind, lut = _tile_codebook(quant_args, bits)
        labels = _labels_for(dev, bits, kind, lut)
        E = torch.empty_like(weights)
        for end in range(process_end, process_begin, -buffer_rows):
            begin = end - buffer_rows
            for local_end in range(buffer_rows, 0, -16):
                r0 = begin + local_end - 16
                r1 = r0 + 16
                comp = _baddbmm_ldlq(P[:, r0:r1], Ls[:, r1:end, r0:r1].transpose(1, 2), E[:, r1:end], tf32=tf32)
                _native.ldlq_step_encode(weights, comp.contiguous(), r0, bits, labels, ctx, wq, E, enc)
                if pb:
                    progress += 1
                    pb.update(progress)
                yield
            if begin:
                _baddbmm_ldlq(P[:, :begin], Ls[:, begin:end, :begin].transpose(1, 2), E[:, begin:end], tf32=tf32,
                              inplace=True)
        return wq, enc, P
    for end in range(process_end, process_begin, -buffer_rows):
        begin = end - buffer_rows
        for local_end in range(buffer_rows, 0, -16):
            r0 = begin + local_end - 16
            r1 = r0 + 16
            err = src(weights, slice(r1, end)) - wq[:, r1:end]
            ldl = src(Ls, slice(r1, end), slice(r0, r1))
            comp = _baddbmm_ldlq(P[:, r0:r1], ldl.transpose(1, 2), err, tf32=tf32)
            rows = src(weights, slice(r0, r1)) + comp
            tiles = rows.reshape(B, 16, tiles_n, 16).permute(0, 2, 1, 3).reshape(B * tiles_n, 256)
            tiles = tiles[:, perm]
            q, idx = _quantize_step_tiles(tiles, plan, r0 // 16, quant_args)
            enc[:, r0 // 16] = idx.reshape(B, tiles_n, 256)
            q = q[:, perm_i]
            wq[:, r0:r1] = q.reshape(B, tiles_n, 16, 16).permute(0, 2, 1, 3).reshape(B, 16, size_n)
            if pb:
                progress += 1
                pb.update(progress)
            yield
        if begin:
            err = src(weights, slice(begin, end)) - wq[:, begin:end]
            ldl = src(Ls, slice(begin, end), slice(0, begin))
            _baddbmm_ldlq(P[:, :begin], ldl.transpose(1, 2), err, tf32=tf32, inplace=True)
    return wq, enc, P


def _sync(devices):
    """Host waits for the calling stream and the quantizer stream of each device.

    The reference synchronises whole devices (kquant/exl3_encoder_backend.py:418-420);
    this build only orders the two streams its work runs on, so unrelated work on
    other streams of the same device (data generation, copies) keeps overlapping.
    """
    for d in devices:
        torch.cuda.current_stream(d).synchronize()
        get_quant_stream(d).synchronize()


def _buffer_rows(quant_args: dict, size_k: int) -> int:
    rows = max(quant_args.get("buf_size_k", 128), 16)
    if rows % 16 or size_k % rows:
        raise ValueError("LDLQ buffer must tile the EXL K dimension")
    return rows


def _engine_ldlq(W, Ls, quant_args, rate=None):
    """W [B, k, n] (contiguous) and Ls [B, k, k] on the chain engine; returns (What, enc)."""
    B, size_k, size_n = W.shape
    wq = torch.empty_like(W)
    enc = torch.empty((B, size_k // 16, size_n // 16, 256), dtype=torch.int16, device=W.device)
    members = [_ChainMember(W[b], Ls[b], wq[b], enc[b], quant_args, rate=rate) for b in range(B)]
    _chain_traverse(members, W.device)
    return wq, enc


def ldlq(weight: torch.Tensor, L: torch.Tensor, quant_args: dict, pb=None):
    """Block LDLQ of one matrix at uniform K (kquant/exl3_encoder_backend.py:389-505).

    weight [k, n] fp32, L [k, k] block-LDL factor.  Returns (What [k, n],
    encoded int16 [k/16, n/16, 256]).
    """
    devices = quant_args["devices"]
    _sync(devices)
    size_k, size_n = weight.shape
    assert size_k % 16 == 0 and size_n % 128 == 0
    assert L.device == torch.device(devices[0])
    rows = _buffer_rows(quant_args, size_k)
    with torch.cuda.stream(get_quant_stream(devices[0])):
        w = weight.to(L.device)
        if len(devices) == 1 and pb is None:
            wq, enc = _engine_ldlq(w.contiguous().unsqueeze(0), L.unsqueeze(0), quant_args)
        else:
            plan = _RatePlan(int(quant_args["K"]), None, 1, size_n // 16, L.device)
            wq, enc, _ = _ldlq_traverse(w.unsqueeze(0), L.unsqueeze(0), quant_args, plan, buffer_rows=rows,
                                        tf32=bool(quant_args.get("ldlq_tf32", False)), pb=pb)
    _sync(devices)
    return wq[0].to(weight.device), enc[0].to(weight.device)


def ldlq_mixed(weight: torch.Tensor, L: torch.Tensor, quant_args: dict, pb=None):
    """Dense-H LDLQ with K chosen per tile on one axis (kquant/exl3_encoder_backend.py:539-665)."""
    devices = quant_args["devices"]
    _sync(devices)
    if L.device != torch.device(devices[0]):
        raise ValueError("mixed-rate LDLQ decomposition is on the wrong device")
    size_k, size_n = weight.shape
    axis, bits = mixed_rate_spec(size_k, size_n, quant_args)
    rows = max(quant_args.get("buf_size_k", 128), 16)
    if rows % 16 or size_k % rows:
        raise ValueError("mixed-rate LDLQ buffer must tile the EXL K dimension")
    with torch.cuda.stream(get_quant_stream(devices[0])):
        w = weight.to(L.device)
        if len(devices) == 1 and pb is None:
            wq, enc = _engine_ldlq(w.contiguous().unsqueeze(0), L.unsqueeze(0), quant_args, rate=(axis, bits))
        else:
            plan = _RatePlan([bits], axis, 1, size_n // 16, L.device)
            wq, enc, _ = _ldlq_traverse(w.unsqueeze(0), L.unsqueeze(0), quant_args, plan, buffer_rows=rows,
                                        tf32=bool(quant_args.get("ldlq_tf32", False)), pb=pb)
    _sync(devices)
    return wq[0].to(weight.device), enc[0].to(weight.device)


def ldlq_batched(weights: torch.Tensor, Ls: torch.Tensor, quant_args: dict, pb=None):
    """Same-shape tensors with per-tensor L, one tile launch per step (kquant/exl3_encoder_backend.py:1495-1583)."""
    devices = quant_args["devices"]
    _sync(devices)
    B, size_k, size_n = weights.shape
    assert weights.device == torch.device(devices[0]) and Ls.device == weights.device
    assert Ls.shape == (B, size_k, size_k)
    assert size_k % 16 == 0 and size_n % 128 == 0
    rows = _buffer_rows(quant_args, size_k)
    with torch.cuda.stream(get_quant_stream(devices[0])):
        if len(devices) == 1 and pb is None:
            wq, enc = _engine_ldlq(weights.contiguous(), Ls, quant_args)
        else:
            plan = _RatePlan(int(quant_args["K"]), None, B, size_n // 16, weights.device)
            wq, enc, _ = _ldlq_traverse(weights, Ls, quant_args, plan, buffer_rows=rows,
                                        tf32=bool(quant_args.get("ldlq_tf32", False)), pb=pb)
    _sync(devices)
    return wq, enc


def _make_mixed_ldlq_grouping(position_bits, device):
    """Gather plan (order, inverse, slices) of one step (kquant/exl3_encoder_backend.py:668-698)."""
    values = tuple(int(v) for v in position_bits)
    widths = tuple(sorted(set(values)))
    if len(widths) == 1:
        return None, None, ((widths[0], 0, len(values)),)
    order = tuple(p for w in widths for p, v in enumerate(values) if v == w)
    inverse = [0] * len(order)
    for grouped, original in enumerate(order):
        inverse[original] = grouped
    slices, begin = [], 0
    for w in widths:
        end = begin + values.count(w)
        slices.append((w, begin, end))
        begin = end
    return (torch.tensor(order, dtype=torch.int64, device=device),
            torch.tensor(inverse, dtype=torch.int64, device=device), tuple(slices))


def _prepare_mixed_ldlq_groupings(rate_axis, tile_bits, tiles_k, tiles_n, device):
    """Per-step gather plans for a batch of rate maps (kquant/exl3_encoder_backend.py:701-722)."""
    if rate_axis == "n":
        return _make_mixed_ldlq_grouping((v for m in tile_bits for v in m), device), None
    cache, plans = {}, []
    for t in range(tiles_k):
        key = tuple(bits[t] for bits in tile_bits)
        if key not in cache:
            cache[key] = _make_mixed_ldlq_grouping((w for w in key for _ in range(tiles_n)), device)
        plans.append(cache[key])
    return None, plans


def ldlq_mixed_batched(weights, Ls, quant_args_list, pb=None, *, synchronize=True, prepared_groupings=None,
                       process_begin=0, process_end=None, initial_weights_q=None, initial_encoded_q=None,
                       initial_product_cache=None, return_product_cache=False, source_indices=None):
    """Batch independent heterogeneous-rate LDLQ traversals (kquant/exl3_encoder_backend.py:745-996).

    Members may carry different K2/K3/K4 maps on one shared rate axis; a
    buffer-aligned [process_begin, process_end) interval with continuation
    state supports exact common-prefix reuse; ``source_indices`` lets members
    share a source weight/L without copying it.
    """
    if weights.ndim != 3 or Ls.ndim != 3:
        raise ValueError("batched mixed LDLQ expects rank-three weights and Ls")
    S, size_k, size_n = weights.shape
    B = len(quant_args_list)
    if S <= 0 or B <= 0 or Ls.shape != (S, size_k, size_k):
        raise ValueError("batched mixed LDLQ weight/L shapes do not agree")
    if weights.dtype != torch.float or Ls.dtype != torch.float:
        raise TypeError("batched mixed LDLQ weights and Ls must be float32")
    if weights.device != Ls.device or weights.device.type != "cuda":
        raise ValueError("batched mixed LDLQ inputs must share one CUDA device")
    if source_indices is None:
        if S != B:
            raise ValueError("batched mixed LDLQ needs one source per member without source_indices")
    else:
        if source_indices.shape != (B,) or source_indices.dtype != torch.long or source_indices.device != weights.device:
            raise ValueError("mixed LDLQ source_indices must be device-local int64 [B]")
        if bool(torch.any(source_indices < 0)) or bool(torch.any(source_indices >= S)):
            raise ValueError("mixed LDLQ source_indices are out of range")
    devices = quant_args_list[0]["devices"]
    if weights.device != torch.device(devices[0]):
        raise ValueError("batched mixed LDLQ inputs are on the wrong device")
    if any(a.get("devices") != devices for a in quant_args_list):
        raise ValueError("batched mixed LDLQ members must share devices")
    tf32 = bool(quant_args_list[0].get("ldlq_tf32", False))
    if any(bool(a.get("ldlq_tf32", False)) != tf32 for a in quant_args_list):
        raise ValueError("batched mixed LDLQ members must share TF32 policy")
    if synchronize:
        _sync(devices)
    normalized = [mixed_rate_spec(size_k, size_n, a) for a in quant_args_list]
    axis = normalized[0][0]
    if any(ax != axis for ax, _ in normalized):
        raise ValueError("batched mixed LDLQ members must share one rate axis")
    rows = max(quant_args_list[0].get("buf_size_k", 128), 16)
    if any(max(a.get("buf_size_k", 128), 16) != rows for a in quant_args_list):
        raise ValueError("batched mixed LDLQ members must share one buffer size")
    if rows % 16 or size_k % rows:
        raise ValueError("batched mixed LDLQ buffer must tile the EXL K dimension")
    if process_end is None:
        process_end = size_k
    if (isinstance(process_begin, bool) or isinstance(process_end, bool)
            or not isinstance(process_begin, int) or not isinstance(process_end, int)
            or not 0 <= process_begin < process_end <= size_k
            or process_begin % rows or process_end % rows):
        raise ValueError("mixed LDLQ process interval must be buffer-aligned")
    init = (initial_weights_q, initial_encoded_q, initial_product_cache)
    if any(v is not None for v in init) and not all(v is not None for v in init):
        raise ValueError("mixed LDLQ continuation requires all three state tensors")
    if initial_weights_q is None and process_end != size_k:
        raise ValueError("a lower mixed LDLQ interval requires continuation state")
    state = None
    if initial_weights_q is not None:
        ew, ee = (B, size_k, size_n), (B, size_k // 16, size_n // 16, 256)
        if (initial_weights_q.shape != ew or initial_weights_q.dtype != weights.dtype
                or initial_weights_q.device != weights.device
                or initial_product_cache.shape != ew or initial_product_cache.dtype != weights.dtype
                or initial_product_cache.device != weights.device
                or initial_encoded_q.shape != ee or initial_encoded_q.dtype != torch.int16
                or initial_encoded_q.device != weights.device):
            raise ValueError("mixed LDLQ continuation state has invalid shape or type")
        state = (initial_weights_q, initial_encoded_q, initial_product_cache)
    del prepared_groupings  # the rate plan below is built once per call and cached per step key
    if (state is None and source_indices is None and process_begin == 0 and process_end == size_k
            and len(devices) == 1):
        wq = torch.empty((B, size_k, size_n), dtype=weights.dtype, device=weights.device)
        enc = torch.empty((B, size_k // 16, size_n // 16, 256), dtype=torch.int16, device=weights.device)
        P = torch.zeros_like(wq)
        with torch.cuda.stream(get_quant_stream(devices[0])):
            members = [_ChainMember(weights[b], Ls[b], wq[b], enc[b], quant_args_list[b], rate=(axis, bits),
                                    P=P[b]) for b, (_, bits) in enumerate(normalized)]
            _chain_traverse(members, weights.device)
        if synchronize:
            _sync(devices)
        return (wq, enc, P) if return_product_cache else (wq, enc)
    plan = _RatePlan([bits for _, bits in normalized], axis, B, size_n // 16, weights.device)
    with torch.cuda.stream(get_quant_stream(devices[0])):
        wq, enc, P = _ldlq_traverse(weights, Ls, quant_args_list[0], plan, buffer_rows=rows, tf32=tf32,
                                    process_begin=process_begin, process_end=process_end, state=state,
                                    source_indices=source_indices, pb=pb)
    if synchronize:
        _sync(devices)
    if return_product_cache:
        return wq, enc, P
    return wq, enc


def ldlq_mixed_n_candidates_reuse(weights: torch.Tensor, Ls: torch.Tensor, quant_args_groups):
    """Encode output-axis candidates once per changed tile (kquant/exl3_encoder_backend.py:999-1160).

    LDLQ couples rows, not output columns.  Candidates that differ only in the
    n-axis rate map share every unchanged output tile.  The all-K3 base is
    encoded once, the union of each source's K2 / K4 replacement columns once,
    and the candidates are assembled from those.  Output is source-major.
    """
    if weights.ndim != 3 or Ls.ndim != 3:
        raise ValueError("output-axis reuse expects rank-three weights and Ls")
    S, size_k, size_n = weights.shape
    if S <= 0 or Ls.shape != (S, size_k, size_k):
        raise ValueError("output-axis reuse weight/L shapes do not agree")
    if len(quant_args_groups) != S or any(not g for g in quant_args_groups):
        raise ValueError("output-axis reuse needs candidates for every source")
    maps = []
    for group in quant_args_groups:
        norm = [mixed_rate_spec(size_k, size_n, a) for a in group]
        if any(ax != "n" for ax, _ in norm):
            raise ValueError("output-axis reuse supports only mixed_rate_axis='n'")
        if norm[0][1] != (3,) * (size_n // 16):
            raise ValueError("output-axis reuse requires an all-K3 first candidate")
        maps.append([bits for _, bits in norm])
    dev = weights.device
    specs = []
    for s, cand in enumerate(maps):
        width = {}
        for bits in cand[1:]:
            for tile, w in enumerate(bits):
                if w == 3:
                    continue
                if width.setdefault(tile, w) != w:
                    raise ValueError("one output tile uses multiple non-K3 widths across candidates")
        for w in (2, 4):
            pos = tuple(t for t, x in width.items() if x == w)
            if pos:
                specs.append((s, w, pos))

    def cols(tiles):
        return torch.tensor([c for t in tiles for c in range(16 * t, 16 * t + 16)], dtype=torch.int64, device=dev)

    # The all-K3 base of every source and the K2 / K4 replacement columns are
    # independent LDLQ problems (columns do not couple): one chain-engine run.
    devices = quant_args_groups[0][0]["devices"]
    _sync(devices)
    base_wq = torch.empty_like(weights)
    base_enc = torch.empty((S, size_k // 16, size_n // 16, 256), dtype=torch.int16, device=dev)
    overrides = {}
    with torch.cuda.stream(get_quant_stream(devices[0])):
        members = [_ChainMember(weights[s], Ls[s], base_wq[s], base_enc[s], quant_args_groups[s][0], rate=3)
                   for s in range(S)]
        for s, w, pos in specs:
            sub = weights[s].index_select(1, cols(pos)).contiguous()
            owq = torch.empty_like(sub)
            oenc = torch.empty((size_k // 16, len(pos), 256), dtype=torch.int16, device=dev)
            members.append(_ChainMember(sub, Ls[s], owq, oenc, quant_args_groups[s][0], rate=w))
            overrides[(s, w)] = (pos, owq, oenc)
        _chain_traverse(members, dev)
    _sync(devices)

    out_wq, out_enc = [], []
    for s, cand in enumerate(maps):
        for c, bits in enumerate(cand):
            if c == 0:
                out_wq.append(base_wq[s])
                out_enc.append(base_enc[s])
                continue
            wq = base_wq[s].clone()
            enc = base_enc[s].clone()
            for w in (2, 4):
                target = tuple(t for t, x in enumerate(bits) if x == w)
                if not target:
                    continue
                pos, rwq, renc = overrides[(s, w)]
                local = {t: i for i, t in enumerate(pos)}
                lt = tuple(local[t] for t in target)
                wq.index_copy_(1, cols(target), rwq.index_select(1, cols(lt)))
                enc.index_copy_(1, torch.tensor(target, dtype=torch.int64, device=dev),
                                renc.index_select(1, torch.tensor(lt, dtype=torch.int64, device=dev)))
            out_wq.append(wq)
            out_enc.append(enc)
    return torch.stack(out_wq), torch.stack(out_enc)


def ldlq_mixed_k_candidates_prefix_reuse(weights: torch.Tensor, Ls: torch.Tensor, quant_args_groups):
    """Input-axis candidates through a shared backward prefix (kquant/exl3_encoder_backend.py:1163-1345).

    The common buffer-aligned suffix of each source's rate maps is traversed
    once; the remaining rows proceed as a trie of live LDLQ states, forking
    only where candidate maps diverge.  Results equal independent traversals.
    """
    if weights.ndim != 3 or Ls.ndim != 3:
        raise ValueError("input-axis prefix reuse expects rank-three weights and Ls")
    S, size_k, size_n = weights.shape
    if S <= 0 or Ls.shape != (S, size_k, size_k):
        raise ValueError("input-axis prefix reuse weight/L shapes do not agree")
    if len(quant_args_groups) != S or any(not g for g in quant_args_groups):
        raise ValueError("input-axis prefix reuse needs candidates for every source")
    if not any(len(g) > 1 for g in quant_args_groups):
        raise ValueError("input-axis prefix reuse needs at least one multi-candidate source")
    maps = []
    for group in quant_args_groups:
        norm = [mixed_rate_spec(size_k, size_n, a) for a in group]
        if any(ax != "k" for ax, _ in norm):
            raise ValueError("input-axis prefix reuse supports only mixed_rate_axis='k'")
        maps.append([bits for _, bits in norm])
    rows = max(quant_args_groups[0][0].get("buf_size_k", 128), 16)
    if any(max(a.get("buf_size_k", 128), 16) != rows for g in quant_args_groups for a in g):
        raise ValueError("input-axis prefix reuse requires one LDLQ buffer size")
    if rows % 16 or size_k % rows:
        raise ValueError("input-axis prefix reuse buffer must tile the EXL K dimension")
    flat = [(s, c) for s, g in enumerate(quant_args_groups) for c in range(len(g))]
    dev = weights.device
    devices = quant_args_groups[0][0]["devices"]
    # Trie of LDLQ states as chain-engine members: a node holds the candidates
    # whose maps agree on every buffer traversed so far; when one of its chains
    # reaches a buffer where they differ, the node splits.  The part holding
    # the node's representative candidate keeps its arrays; every other part
    # gets fresh ones, filled column slice by column slice as the node's
    # chains arrive, and continues from the same row.
    node = {}                                   # id(member) -> [source, candidates, representative]

    def new_member(s, cands, like=None):
        qa = quant_args_groups[s][cands[0]]
        rate = ("k", maps[s][cands[0]])
        if like is None:
            m = _ChainMember(weights[s], Ls[s], torch.empty((size_k, size_n), dtype=weights.dtype, device=dev),
                             torch.empty((size_k // 16, size_n // 16, 256), dtype=torch.int16, device=dev), qa,
                             rate=rate)
        else:
            m = _ChainMember(like.W, like.L, torch.empty_like(like.wq), torch.empty_like(like.enc), qa, rate=rate,
                             P=torch.empty_like(like.P), E=torch.empty_like(like.E))
        node[id(m)] = [s, tuple(cands), cands[0]]
        return m

    def partition(s, cands, begin, end):
        parts: dict = {}
        for c in cands:
            parts.setdefault(maps[s][c][begin // 16:end // 16], []).append(c)
        return list(parts.values())

    forks: dict = {}

    def on_buffer(chain):
        m = chain.m
        r0, end = chain.steps[chain.pos]
        key = (id(m), end)
        if key not in forks:
            s, cands, rep = node[id(m)]
            parts = partition(s, cands, end - rows, end)
            if len(parts) == 1:
                forks[key] = None
            else:
                children = []
                for part in parts:
                    if rep in part:
                        node[id(m)][1] = tuple(part)
                    else:
                        children.append(new_member(s, part, like=m))
                forks[key] = children
        children = forks[key]
        if not children:
            return None
        cs = slice(16 * chain.tile_col0, 16 * (chain.tile_col0 + chain.n_tiles))
        ts = slice(chain.tile_col0, chain.tile_col0 + chain.n_tiles)
        out = [chain]
        for child in children:
            child.wq[:, cs] = m.wq[:, cs]
            child.enc[:, ts] = m.enc[:, ts]
            child.P[:, cs] = m.P[:, cs]
            child.E[:, cs] = m.E[:, cs]
            out.append(_Chain(child, chain.tile_col0, chain.n_tiles, steps=chain.steps, pos=chain.pos))
        return out

    _sync(devices)
    with torch.cuda.stream(get_quant_stream(devices[0])):
        roots = [new_member(s, part) for s, g in enumerate(quant_args_groups)
                 for part in partition(s, tuple(range(len(g))), size_k - rows, size_k)]
        _chain_traverse(roots, dev, on_buffer=on_buffer)
        members = {id(m): m for m in roots}
        for children in forks.values():
            for m in children or ():
                members[id(m)] = m
        where = {}
        for mid, (s, cands, _) in node.items():
            for c in cands:
                where[(s, c)] = members[mid]
        if set(where) != set(flat):
            raise AssertionError("input-axis prefix trie lost a rate candidate")
        wq = torch.stack([where[f].wq for f in flat])
        enc = torch.stack([where[f].enc for f in flat])
    _sync(devices)
    return wq, enc


def fallback_quant(weight: torch.Tensor, q_device, quant_args: dict, pb=None):
    """Tile quantization without feedback, for an unusable H (kquant/exl3_encoder_backend.py:1348-1463).

    Returns (What, encoded, mse).
    """
    devices = quant_args["devices"]
    _sync(devices)
    size_k, size_n = weight.shape
    assert size_k % 16 == 0 and size_n % 128 == 0
    assert weight.device == torch.device(devices[0])
    tn = size_n // 16
    dev = weight.device
    with torch.cuda.stream(get_quant_stream(devices[0])):
        tiles = weight.reshape(size_k // 16, 16, tn, 16).permute(0, 2, 1, 3).reshape(-1, 256)
        tiles = tiles[:, tensor_core_perm(dev)]
        q, idx = quantize_tiles_multigpu(tiles, quant_args)
        q = q[:, tensor_core_perm_i(dev)]
        wq = q.reshape(size_k // 16, tn, 16, 16).permute(0, 2, 1, 3).reshape(size_k, size_n)
        enc = idx.reshape(size_k // 16, tn, 256)
        mse = (torch.sum((weight.float() - wq.float()).pow(2), dtype=torch.float64) / weight.numel()).item()
        if pb:
            pb.update(size_k // 16)
    _sync(devices)
    return wq, enc, mse


# --------------------------------------------------------------------------
# proxy error, packing
# --------------------------------------------------------------------------


# The proxy traces run as one fused tcgen05 GEMM + trace kernel (TF32 operands,
# fp32 accumulation, fp64 reduction) when the shapes tile; the proxy is a
# 1%-tolerance measurement, so TF32 operands are within its contract.
PROXY_ON_TENSOR_CORES = True


def block_trace_parts(A, B, block_size=1024):
    """Device terms of trace(A^T B A) (kquant/exl3_encoder_backend.py:1466-1479).

    On the tensor-core path the result is a single term:
    trace(A^T B A) = sum((A^T B) * A^T), computed by kq_trace_abt with
    operands A^T [n, k] and B^T [k, k] (no symmetry of B assumed).  Otherwise
    the column blocks of B are reduced with cuBLAS FP32.
    """
    k, n = A.shape
    if (PROXY_ON_TENSOR_CORES and A.is_cuda and B.is_cuda and A.dtype == torch.float32 and B.dtype == torch.float32
            and B.shape == (k, k) and _native.trace_abt_supported(n, k, k)):
        At = A.T.contiguous()
        return _native.trace_abt(At, B.T.contiguous(), At).reshape(1)
    parts = []
    for j in range(0, B.shape[1], block_size):
        e = min(j + block_size, B.shape[1])
        parts.append(torch.sum((A.T @ B[:, j:e]) * A[j:e, :].T))
    return torch.stack(parts)


def block_trace(A, B, block_size=1024):
    """trace(A^T B A) summed in fp64 on the host (kquant/exl3_encoder_backend.py:1482-1492)."""
    total = 0.0
    for p in block_trace_parts(A, B, block_size).cpu():
        total += p.item()
    _native.check_trace_errors()
    return total


def pack_trellis(encoded: torch.Tensor, quant_args: dict) -> torch.Tensor:
    """[tk, tn, 256] int16 states -> [tk, tn, 16K] int16 words (kquant/exl3_encoder_backend.py:1666-1677)."""
    K = quant_args["K"]
    assert encoded.ndim == 3 and encoded.shape[2] == 256
    assert encoded.dtype == torch.int16
    return _native.pack_trellis(encoded.contiguous(), int(K))


# --------------------------------------------------------------------------
# global scale search (kquant/exl3_encoder_backend.py:1688-1808)
# --------------------------------------------------------------------------


def sample_scale_tiles(weight_r: torch.Tensor, width: int = 3) -> torch.Tensor:
    """Wrapped-diagonal tiles plus the highest- and lowest-RMS tiles, tensor-core ordered."""
    dev = weight_r.device
    tk, tn = weight_r.shape[0] // 16, weight_r.shape[1] // 16
    w4 = weight_r.view(tk, 16, tn, 16)
    diag = max(tk, tn)
    ii = torch.arange(diag, device=dev).repeat_interleave(width)
    ww = torch.arange(width, device=dev).repeat(diag)
    kk, nn = ii % tk, (ii + ww) % tn
    num_x = max(8, (diag * width) // 16)
    ms = w4.square().mean(dim=(1, 3)).flatten()
    num_x = min(num_x, (ms.shape[0] + 1) // 2)
    ext = torch.cat((torch.topk(ms, num_x).indices, torch.topk(ms, num_x, largest=False).indices))
    tiles = w4[torch.cat((kk, ext // tn)), :, torch.cat((nn, ext % tn)), :].reshape(-1, 256)
    return tiles[:, tensor_core_perm(dev)].contiguous()


def g_scale_search_batch(samples: list[torch.Tensor], quant_args: dict):
    """Coarse grid (0.1..1.9 on a 1/3 subsample), fine 5-point grid, parabolic refine.

    Returns [(scale, mse tensor)] per sample set; all evaluations of a stage
    share as few tile launches as the 65,536-tile batch limit allows.
    """
    n_t = len(samples)
    dev = samples[0].device
    max_tiles = 65536

    def evaluate(pairs, sets):
        out = torch.empty(len(pairs), dtype=torch.float, device=dev)
        i = 0
        while i < len(pairs):
            j, tot = i, 0
            while j < len(pairs) and tot + sets[pairs[j][0]].shape[0] <= max_tiles:
                tot += sets[pairs[j][0]].shape[0]
                j += 1
            j = max(j, i + 1)
            batch = torch.cat([sets[t] * s for t, s in pairs[i:j]])
            q, _ = quantize_tiles_multigpu(batch, quant_args)
            off = 0
            for p, (t, s) in enumerate(pairs[i:j]):
                cnt = sets[t].shape[0]
                out[i + p] = (q[off:off + cnt] / s - sets[t]).square().mean()
                off += cnt
            i = j
        return out

    coarse = [0.1 + 0.2 * i for i in range(10)]
    subs = [s[::3] for s in samples]
    mse1 = evaluate([(t, s) for t in range(n_t) for s in coarse], subs).view(n_t, len(coarse))
    centers = [coarse[c] for c in mse1.argmin(dim=1).tolist()]
    step = 0.075
    fine = [[c + step * (i - 2) for i in range(5)] for c in centers]
    mse2 = evaluate([(t, s) for t in range(n_t) for s in fine[t]], samples).view(n_t, 5)
    host = mse2.tolist()
    results = []
    for t in range(n_t):
        best = min(range(5), key=lambda i: host[t][i])
        offset = 0.0
        if 0 < best < 4:
            y0, y1, y2 = host[t][best - 1], host[t][best], host[t][best + 1]
            denom = y0 - 2.0 * y1 + y2
            offset = 0.5 * (y0 - y2) / denom if denom > 0 else 0.0
            offset = max(-0.5, min(0.5, offset))
        results.append((max(fine[t][best] + offset * step, 0.01), mse2[t, best]))
    return results


def g_scale_gss(weight_r: torch.Tensor, verbose: bool, quant_args: dict, width: int = 3, pb=None):
    devices = quant_args["devices"]
    _sync(devices)
    with torch.cuda.stream(get_quant_stream(devices[0])):
        tiles = sample_scale_tiles(weight_r, width)
        if pb:
            pb.update(50)
        best_scale, best_mse = g_scale_search_batch([tiles], quant_args)[0]
        if pb:
            pb.update(100)
        if verbose:
            print(f"     - scale search: min = {best_scale:.6f}, mse: {best_mse.item():.6f}")
    _sync(devices)
    return best_scale, best_mse


# --------------------------------------------------------------------------
# regularisation (kquant/exl3_encoder_backend.py:1811-2042)
# --------------------------------------------------------------------------


def block_rms(x: torch.Tensor, dim: int, keepdim: bool = False, blocksize: int = 32):
    """sqrt(mean(x^2, dim)) accumulated over blocks of ``blocksize`` along ``dim``."""
    acc = None
    for blk in torch.split(x, blocksize, dim=dim):
        part = blk.square().sum(dim=dim, keepdim=keepdim)
        acc = part if acc is None else acc + part
    return (acc / x.size(dim)).sqrt()


def block_rms_n(x: torch.Tensor, dim: int = 0, blocksize: int = 32):
    acc, n = None, 0
    for blk in torch.split(x, blocksize, dim=dim):
        part = blk.square().sum()
        n += blk.numel()
        acc = part if acc is None else acc + part
    return (acc / n).sqrt()


def block_nmse(x: torch.Tensor, y: torch.Tensor, dim: int = 0, blocksize: int = 32):
    sq = diff = None
    for bx, by in zip(torch.split(x, blocksize, dim=dim), torch.split(y, blocksize, dim=dim)):
        a, b = by.square().sum(), (bx - by).square().sum()
        sq = a if sq is None else sq + a
        diff = b if diff is None else diff + b
    return diff.item() / (sq.item() + 1e-20)


_SHARED_INPUT_SCALES: dict = {}


def output_signs(n: int, device, quant_args: dict) -> torch.Tensor:
    """Output sign flips, optionally from their own seed (kquant/exl3_encoder_backend.py:1867-1877)."""
    if "sv_seed" in quant_args:
        torch.manual_seed(quant_args["sv_seed"])
    return (torch.randn(n, device=device).sign() + 1e-5).sign().to(torch.float).unsqueeze(0)


def relocate_g_scale_to_sv(su: torch.Tensor, sv: torch.Tensor, g_scale: float):
    if not math.isfinite(float(g_scale)) or float(g_scale) <= 0.0:
        raise ValueError("g_scale must be positive and finite")
    return su * g_scale, sv / g_scale


def apply_g_scale(weight, su, sv, g_scale: float, *, into_sv: bool = False):
    """Scale the regularised weight; fold 1/g into ``sv`` or ``su`` (kquant/exl3_encoder_backend.py:2018-2042)."""
    if not math.isfinite(float(g_scale)) or float(g_scale) <= 0.0:
        raise ValueError("g_scale must be positive and finite")
    weight *= g_scale
    if into_sv:
        sv /= g_scale
    else:
        su /= g_scale
    return weight, su, sv


def regularize(weight, su, sv, quant_args: dict, verbose: bool, H_diag, pb, skip_g_scale: bool = False,
               q_fallback: bool = False):
    """Sign flips, channel RMS scales and both block Hadamards, then the global scale.

    ``weight`` is transformed in place.  Returns (apply_out_scales, weight,
    g_scale, su, sv) (kquant/exl3_encoder_backend.py:1880-1999).
    """
    force = quant_args["apply_out_scales"]
    if not q_fallback and H_diag is not None:
        d = torch.sort(H_diag.sqrt(), descending=True).values
        skew = d[: d.shape[0] // 50].sum() / d.sum()
        if verbose:
            print(f"     - input state skew: {skew.item():.6f}")
        apply_out = (skew.item() < 0.15) if force is None else force
    else:
        apply_out = True if force is None else force
    if q_fallback:
        apply_out = force
    ocs = block_rms(weight, dim=0, keepdim=True)
    mean = ocs.mean().item()
    if mean > 1e-30:
        ocs /= mean
        quant_args["zeros"] = False
    else:
        quant_args["zeros"] = True
        if force is not None:
            apply_out = True
    zero_cols = ocs.abs() < 1e-30
    if apply_out:
        ocs[zero_cols] = 0.1
        sv = (sv * ocs + 1e-10).float()
    weight /= sv
    sv[zero_cols] = 0.0
    blockwise_preapply_had_r_(weight, had_n)
    ics = block_rms(weight, dim=1, keepdim=True)
    ics[ics.abs() < 1e-30] = 0.1
    key = quant_args.get("shared_input_scales_key")
    if key is not None:
        ics = _SHARED_INPUT_SCALES.setdefault(key, ics)
    su = (su * ics / (-codebook_scale) + 1e-10).float()
    weight /= su
    blockwise_preapply_had_l_(weight, had_k)
    mse_scale = None
    if not skip_g_scale:
        g_scale, mse_scale = g_scale_gss(weight, False, quant_args, pb=pb)
    else:
        g_scale = 1.0
    weight, su, sv = apply_g_scale(weight, su, sv, g_scale, into_sv=bool(quant_args.get("g_scale_into_sv")))
    if verbose:
        print(f"     - su/sv std: {su.std().item():.6f}   {sv.std().item():.6f}")
        print(f"     - global scale: {g_scale:.6f}")
        if mse_scale is not None:
            print(f"     - sample mse: {mse_scale.item():.6f}")
        print(f"     - apply_out_scales: {apply_out}")
    return apply_out, weight, g_scale, su, sv


# --------------------------------------------------------------------------
# top-level encoders (kquant/exl3_encoder_backend.py:2045-2765)
# --------------------------------------------------------------------------


class _NoProgress:
    def __init__(self, *args, **kwargs):
        pass

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        return None

    def update(self, value):
        return None

    def new_task(self, text, count):
        return None


ProgressBar = _NoProgress


def _codebook_tensors(quant_args: dict) -> dict:
    out = {}
    if quant_args.get("mcg"):
        out["mcg"] = torch.tensor(codebook_mcg_mult, dtype=torch.uint32).view(torch.int)
    if quant_args.get("mul1"):
        out["mul1"] = torch.tensor(codebook_mul1_mult, dtype=torch.uint32).view(torch.int)
    return out


def _reconstruct(wq: torch.Tensor, su: torch.Tensor, sv: torch.Tensor) -> torch.Tensor:
    """Original-basis weight had_r(had_l(What) * su) * sv (kquant/exl3_encoder_backend.py:2211-2216).

    One pass over What on the Walsh-Hadamard kernel (``kq_reconstruct_rotated``,
    k and n multiples of 128 as the encoder requires); the reconstruction is an output only
    (it never feeds the codes), so fp32 rounding differences from the
    reference's matmul form are within its 1e-3 reconstruction bound.
    """
    return _native.reconstruct_rotated(wq.contiguous(), su, sv)


def quantize_qsrt(weight: torch.Tensor, H_data: dict, quant_args: dict, return_weight_q: bool,
                  progress_str: str | None = None, verbose: bool = False,
                  swap_to_device: torch.device | None = None, save_reg: str | None = None):
    """Encode one [k, n] fp32 matrix against its captured Hessian.

    Returns (weight_q or None, proxy error, {"suh", "svh", "trellis"} plus
    "mcg"/"mul1" markers) and updates ``quant_args`` with
    apply_out_scales / g_scale / q_fallback (kquant/exl3_encoder_backend.py:2045-2255).
    """
    assert weight.dtype == torch.float
    if "seed" in quant_args:
        torch.manual_seed(quant_args["seed"])
    devices = quant_args["devices"]
    if weight.device != torch.device(devices[0]):
        weight = weight.to(devices[0])
    device = weight.device if swap_to_device is None else swap_to_device
    k, n = weight.shape
    tiles_k = k // 16
    q_fallback, H, L, su, H_diag = finalize_capture_H(H_data, quant_args, verbose)
    if H is not None and H.is_cuda:
        H = H.to(device)
    if su.is_cuda:
        su = su.to(device)
    if H_diag is not None and H_diag.is_cuda:
        H_diag = H_diag.to(device)
    sv = output_signs(n, device, quant_args)
    if H_data["L"] is not None:
        H_data["L"] = _host_copy(H_data["L"])
    if L is not None:
        L = L.to(device)
    if swap_to_device is not None:
        weight = weight.to(swap_to_device)
    weight_ref = weight.cpu() if verbose else None
    apply_out_scales, weight_r, g_scale, su, sv = regularize(weight, su, sv, quant_args, verbose, H_diag, None,
                                                             q_fallback=q_fallback)
    del weight
    mixed = "mixed_rate_axis" in quant_args or "mixed_tile_bits" in quant_args
    if not q_fallback:
        if mixed:
            weight_q, encoded_q = ldlq_mixed(weight_r, L, quant_args)
        else:
            weight_q, encoded_q = ldlq(weight_r, L, quant_args)
        del L
        try:
            Hd = _device_H(H_data, H, device)
            num = block_trace(weight_r - weight_q, Hd)
            den = block_trace(weight_r, Hd)
            proxy_err = num / max(den, 1e-8)
        except torch.OutOfMemoryError:
            proxy_err = -1.0
    else:
        if mixed:
            raise ValueError("mixed-rate quantization requires a non-fallback dense Hessian")
        weight_q, encoded_q, proxy_err = fallback_quant(weight_r, device, quant_args)
    if return_weight_q or verbose:
        weight_q = _reconstruct(weight_q.to(device), su, sv)
        if verbose:
            print(f"     - quant nmse: {block_nmse(weight_q, weight_ref.to(device)):.6f}")
    suh = su.flatten().contiguous().to(dtype=torch.half, copy=True)
    svh = sv.flatten().contiguous().to(dtype=torch.half, copy=True)
    pack_fn = quant_args.get("pack_trellis_fn", pack_trellis)
    trellis = pack_fn(encoded_q.to(device), quant_args)
    out_tensors = {"suh": suh, "svh": svh, "trellis": trellis, **_codebook_tensors(quant_args)}
    quant_args.update({"apply_out_scales": apply_out_scales, "g_scale": g_scale, "q_fallback": q_fallback})
    return weight_q, proxy_err, out_tensors


_PREP_KEYS = ("K", "seed", "sv_seed", "sigma_reg", "devices", "device_ratios", "apply_out_scales", "mcg", "mul1",
              "shared_input_scales_key", "g_scale_into_sv", "buf_size_k", "ldlq_tf32", "tailbite_context",
              "g_scale_override")


def _trace_rows(parts: list[torch.Tensor]) -> list[float]:
    """Sum each row of block-trace terms on the host, in order, in fp64."""
    if not parts:
        return []
    width = max(p.numel() for p in parts)
    rows = torch.stack([torch.nn.functional.pad(p.double(), (0, width - p.numel())) for p in parts]).cpu()
    _native.check_trace_errors()
    values = []
    for row in rows:
        total = 0.0
        for p in row:
            total += p.item()
        values.append(total)
    return values


def quantize_qsrt_batch(weights: list[torch.Tensor], H_datas: list[dict], quant_args_groups: list[list[dict]], *,
                        return_weight_q: bool = True, verbose: bool = False):
    """Prepare each source once and encode all of its rate candidates together.

    Returns, per source, a list of {"weight_q", "encoded", "suh", "svh",
    "proxy", "g_scale"} (kquant/exl3_encoder_backend.py:2258-2535).
    """
    S = len(weights)
    if S <= 0 or len(H_datas) != S or len(quant_args_groups) != S:
        raise ValueError("QSRT batch inputs must have equal nonzero lengths")
    if any(not g for g in quant_args_groups):
        raise ValueError("every QSRT source needs at least one rate candidate")
    if any(w.ndim != 2 or w.dtype != torch.float for w in weights):
        raise TypeError("QSRT batch weights must be float32 matrices")
    shape = weights[0].shape
    if any(w.shape != shape for w in weights):
        raise ValueError("QSRT batch sources must have one matrix shape")
    for group in quant_args_groups:
        ref = group[0]
        for args in group:
            mixed_rate_spec(shape[0], shape[1], args)
            for key in _PREP_KEYS:
                if args.get(key) != ref.get(key):
                    raise ValueError(f"QSRT candidates changed preparation argument {key}")
    devices = quant_args_groups[0][0]["devices"]
    device = torch.device(devices[0])
    if any(g[0].get("devices") != devices for g in quant_args_groups):
        raise ValueError("QSRT source groups must share devices")
    if any(w.device != device for w in weights):
        raise ValueError("QSRT batch weights must already be on the quant device")

    prepared = []
    for weight, H_data, group in zip(weights, H_datas, quant_args_groups):
        args = group[0]
        if "seed" in args:
            torch.manual_seed(args["seed"])
        q_fallback, H, L, su, H_diag = finalize_capture_H(H_data, args, verbose)
        if q_fallback or H is None or L is None:
            raise ValueError("mixed-rate batching requires a non-fallback dense Hessian")
        H, L, su = _device_H(H_data, H, device), L.to(device), su.to(device)
        if H_diag is not None:
            H_diag = H_diag.to(device)
        if H_data["L"] is not None:
            H_data["L"] = _host_copy(H_data["L"])
        sv = output_signs(weight.shape[1], device, args)
        apply_out, weight_r, _, su, sv = regularize(weight, su, sv, args, verbose, H_diag, None, skip_g_scale=True)
        prepared.append({"H": H, "L": L, "weight_r": weight_r, "su": su, "sv": sv, "apply_out_scales": apply_out})

    scales: list = [None] * S
    search_sources, search_samples = [], []
    for s, (item, group) in enumerate(zip(prepared, quant_args_groups)):
        override = group[0].get("g_scale_override")
        if override is None:
            search_sources.append(s)
            search_samples.append(sample_scale_tiles(item["weight_r"]))
        else:
            if (isinstance(override, bool) or not isinstance(override, (int, float))
                    or not math.isfinite(float(override)) or float(override) <= 0.0):
                raise ValueError("g_scale_override must be positive and finite")
            scales[s] = (float(override), None)
    if search_samples:
        for s, res in zip(search_sources, g_scale_search_batch(search_samples,
                                                               quant_args_groups[search_sources[0]][0])):
            scales[s] = res
    del search_samples
    if any(r is None for r in scales):
        raise AssertionError("global scale search did not cover every source")
    for item, group, (g_scale, _) in zip(prepared, quant_args_groups, scales):
        item["weight_r"], item["su"], item["sv"] = apply_g_scale(
            item["weight_r"], item["su"], item["sv"], g_scale, into_sv=bool(group[0].get("g_scale_into_sv")))
        item["g_scale"] = g_scale

    flat = [(s, c) for s, g in enumerate(quant_args_groups) for c in range(len(g))]
    specs = [[mixed_rate_spec(shape[0], shape[1], a) for a in g] for g in quant_args_groups]
    reuse_n = all(all(ax == "n" for ax, _ in sp) and sp[0][1] == (3,) * (shape[1] // 16) for sp in specs)
    reuse_k = any(len(g) > 1 for g in quant_args_groups) and all(all(ax == "k" for ax, _ in sp) for sp in specs)
    source_weights = None
    if reuse_n:
        source_weights = torch.stack([it["weight_r"] for it in prepared])
        weights_q, encoded_q = ldlq_mixed_n_candidates_reuse(
            source_weights, torch.stack([it["L"] for it in prepared]), quant_args_groups)
    elif reuse_k:
        source_weights = torch.stack([it["weight_r"] for it in prepared])
        weights_q, encoded_q = ldlq_mixed_k_candidates_prefix_reuse(
            source_weights, torch.stack([it["L"] for it in prepared]), quant_args_groups)
    else:
        weights_batch = torch.stack([prepared[s]["weight_r"] for s, _ in flat])
        weights_q, encoded_q = ldlq_mixed_batched(
            weights_batch, torch.stack([prepared[s]["L"] for s, _ in flat]),
            [quant_args_groups[s][c] for s, c in flat])

    den_parts = [block_trace_parts(it["weight_r"], it["H"]) for it in prepared]
    num_parts, pending = [], []
    for f, (s, c) in enumerate(flat):
        item = prepared[s]
        args = quant_args_groups[s][c]
        src = source_weights[s] if source_weights is not None else weights_batch[f]
        num_parts.append(block_trace_parts(src - weights_q[f], item["H"]))
        if "suh" not in item:
            item["suh"] = item["su"].flatten().contiguous().to(dtype=torch.half, copy=True)
            item["svh"] = item["sv"].flatten().contiguous().to(dtype=torch.half, copy=True)
        recon = None
        if return_weight_q:
            recon = _reconstruct(weights_q[f], item["suh"].float().unsqueeze(1),
                                 item["svh"].float().unsqueeze(0)).contiguous()
        args.update({"apply_out_scales": item["apply_out_scales"], "g_scale": item["g_scale"], "q_fallback": False,
                     "zeros": quant_args_groups[s][0].get("zeros", False)})
        pending.append((s, recon, encoded_q[f].contiguous(), item["suh"], item["svh"]))
    traces = _trace_rows(den_parts + num_parts)
    dens, nums = traces[:S], traces[S:]
    results = [[] for _ in range(S)]
    for num, (s, recon, enc, suh, svh) in zip(nums, pending):
        results[s].append({"weight_q": recon, "encoded": enc, "suh": suh, "svh": svh,
                           "proxy": num / max(dens[s], 1e-8), "g_scale": prepared[s]["g_scale"]})
    return results


def _uniform_prepare(weights: list[torch.Tensor], H_datas: list[dict], quant_args_list: list[dict],
                     verbose: bool, search: bool = True):
    """Phase 1 of quantize_uniform_batch: H finalisation, regularisation, global scale.

    Consumes the RNG exactly as the reference does (reseeded per matrix).
    Returns the batch state; ``state["ldlq"]`` is None when every member fell
    back (``state["results"]`` is then complete).  With ``search=False`` it
    stops before the scale search, leaving ``state["samples"]`` for a search
    shared with other batches (:func:`_uniform_apply_scales` then finishes).
    """
    if any("mixed_rate_axis" in a or "mixed_tile_bits" in a for a in quant_args_list):
        raise ValueError("mixed-rate LDLQ is currently supported by quantize_qsrt, not the same-K batch API")
    n_t = len(weights)
    qa0 = quant_args_list[0]
    device = torch.device(qa0["devices"][0])
    shared_H = all(h is H_datas[0] for h in H_datas)
    assert shared_H or all(w.shape == weights[0].shape for w in weights)
    assert all(w.shape[0] == weights[0].shape[0] for w in weights)
    assert all(a["K"] == qa0["K"] for a in quant_args_list)
    results: list = [None] * n_t
    finalized, batch = [], []
    for t in range(n_t):
        qa = quant_args_list[t]
        if "seed" in qa:
            torch.manual_seed(qa["seed"])
        q_fallback, H, L, su, H_diag = finalize_capture_H(H_datas[t], qa, verbose)
        if q_fallback:
            finalized.append(None)
        else:
            finalized.append((H, L, su, H_diag))
            batch.append(t)
    for t in range(n_t):
        if finalized[t] is None:
            results[t] = quantize_qsrt(weights[t], H_datas[t], quant_args_list[t], False, None, verbose)[1:]
    state = {"results": results, "H_datas": H_datas, "quant_args_list": quant_args_list, "device": device,
             "shared_H": shared_H, "finalized": finalized, "batch": batch, "ldlq": None}
    if not batch:
        return state
    regs = {}
    for t in batch:
        qa = quant_args_list[t]
        if "seed" in qa:
            torch.manual_seed(qa["seed"])
        H, L, su, H_diag = finalized[t]
        w = weights[t] if weights[t].device == device else weights[t].to(device)
        su = su.to(device) if su.is_cuda else su
        if H_diag is not None and H_diag.is_cuda:
            H_diag = H_diag.to(device)
        sv = output_signs(w.shape[1], device, qa)
        apply_out, wr, _, su, sv = regularize(w, su, sv, qa, verbose, H_diag, None, skip_g_scale=True)
        regs[t] = [wr, su, sv, apply_out]
        weights[t] = None
    state.update(regs=regs, samples=[sample_scale_tiles(regs[t][0]) for t in batch])
    if not search:
        return state
    return _uniform_apply_scales(state, g_scale_search_batch(state["samples"], qa0))


def _search_key(quant_args: dict):
    """Launch-compatibility key of a scale search: same K, codebook, context and devices."""
    bits = int(quant_args["K"])
    kind, lut = _tile_codebook(quant_args, bits)
    return (bits, kind, id(lut), int(quant_args.get("tailbite_context", 128)), tuple(quant_args["devices"]))


def _uniform_apply_scales(state: dict, scales):
    """Phase 1b: apply the searched global scales and set up the LDLQ operands."""
    batch, regs, finalized = state["batch"], state["regs"], state["finalized"]
    quant_args_list, device, shared_H = state["quant_args_list"], state["device"], state["shared_H"]
    qa0 = quant_args_list[0]
    state.pop("samples", None)
    g_scales = {}
    for t, (g, _) in zip(batch, scales):
        regs[t][0] *= g
        if quant_args_list[t].get("g_scale_into_sv"):
            regs[t][2] /= g
        else:
            regs[t][1] /= g
        g_scales[t] = g
    # LDLQ operands: a shared H concatenates the members along N into one
    # traversal; distinct Hessians of one shape are stacked.
    if shared_H:
        L = finalized[batch[0]][1].to(device)
        widths = [regs[t][0].shape[1] for t in batch]
        W = torch.cat([regs[t][0] for t in batch], dim=1).unsqueeze(0)
        Ls = L.unsqueeze(0)
    else:
        widths = None
        Ls = torch.stack([finalized[t][1].to(device) for t in batch])
        W = torch.stack([regs[t][0] for t in batch])
    for t in batch:
        regs[t][0] = None
    _, size_k, size_n = W.shape
    assert size_k % 16 == 0 and size_n % 128 == 0
    kind, lut = _tile_codebook(qa0, int(qa0["K"]))
    _labels_for(device, int(qa0["K"]), kind, lut)    # built before any traversal stream uses it
    state.update(regs=regs, g_scales=g_scales, widths=widths, ldlq=(W, Ls))
    return state


def _uniform_members(state: dict):
    """Chain-engine members of a prepared batch: one per stacked matrix; returns (members, What, enc)."""
    W, Ls = state["ldlq"]
    qa0 = state["quant_args_list"][0]
    B, size_k, size_n = W.shape
    wq = torch.empty_like(W)
    enc = torch.empty((B, size_k // 16, size_n // 16, 256), dtype=torch.int16, device=W.device)
    members = [_ChainMember(W[b], Ls[b if Ls.shape[0] == B else 0], wq[b], enc[b], qa0) for b in range(B)]
    return members, wq, enc


def _uniform_finish(state: dict, wq: torch.Tensor, enc: torch.Tensor):
    """Phase 3: proxy, optional error metrics, packing and outputs of a traversed batch."""
    results, batch, regs = state["results"], state["batch"], state["regs"]
    quant_args_list, H_datas, finalized = state["quant_args_list"], state["H_datas"], state["finalized"]
    device, shared_H, g_scales = state["device"], state["shared_H"], state["g_scales"]
    W, _ = state["ldlq"]
    state["ldlq"] = None
    if shared_H:
        widths = state["widths"]
        wrs = list(torch.split(W[0], widths, dim=1))
        wqs = list(torch.split(wq[0], widths, dim=1))
        encs = list(torch.split(enc[0], [w // 16 for w in widths], dim=1))
    else:
        wrs, wqs, encs = list(W.unbind(0)), list(wq.unbind(0)), list(enc.unbind(0))
    del W, wq, enc
    Hd = None
    for bi, t in enumerate(batch):
        qa = quant_args_list[t]
        _, su, sv, apply_out = regs[t]
        if Hd is None or not shared_H:
            Hd = _device_H(H_datas[t], finalized[t][0], device)
        try:
            num = block_trace(wrs[bi] - wqs[bi], Hd)
            den = block_trace(wrs[bi], Hd)
            proxy = num / max(den, 1e-8)
        except torch.OutOfMemoryError:
            proxy = -1.0
        if qa.get("return_error_metrics") and proxy >= 0.0:
            wr_o = _reconstruct(wrs[bi].to(device), su, sv)
            wq_o = _reconstruct(wqs[bi].to(device), su, sv)
            cerr = wr_o - wq_o
            eh = qa.get("error_hessian")
            if eh is None:
                cnum, cden = num, den
            else:
                if eh.shape != (wr_o.shape[0], wr_o.shape[0]):
                    raise ValueError("error_hessian shape does not match quantized input dimension: "
                                     f"{eh.shape} vs {wr_o.shape[0]}")
                eh = eh.to(device)
                cnum, cden = block_trace(cerr, eh), block_trace(wr_o, eh)
            qa["error_metrics"] = {"numerator": float(cnum), "denominator": float(cden),
                                   "encoder_numerator": float(num), "encoder_denominator": float(den),
                                   "residual_by_input": cerr.square().sum(dim=1).cpu()}
        wrs[bi] = wqs[bi] = None
        out = {"suh": su.flatten().contiguous().to(dtype=torch.half, copy=True),
               "svh": sv.flatten().contiguous().to(dtype=torch.half, copy=True),
               "trellis": pack_trellis(encs[bi].contiguous(), qa), **_codebook_tensors(qa)}
        encs[bi] = None
        qa.update({"apply_out_scales": apply_out, "g_scale": g_scales[t], "q_fallback": False})
        results[t] = (proxy, out)
    return results


def quantize_uniform_batch(weights: list[torch.Tensor], H_datas: list[dict], quant_args_list: list[dict],
                           progress_str: str | None = None, verbose: bool = False):
    """Encode same-K linears together (kquant/exl3_encoder_backend.py:2538-2765).

    A shared H object concatenates the regularised weights along N into one
    LDLQ traversal; distinct Hessians of one shape go through one batched
    traversal.  Returns [(proxy, out_tensors)] per input and updates each
    quant_args.
    """
    state = _uniform_prepare(weights, H_datas, quant_args_list, verbose)
    if state["ldlq"] is None:
        return state["results"]
    devices = quant_args_list[0]["devices"]
    _sync(devices)
    with torch.cuda.stream(get_quant_stream(state["device"])):
        if len(devices) == 1:
            members, wq, enc = _uniform_members(state)
            _chain_traverse(members, state["device"])
        else:
            wq, enc = _uniform_traversal_multigpu(state)
    _sync(devices)
    return _uniform_finish(state, wq, enc)


def _uniform_traversal_multigpu(state: dict):
    """Uniform-batch traversal whose tile launches split across several devices (quantize_tiles_multigpu)."""
    W, Ls = state["ldlq"]
    qa0 = state["quant_args_list"][0]
    plan = _RatePlan(int(qa0["K"]), None, W.shape[0], W.shape[2] // 16, W.device)
    wq, enc, _ = _ldlq_traverse(W, Ls, qa0, plan, buffer_rows=_buffer_rows(qa0, W.shape[1]),
                                tf32=bool(qa0.get("ldlq_tf32", False)))
    return wq, enc


def quantize_uniform_batches(groups, verbose: bool = False):
    """Several independent ``quantize_uniform_batch`` calls whose LDLQ traversals share launches.

    ``groups`` is a list of (weights, H_datas, quant_args_list).  The
    preparation phases run in order (same RNG seeding as sequential calls),
    the global-scale searches of all groups with the same (K, codebook,
    context) share their tile launches, then every matrix of every group is
    one set of chains in a single chain-engine run (:func:`_chain_traverse`),
    then the outputs are built in order.  Results equal the sequential calls bit for bit: a chain step's
    arithmetic does not depend on which other chains share its launch.
    Returns one result list per group.  Groups spanning several devices run
    sequentially.
    """
    groups = [(list(w), list(h), list(q)) for w, h, q in groups]
    if any(len(q[0]["devices"]) > 1 for _, _, q in groups) or len(groups) < 2:
        return [quantize_uniform_batch(w, h, q, None, verbose) for w, h, q in groups]
    states = [_uniform_prepare(w, h, q, verbose, search=False) for w, h, q in groups]
    # one scale search per (K, codebook, context, devices) over every group's samples
    pending = [i for i, st in enumerate(states) if st.get("samples")]
    by_key: dict = {}
    for i in pending:
        by_key.setdefault(_search_key(states[i]["quant_args_list"][0]), []).append(i)
    for idx in by_key.values():
        samples = [t for i in idx for t in states[i]["samples"]]
        scales = g_scale_search_batch(samples, states[idx[0]]["quant_args_list"][0])
        at = 0
        for i in idx:
            n = len(states[i]["samples"])
            _uniform_apply_scales(states[i], scales[at:at + n])
            at += n
    live = [i for i, st in enumerate(states) if st["ldlq"] is not None]
    out = {}
    by_device: dict = {}
    for i in live:
        by_device.setdefault(str(states[i]["device"]), []).append(i)
    for dev_name, idx in by_device.items():
        dev = torch.device(dev_name)
        _sync([dev_name])
        with torch.cuda.stream(get_quant_stream(dev)):
            members = []
            for i in idx:
                m, wq, enc = _uniform_members(states[i])
                members += m
                out[i] = (wq, enc)
            _chain_traverse(members, dev)
        _sync([dev_name])
    return [st["results"] if st["ldlq"] is None else _uniform_finish(st, *out[i]) for i, st in enumerate(states)]


# --------------------------------------------------------------------------
# LDLQ chain engine
# --------------------------------------------------------------------------

# Tile columns per chain.  Columns of a matrix are independent under LDLQ
# (the feedback of column j reads only column j of the error rows), so a
# matrix splits into chains that may sit at different rows.  Narrow chains
# let a launch be filled to whole waves of 2 x SMs tiles.
CHAIN_TILES = 32


class _ChainMember:
    """One [k, n] matrix of a chain-engine run with its LDLQ state.

    ``rate`` gives the per-tile K: an int (uniform), ("n", bits per tile
    column) or ("k", bits per tile row) as in mixed_rate_spec.  ``state``
    optionally supplies (What, enc, P, E) arrays to fill instead of fresh ones.
    """

    def __init__(self, W, L, wq, enc, quant_args, rate=None, P=None, E=None):
        self.W = W
        self.L = L if L.is_contiguous() else L.contiguous()
        self.wq = wq
        self.enc = enc
        self.k, self.n = W.shape
        assert W.is_contiguous() and wq.is_contiguous() and enc.is_contiguous()
        assert self.k % 16 == 0 and self.n % 16 == 0
        self.P = torch.zeros_like(W) if P is None else P
        self.E = torch.empty_like(W) if E is None else E
        self.buffer_rows = _buffer_rows(quant_args, self.k)
        self.tf32 = bool(quant_args.get("ldlq_tf32", False))
        self.rate = int(quant_args["K"]) if rate is None else rate
        bits = {self.rate} if isinstance(self.rate, int) else set(self.rate[1])
        if not bits <= set(TRELLIS_BITS):
            raise ValueError("the trellis kernels support K1--K8")
        # K2..K4 run on the chain kernel; K1 and K5..K8 (uniform only) step by step
        self.chain_ok = bits <= {2, 3, 4}
        self.quant_args = quant_args
        self.ctx = int(quant_args.get("tailbite_context", 128))
        if not 1 <= self.ctx <= 128:
            raise ValueError("tailbite_context must be in 1..128")
        self.labels = {}
        for K in bits:
            kind, lut = _tile_codebook(quant_args, K)
            self.labels[K] = _labels_for(W.device, K, kind, lut)

    def column_runs(self, width: int):
        """Tile-column ranges of the chains: runs of one K along n, cut to at most ``width`` tiles."""
        tn = self.n // 16
        if isinstance(self.rate, tuple) and self.rate[0] == "n":
            bits = self.rate[1]
            runs, c0 = [], 0
            for c in range(1, tn + 1):
                if c == tn or bits[c] != bits[c0]:
                    runs.append((c0, c))
                    c0 = c
        else:
            runs = [(0, tn)]
        out = []
        for c0, c1 in runs:
            out += [(c, min(width, c1 - c)) for c in range(c0, c1, width)]
        return out

    def bits_at(self, r0: int, tile_col: int) -> int:
        if isinstance(self.rate, int):
            return self.rate
        axis, bits = self.rate
        return bits[tile_col] if axis == "n" else bits[r0 // 16]


class _Chain:
    def __init__(self, member: _ChainMember, tile_col0: int, n_tiles: int, steps=None, pos: int = 0):
        self.m = member
        self.tile_col0 = tile_col0
        self.n_tiles = n_tiles
        rows = member.buffer_rows
        # (r0, end) of every step, in traversal order (backward over 128-row buffers)
        self.steps = steps if steps is not None else [(end - rows + le - 16, end) for end in range(member.k, 0, -rows)
                                                      for le in range(rows, 0, -16)]
        self.pos = pos

    @property
    def remaining(self):
        return len(self.steps) - self.pos

    @property
    def K(self):
        return self.m.bits_at(self.steps[self.pos][0], self.tile_col0)

    def item(self):
        m = self.m
        r0, end = self.steps[self.pos]
        K = self.K
        return _native.ChainItem(m.W.data_ptr(), m.P.data_ptr(), m.L.data_ptr(), m.E.data_ptr(), m.wq.data_ptr(),
                                 m.enc.data_ptr(), m.k, m.n, r0, end, self.tile_col0, self.n_tiles,
                                 m.labels[K].data_ptr(), K, 0)

    def advance(self):
        """Step done: after a buffer's last step, P[:begin] += L[begin:end, :begin]^T E[begin:end] (own columns)."""
        r0, end = self.steps[self.pos]
        self.pos += 1
        begin = end - self.m.buffer_rows
        if r0 == begin and begin > 0:
            m = self.m
            c0, c1 = 16 * self.tile_col0, 16 * (self.tile_col0 + self.n_tiles)
            previous = torch.backends.cuda.matmul.allow_tf32
            torch.backends.cuda.matmul.allow_tf32 = m.tf32
            try:
                m.P[:begin, c0:c1].addmm_(m.L[begin:end, :begin].T, m.E[begin:end, c0:c1])
            finally:
                torch.backends.cuda.matmul.allow_tf32 = previous


def _launch_key(c: _Chain):
    return c.K, c.m.labels[c.K].data_ptr()


MAX_CTA_PAIRS = 4   # tile pairs per CTA of one chain launch


def _launch_fits(chains, sms: int) -> bool:
    """Whether a mixed chain launch fits (kq_ldlq_chain_step): each (K, label table) group's tile pairs in runs
    of m per CTA, m from ceil(pairs / SMs) up to MAX_CTA_PAIRS, need at most one CTA per SM."""
    pairs: dict = {}
    for c in chains:
        k = _launch_key(c)
        pairs[k] = pairs.get(k, 0) + (c.n_tiles + 1) // 2
    total = sum(pairs.values())
    for m in range(max(1, -(-total // sms)), MAX_CTA_PAIRS + 1):
        if sum(-(-p // m) for p in pairs.values()) <= sms:
            return True
    return False


def _select_launch(cands: list, cap: int, sms: int) -> list:
    """Chains for one launch, in priority order, within ``cap`` tiles and KQ_CHAIN_MAX_ITEMS items.

    Chains of different K (or codebook) share a launch pair-aligned: every
    item starts at an even tile (an odd-length chain, an odd run of one K
    along n, only last) and each CTA runs two pairs of one K, so the pairs of
    each (K, labels) group, halved and rounded up, must fit the SMs.
    """
    sel, tot = [], 0
    for c in cands:
        if len(sel) >= _native.KQ_CHAIN_MAX_ITEMS:
            break
        if tot + c.n_tiles <= cap or not sel:
            sel.append(c)
            tot += c.n_tiles
    if len({_launch_key(c) for c in sel}) <= 1:
        return sel
    evens, odd, tot = [], None, 0
    for c in cands:
        if len(evens) + (odd is not None) >= _native.KQ_CHAIN_MAX_ITEMS:
            break
        if tot + c.n_tiles > cap and (evens or odd is not None):
            continue
        if c.n_tiles % 2:
            if odd is None and _launch_fits(evens + [c], sms):
                odd = c
                tot += c.n_tiles
        elif _launch_fits(evens + [c] + ([odd] if odd is not None else []), sms):
            evens.append(c)
            tot += c.n_tiles
    return evens + ([odd] if odd is not None else [])


def _member_step_gen(m: _ChainMember):
    tiles_n = m.n // 16
    plan = _RatePlan(int(m.rate), None, 1, tiles_n, m.W.device)
    return _ldlq_traverse_steps(m.W.unsqueeze(0), m.L.unsqueeze(0), m.quant_args, plan, buffer_rows=m.buffer_rows,
                                tf32=m.tf32, state=(m.wq.unsqueeze(0), m.enc.unsqueeze(0), m.P.unsqueeze(0)))


@lru_cache
def _side_stream_cached(device: torch.device, i: int):
    return torch.cuda.Stream(device=device)


def _side_stream(device, i: int):
    """The i-th side stream of a device, created once and reused."""
    d = torch.device(device)
    if d.index is None:
        d = torch.device(d.type, torch.cuda.current_device())
    return _side_stream_cached(d, i)


def _members_steps(ms: list) -> None:
    """LDLQ of members at rates the chain kernel does not cover (K1, K5..K8): one launch per 16-row step.

    The steps are those of :func:`_ldlq_traverse_steps` (feedback by FP32
    GEMM, tile gather, the wide-butterfly Viterbi kernel, scatter), written
    into each member's own What / codes / feedback arrays.  Several members
    advance in turn, each on its own stream, so one member's last partial
    wave of tiles shares the GPU with the others' launches; every member's
    arithmetic is unchanged.
    """
    if not ms:
        return
    if len(ms) == 1:
        _drive(_member_step_gen(ms[0]))
        return
    dev = ms[0].W.device
    cur = torch.cuda.current_stream(dev)
    live = []
    for i, m in enumerate(ms):
        st = _side_stream(dev, i)
        st.wait_stream(cur)
        with torch.cuda.stream(st):
            live.append((st, _member_step_gen(m)))
    streams = [st for st, _ in live]
    while live:
        nxt = []
        for st, gen in live:
            with torch.cuda.stream(st):
                try:
                    next(gen)
                    nxt.append((st, gen))
                except StopIteration:
                    pass
        live = nxt
    for st in streams:
        cur.wait_stream(st)


def _chain_traverse(members: list, device: torch.device, chain_tiles: int | None = None, on_buffer=None) -> None:
    """Block-LDLQ of every member (kquant/exl3_encoder_backend.py:389-505 per matrix), fills What and codes.

    Each member splits into column chains of at most ``CHAIN_TILES`` tiles
    and one K along the output axis.  Every launch (``kq_ldlq_chain_step``)
    advances a set of chains by one 16-row step: the chains with the most
    steps left first (the critical path), then any others that fit, all with
    the same tail-biting context; chains of different K share launches.  A
    launch holds up to 2 p x SMs tiles (p tile pairs per CTA, p up to 4) while
    the work left exceeds what p - 1 pairs per SM along the critical path
    would cover; one wave (2 x SMs) at the end.  The kernel computes each step's feedback
    product itself; the buffer-end feedback updates run between launches on
    the same stream.  ``on_buffer(chain)``, when given, is called when a chain
    is about to start a new 128-row buffer and may return replacement chains
    (the forks of a candidate trie).
    """
    width = chain_tiles or CHAIN_TILES
    _members_steps([m for m in members if not m.chain_ok])
    members = [m for m in members if m.chain_ok]
    chains = [_Chain(m, c0, nt) for m in members for c0, nt in m.column_runs(width)]
    sms = torch.cuda.get_device_properties(device).multi_processor_count
    order = {id(c): i for i, c in enumerate(chains)}
    serial = len(chains)
    live = list(chains)
    asked = set()
    while live:
        if on_buffer is not None:
            grown = []
            for c in live:
                r0, end = c.steps[c.pos]
                if r0 == end - 16 and end < c.m.k and (id(c), c.pos) not in asked:
                    asked.add((id(c), c.pos))
                    new = on_buffer(c)
                    if new:
                        for n in new:
                            order[id(n)] = serial
                            serial += 1
                        grown += new
                        continue
                grown.append(c)
            live = grown
        live.sort(key=lambda c: (-c.remaining, order[id(c)]))
        ctx = live[0].m.ctx
        same = [c for c in live if c.m.ctx == ctx]
        # Two tile pairs per SM (each CTA hides one pair's tracebacks under the
        # other's forward steps) while the remaining work exceeds what one-wave
        # launches along the critical path would cover; one pair per SM after.
        work = sum(c.n_tiles * c.remaining for c in same)
        crit = same[0].remaining
        # p tile pairs per SM: the largest p whose launches along the critical path
        # would still not cover the work left; a launch of p > 1 pairs per SM
        # pays only when it comes out at least 90% full.
        p = 1
        while p < MAX_CTA_PAIRS and work > 2 * sms * (p + 1) * crit:
            p += 1
        if p == 1 and work > 2 * sms * crit:
            p = 2
        while True:
            sel = _select_launch(same, 2 * p * sms, sms)
            if p == 1 or sum(c.n_tiles for c in sel) >= 0.9 * 2 * p * sms:
                break
            p -= 1
        _native.ldlq_chain_step([c.item() for c in sel], ctx, device)
        for c in sel:
            c.advance()
        live = [c for c in live if c.remaining > 0]


def pack_signs(signs: torch.Tensor, quant_args: dict) -> torch.Tensor:
    """Sign-bit packing of the upstream EXL3 format (kquant/exl3_encoder_backend.py:1680-1685).

    The upstream kernel is not part of the reference tree and its bit order is
    unpinned, so this entry point refuses rather than guess a format.
    """
    raise NotImplementedError("pack_signs: upstream EXL3 sign packing is not pinned by the reference")
