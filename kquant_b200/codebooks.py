"""SQG E4M3 codebook tables for the L16 bitshift trellis.

A codebook maps every 16-bit trellis state ``t`` to one finite E4M3 byte.
The Viterbi kernel widens that byte to binary16 (exactly) and uses it as the
reconstruction label of ``t``.  The tables are built once, on the host, and
cached.  They are format definitions: the mixer constants, the rational
inverse-normal approximation, and the T12 modal rule must match the
reference byte for byte.  The reference's SHA-256 fixtures pin them
(``tests/test_sqg_e4m3.py:32-69`` in the reference).

Reference: ``kquant/sqg_e4m3.py`` (``_mix_width`` :41-61,
``_sqg_cpu_bytes`` :83-120, ``sqg_cheb_normal_rank_e4m3_bytes`` :217-231,
``sqg_xor_cheb_t12_rank_lut_bytes`` :234-248,
``sqg_xor_rank_permutation`` :251-275, ``sqg_codebook_bytes`` :305-333,
``sqg_k2_eight_stratum_rank_permutation`` :356-382, ``sqg_rank_permutation``
:411-438).
"""

from __future__ import annotations

from functools import lru_cache

import numpy as np
import torch

SQG_NORMAL_E4M3 = "sqg-normal-e4m3"
SQG_CHEB_NORMAL_E4M3 = "sqg-cheb-normal-e4m3"
SQG_CHEB = "sqg_cheb"
SQG_XOR_CHEB_T12 = "sqg_xor_cheb_t12"
QSRT_CODEBOOKS = (SQG_XOR_CHEB_T12, SQG_NORMAL_E4M3, SQG_CHEB_NORMAL_E4M3, SQG_CHEB)

STATES = 1 << 16
_CLIP = 1.0 / 2048.0
# Rational inverse-normal approximation in x = (2p - 1)^2 (odd in 2p - 1).
_NUM = (1.25667142, 2.87422731, -9.02398882, 5.36810336, -0.46703015)
_DEN = (1.0, 2.07630930, -8.08332684, 6.32135736, -1.31208298)


def _check_bits(bits: int) -> None:
    if isinstance(bits, bool) or not isinstance(bits, int) or bits not in (2, 3, 4):
        raise ValueError("SQG supports integer K2, K3, or K4")


def _check_mode(mode: str) -> None:
    if mode != "normal":
        raise ValueError("the supported R44 mode is 'normal'")


def _xorshift_mix(v: np.ndarray, width: int, mults: tuple[int, int],
                  shifts: tuple[int, int, int]) -> np.ndarray:
    """Bijective xorshift / odd-multiply mixer modulo 2**width."""
    mask = (1 << width) - 1
    clamp = lambda s: min(max(s, 1), width - 1)  # noqa: E731
    r = v & mask
    for m, s in zip(mults, shifts[:2]):
        r = r ^ (r >> clamp(s))
        r = (r * (m | 1)) & mask
    r = r ^ (r >> clamp(shifts[2]))
    return r & mask


def _bit_reverse(v: np.ndarray, bits: int) -> np.ndarray:
    out = np.zeros_like(v)
    for i in range(bits):
        out |= ((v >> i) & 1) << (bits - 1 - i)
    return out


def _graph_fields(bits: int) -> tuple[np.ndarray, np.ndarray, int]:
    t = np.arange(STATES, dtype=np.int64)
    return t >> bits, t & ((1 << bits) - 1), 16 - bits


def _r44_phase_and_stratum(bits: int) -> tuple[np.ndarray, np.ndarray, int]:
    history, branch, width = _graph_fields(bits)
    phase = _xorshift_mix(history, width, (0x65AF, 0x16BF), (6, 4, 5))
    syndrome = _xorshift_mix(history ^ 0x5105, width, (0x8693, 0x2A21), (2, 4, 4))
    syndrome &= (1 << bits) - 1
    stratum = (7 * (_bit_reverse(branch, bits) ^ syndrome)) & ((1 << bits) - 1)
    return phase, stratum, width


def _to_e4m3_bytes(values: torch.Tensor) -> torch.Tensor:
    return values.to(torch.float8_e4m3fn).view(torch.uint8).contiguous()


@lru_cache(maxsize=None)
def sqg_rank_permutation_np(bits: int) -> np.ndarray:
    _check_bits(bits)
    phase, stratum, width = _r44_phase_and_stratum(bits)
    return (stratum << width) | phase


def sqg_rank_permutation(bits: int) -> torch.Tensor:
    """Quantile rank of every state under the R44 SQG graph labelling."""
    return torch.from_numpy(sqg_rank_permutation_np(bits).copy())


@lru_cache(maxsize=None)
def _r44_normal_bytes(bits: int) -> torch.Tensor:
    rank = torch.from_numpy(sqg_rank_permutation_np(bits).copy())
    p = ((rank.double() + 0.5) / STATES).clamp(_CLIP, 1.0 - _CLIP)
    a = 2.0 * p - 1.0
    x = a.square()
    num = torch.full_like(x, _NUM[-1])
    den = torch.full_like(x, _DEN[-1])
    for c in reversed(_NUM[:-1]):
        num = num * x + c
    for c in reversed(_DEN[:-1]):
        den = den * x + c
    values = (1.5 * (a * num / den)).float()
    if not bool(torch.isfinite(values).all()):
        raise RuntimeError("SQG compander produced a non-finite value")
    return _to_e4m3_bytes(values)


def sqg_e4m3_bytes(bits: int, mode: str, *, device="cpu") -> torch.Tensor:
    """65,536 raw E4M3 labels of the R44 normal SQG graph."""
    _check_bits(bits)
    _check_mode(mode)
    return _r44_normal_bytes(bits).to(device=device).contiguous()


def sqg_e4m3_codebook(bits: int, mode: str, *, device="cpu", dtype=torch.float16) -> torch.Tensor:
    if not dtype.is_floating_point:
        raise TypeError("SQG codebook dtype must be floating point")
    return sqg_e4m3_bytes(bits, mode, device=device).view(torch.float8_e4m3fn).to(dtype).contiguous()


def _validate_rank_lut(rank_lut: torch.Tensor) -> torch.Tensor:
    if rank_lut.dtype != torch.uint8:
        raise TypeError("SQG rank LUT must contain raw uint8 E4M3 labels")
    if rank_lut.ndim != 1 or rank_lut.numel() != STATES:
        raise ValueError("SQG rank LUT must contain exactly 65,536 labels")
    rank_lut = rank_lut.detach().to("cpu").contiguous()
    if not bool(torch.isfinite(rank_lut.view(torch.float8_e4m3fn).float()).all()):
        raise ValueError("SQG rank LUT must contain only finite E4M3 labels")
    return rank_lut


def sqg_e4m3_bytes_from_rank_lut(bits: int, rank_lut: torch.Tensor, *, device="cpu") -> torch.Tensor:
    """Label the R44 graph with a rank-indexed E4M3 staircase."""
    _check_bits(bits)
    rank_lut = _validate_rank_lut(rank_lut)
    return rank_lut.index_select(0, sqg_rank_permutation(bits)).to(device=device).contiguous()


def sqg_e4m3_codebook_from_rank_lut(bits: int, rank_lut: torch.Tensor, *, device="cpu",
                                    dtype=torch.float16) -> torch.Tensor:
    if not dtype.is_floating_point:
        raise TypeError("SQG codebook dtype must be floating point")
    raw = sqg_e4m3_bytes_from_rank_lut(bits, rank_lut, device=device)
    return raw.view(torch.float8_e4m3fn).to(dtype).contiguous()


def _canonical_e4m3_staircase(values: torch.Tensor) -> torch.Tensor:
    raw = _to_e4m3_bytes(values.float()).clone()
    raw[(raw & 0x7F) == 0] = 0              # one canonical zero byte
    decoded = raw.view(torch.float8_e4m3fn).float()
    if not bool(torch.isfinite(decoded).all()):
        raise RuntimeError("SQG rank law rounded to a non-finite E4M3 value")
    if not bool(torch.all(decoded[1:] >= decoded[:-1])):
        raise RuntimeError("SQG rank law is not monotone after E4M3 rounding")
    return raw


@lru_cache(maxsize=1)
def sqg_cheb_normal_rank_e4m3_bytes() -> torch.Tensor:
    """Midpoint normal quantiles 1.5 * ndtri((r + 0.5) / 65536), rounded to E4M3."""
    r = torch.arange(STATES, dtype=torch.float64)
    return _canonical_e4m3_staircase(1.5 * torch.special.ndtri((r + 0.5) / STATES))


@lru_cache(maxsize=None)
def sqg_cheb_normal_e4m3_bytes(bits: int) -> torch.Tensor:
    return sqg_e4m3_bytes_from_rank_lut(bits, sqg_cheb_normal_rank_e4m3_bytes()).contiguous()


@lru_cache(maxsize=1)
def sqg_xor_cheb_t12_rank_lut_bytes() -> torch.Tensor:
    """4,096-entry modal compression of the normal staircase (ties -> lower byte)."""
    exact = sqg_cheb_normal_rank_e4m3_bytes().numpy().reshape(1 << 12, 16)
    out = np.empty(1 << 12, dtype=np.uint8)
    for i, block in enumerate(exact):
        counts = np.bincount(block, minlength=256)
        out[i] = np.flatnonzero(counts == counts.max()).min()
    return torch.from_numpy(out)


@lru_cache(maxsize=None)
def _xor_rank_np(bits: int) -> np.ndarray:
    history, branch, width = _graph_fields(bits)
    hmask = (1 << width) - 1
    mixed = history ^ (history >> 11)
    mixed ^= (mixed << 11) & hmask
    product = (0x3FA7D929 * mixed + 0xC928FD8E) & 0xFFFFFFFF
    phase = product & hmask
    syndrome = product >> (32 - bits)
    stratum = _bit_reverse(branch, bits) ^ syndrome
    return (stratum << width) | phase


def sqg_xor_rank_permutation(bits: int) -> torch.Tensor:
    """Carry-mixed SQG rank of every state (a bijection of the 65,536 states)."""
    _check_bits(bits)
    return torch.from_numpy(_xor_rank_np(bits).copy())


@lru_cache(maxsize=None)
def _xor_cheb_t12_bytes(bits: int) -> torch.Tensor:
    return sqg_xor_cheb_t12_rank_lut_bytes().index_select(0, sqg_xor_rank_permutation(bits) >> 4).contiguous()


def sqg_xor_cheb_t12_bytes(bits: int, *, device="cpu") -> torch.Tensor:
    """Production QSRT-E4M3 labels of all L16 states at rate ``bits``."""
    _check_bits(bits)
    return _xor_cheb_t12_bytes(bits).to(device=device).contiguous()


def sqg_k2_eight_stratum_rank_permutation(history_bit: int = 2) -> torch.Tensor:
    """K2 graph labelled through the K3 rank law with a chosen virtual stratum bit."""
    if isinstance(history_bit, bool) or not isinstance(history_bit, int):
        raise TypeError("K2 eight-stratum history bit must be an integer")
    if not 2 <= history_bit < 16:
        raise ValueError("K2 eight-stratum history bit must be in [2, 15]")
    k3 = sqg_rank_permutation(3)
    if history_bit == 2:
        return k3
    t = torch.arange(STATES, dtype=torch.int64)
    swap = ((t >> 2) & 1) ^ ((t >> history_bit) & 1)
    return k3.index_select(0, t ^ (swap << 2) ^ (swap << history_bit)).contiguous()


def sqg_k2_eight_stratum_e4m3_bytes_from_rank_lut(rank_lut: torch.Tensor, *, history_bit: int = 2,
                                                   device="cpu") -> torch.Tensor:
    rank_lut = _validate_rank_lut(rank_lut)
    perm = sqg_k2_eight_stratum_rank_permutation(history_bit)
    return rank_lut.index_select(0, perm).to(device=device).contiguous()


def sqg_codebook_bytes(bits: int, codebook: str, *, rate_axis: str | None = None,
                       device="cpu") -> torch.Tensor:
    """State-indexed E4M3 bytes of a named SQG codebook."""
    if codebook == SQG_XOR_CHEB_T12:
        return sqg_xor_cheb_t12_bytes(bits, device=device)
    if codebook == SQG_NORMAL_E4M3:
        return sqg_e4m3_bytes(bits, "normal", device=device)
    if codebook == SQG_CHEB_NORMAL_E4M3:
        return sqg_cheb_normal_e4m3_bytes(bits).to(device=device).contiguous()
    if codebook == SQG_CHEB:
        if rate_axis not in ("k", "n"):
            raise ValueError("the w2-only K2-Q8H4 profile requires rate_axis 'k' or 'n'")
        staircase = sqg_cheb_normal_rank_e4m3_bytes()
        if bits == 2 and rate_axis == "k":
            return sqg_k2_eight_stratum_e4m3_bytes_from_rank_lut(staircase, history_bit=4, device=device)
        return sqg_e4m3_bytes_from_rank_lut(bits, staircase, device=device).contiguous()
    raise ValueError(f"unsupported SQG codebook: {codebook!r}")


def sqg_codebook(bits: int, codebook: str, *, rate_axis: str | None = None, device="cpu",
                 dtype=torch.float16) -> torch.Tensor:
    if not dtype.is_floating_point:
        raise TypeError("SQG codebook dtype must be floating point")
    raw = sqg_codebook_bytes(bits, codebook, rate_axis=rate_axis, device=device)
    return raw.view(torch.float8_e4m3fn).to(dtype).contiguous()
