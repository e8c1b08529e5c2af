"""QSRT payload closure on the GPU: record packing, unpacking, state closure, decode.

This is the step kquant's encoder wrapper runs on the backend's output
(``kquant/pack/qsrt_encoder.py:1158-1187``, ``:909-1070``): the encoded
``[K/16, N/16, 256]`` states of one Kimi-K3 expert matrix are cut into 24
records of 128 channels along the shared 3072-channel intermediate axis,
each record is packed at its own rate (K2 / K3 / K4) with the native EXL
per-tile word order, and the payload is the records' words in order.  The
closure checks unpack it again and reconstruct the cyclic states.

Names, arguments, errors and the payload layout follow ``kquant/qsrt.py``
(``ModeSpec`` :132-180, R0-R2 :182-211, ``record_contexts`` / ``record_bits`` /
``pair_kinds`` :477-513, ``repack_encoded_records`` :774-803, the descriptor
:866-960, ``pack_qsrt_trellis`` :983-1014, ``unpack_qsrt_trellis_*`` :1017-1104,
``decode_qsrt_exl3_weight`` :1107-1141).  The per-tile packing, unpacking and
closure run on the sm_100a kernels (``kq_pack_trellis``,
``kq_unpack_trellis_states``); records of equal rate share one launch.
"""

from __future__ import annotations

from collections.abc import Sequence
from dataclasses import dataclass
from typing import Literal

import torch

from . import _native
from .codebooks import QSRT_CODEBOOKS, SQG_XOR_CHEB_T12, sqg_codebook

INTERMEDIATE_CHANNELS = 3072
LATENT_CHANNELS = 3584
TILE_CHANNELS = 16
TILE_VALUES = 256
RECORD_CHANNELS = 128
PAIR_CHANNELS = 2 * RECORD_CHANNELS
RECORDS_PER_EXPERT = INTERMEDIATE_CHANNELS // RECORD_CHANNELS
PAIRS_PER_EXPERT = RECORDS_PER_EXPERT // 2
TILES_PER_RECORD_AXIS = RECORD_CHANNELS // TILE_CHANNELS
SCHEMA = "kquant_kimi_k3_qsrt_candidate_v1"
LOGICAL_CANDIDATE_SCHEMAS = (SCHEMA,)
RateAxis = Literal["k", "n"]
MATRIX_RATE_AXIS = {"w1": "n", "w3": "n", "w2": "k"}


@dataclass(frozen=True)
class ModeSpec:
    """Rate-transfer schedule: one K per context, low to high importance; mode_id = K2/K4 exchanges."""

    mode_id: int
    name: str
    context_bits: tuple[int, ...]

    def __post_init__(self) -> None:
        if isinstance(self.mode_id, bool) or not isinstance(self.mode_id, int):
            raise TypeError("mode_id must be an integer")
        if not 0 <= self.mode_id <= 2:
            raise ValueError("QSRT mode_id must be R0, R1, or R2")
        if not self.name:
            raise ValueError("mode name must not be empty")
        bits = self.context_bits
        if not bits or len(bits) % 2:
            raise ValueError("a mode must contain an even, nonzero context count")
        if any(b not in (2, 3, 4) for b in bits):
            raise ValueError("Kimi-K3 QSRT supports only K2, K3, and K4")
        if sum(bits) != 3 * len(bits):
            raise ValueError("a mode must average exactly three trellis bits")
        if INTERMEDIATE_CHANNELS % len(bits) or (INTERMEDIATE_CHANNELS // len(bits)) % RECORD_CHANNELS:
            raise ValueError("each context must contain whole 128-channel records")
        if tuple(sorted(bits)) != bits:
            raise ValueError("context rates must be monotone from K2 through K4")
        per = RECORDS_PER_EXPERT // len(bits)
        if bits.count(2) * per != bits.count(4) * per:
            raise ValueError("K2 and K4 record counts must match")
        if self.mode_id != bits.count(2) * per:
            raise ValueError(f"mode_id must equal the rate-transfer count {bits.count(2) * per}")

    @property
    def context_count(self) -> int:
        return len(self.context_bits)

    @property
    def records_per_context(self) -> int:
        return RECORDS_PER_EXPERT // self.context_count


RATE_TRANSFER_MODES = tuple(
    ModeSpec(r, f"R{r}", (2,) * r + (3,) * (RECORDS_PER_EXPERT - 2 * r) + (4,) * r) for r in range(3))
R0, R1, R2 = RATE_TRANSFER_MODES
_BY_NAME = {m.name: m for m in RATE_TRANSFER_MODES}
_BY_ID = {m.mode_id: m for m in RATE_TRANSFER_MODES}


def resolve_mode(mode) -> ModeSpec:
    if isinstance(mode, ModeSpec):
        return mode
    if isinstance(mode, str):
        try:
            return _BY_NAME[mode.upper()]
        except KeyError as exc:
            raise ValueError(f"unknown QSRT mode: {mode}") from exc
    if isinstance(mode, int) and not isinstance(mode, bool):
        try:
            return _BY_ID[mode]
        except KeyError as exc:
            raise ValueError(f"unknown QSRT mode ID: {mode}") from exc
    raise TypeError("mode must be a ModeSpec, name, or integer ID")


def matrix_rate_axis(matrix: str) -> RateAxis:
    try:
        return MATRIX_RATE_AXIS[matrix]
    except KeyError as exc:
        raise ValueError(f"unknown expert matrix: {matrix}") from exc


def record_contexts(mode) -> tuple[int, ...]:
    """Physical record contexts: lowest and highest context interleaved, moving inward."""
    spec = resolve_mode(mode)
    out: list[int] = []
    for low in range(spec.context_count // 2):
        high = spec.context_count - 1 - low
        for _ in range(spec.records_per_context):
            out.extend((low, high))
    if len(out) != RECORDS_PER_EXPERT:
        raise AssertionError("mode construction did not cover 24 records")
    return tuple(out)


def record_bits(mode) -> tuple[int, ...]:
    spec = resolve_mode(mode)
    return tuple(spec.context_bits[c] for c in record_contexts(spec))


def pair_bits(mode) -> tuple[tuple[int, int], ...]:
    rec = record_bits(mode)
    pairs = tuple(zip(rec[0::2], rec[1::2], strict=True))
    if len(pairs) != PAIRS_PER_EXPERT or any(sum(p) != 6 for p in pairs):
        raise ValueError("every QSRT record pair must have a six-bit rate sum")
    return pairs


def pair_kinds(mode) -> tuple[str, ...]:
    kinds = []
    for p in pair_bits(mode):
        if p == (2, 4):
            kinds.append("P24")
        elif p == (3, 3):
            kinds.append("P33")
        else:
            raise ValueError(f"unsupported QSRT pair schedule: {p}")
    return tuple(kinds)


@dataclass(frozen=True)
class QSRTTrellisDescriptor:
    """TP-independent description of one complete packed expert matrix."""

    mode_id: int
    rate_axis: RateAxis
    k_tiles: int
    n_tiles: int
    schema: str = SCHEMA
    intermediate_channels: int = INTERMEDIATE_CHANNELS
    record_channels: int = RECORD_CHANNELS

    def __post_init__(self) -> None:
        if self.schema not in LOGICAL_CANDIDATE_SCHEMAS:
            raise ValueError(f"unsupported QSRT schema: {self.schema}")
        if self.intermediate_channels != INTERMEDIATE_CHANNELS:
            raise ValueError("Kimi-K3 QSRT requires a 3072-channel intermediate axis")
        if self.record_channels != RECORD_CHANNELS:
            raise ValueError("Kimi-K3 QSRT requires 128-channel records")
        resolve_mode(self.mode_id)
        if self.rate_axis not in ("k", "n"):
            raise ValueError("rate_axis must be 'k' or 'n'")
        if self.k_tiles <= 0 or self.n_tiles <= 0:
            raise ValueError("tile dimensions must be positive")
        rate_tiles = self.k_tiles if self.rate_axis == "k" else self.n_tiles
        if rate_tiles * TILE_CHANNELS != INTERMEDIATE_CHANNELS:
            raise ValueError("rate axis must contain exactly 3072 channels")
        if self.orthogonal_tiles * TILE_CHANNELS != LATENT_CHANNELS:
            raise ValueError("orthogonal axis must contain exactly 3584 channels")

    @property
    def mode(self) -> ModeSpec:
        return resolve_mode(self.mode_id)

    @property
    def orthogonal_tiles(self) -> int:
        return self.n_tiles if self.rate_axis == "k" else self.k_tiles

    @property
    def tiles_per_record(self) -> int:
        return TILES_PER_RECORD_AXIS * self.orthogonal_tiles

    @property
    def words_per_pair(self) -> int:
        return self.tiles_per_record * TILE_CHANNELS * 6

    @property
    def payload_words(self) -> int:
        return PAIRS_PER_EXPERT * self.words_per_pair

    @property
    def payload_bytes(self) -> int:
        return self.payload_words * torch.int16.itemsize

    @property
    def weight_count(self) -> int:
        return self.k_tiles * self.n_tiles * TILE_VALUES

    def to_manifest(self) -> dict:
        return {"schema": self.schema, "mode_id": self.mode_id, "mode": self.mode.name, "rate_axis": self.rate_axis,
                "k_tiles": self.k_tiles, "n_tiles": self.n_tiles,
                "intermediate_channels": self.intermediate_channels, "record_channels": self.record_channels,
                "pair_channels": PAIR_CHANNELS, "record_bits": list(record_bits(self.mode)),
                "pair_kinds": list(pair_kinds(self.mode)), "words_per_pair": self.words_per_pair,
                "payload_words": self.payload_words, "payload_bytes": self.payload_bytes}


@dataclass(frozen=True)
class PackedQSRTTrellis:
    descriptor: QSRTTrellisDescriptor
    payload: torch.Tensor

    def validate(self) -> None:
        if self.payload.dtype != torch.int16:
            raise TypeError("QSRT trellis payload must use torch.int16")
        if self.payload.ndim != 1:
            raise ValueError("QSRT trellis payload must be one-dimensional")
        if self.payload.numel() != self.descriptor.payload_words:
            raise ValueError("QSRT trellis payload length does not match its descriptor")


def _validate_encoded_shape(encoded: torch.Tensor, rate_axis: RateAxis) -> None:
    if encoded.ndim != 3 or encoded.shape[-1] != TILE_VALUES:
        raise ValueError("encoded states must have shape [K/16, N/16, 256]")
    if encoded.dtype == torch.bool or encoded.is_floating_point():
        raise TypeError("encoded states must use an integer dtype")
    if rate_axis not in ("k", "n"):
        raise ValueError("rate_axis must be 'k' or 'n'")
    rate_tiles = encoded.shape[0] if rate_axis == "k" else encoded.shape[1]
    if rate_tiles * TILE_CHANNELS != INTERMEDIATE_CHANNELS:
        raise ValueError("encoded rate axis must contain exactly 3072 channels")


def _validate_permutation(p: torch.Tensor, size: int, name: str) -> None:
    if p.ndim != 1 or p.numel() != size:
        raise ValueError(f"{name} must contain {size} entries")
    if p.dtype == torch.bool or p.is_floating_point():
        raise TypeError(f"{name} must use an integer dtype")
    if not torch.equal(torch.sort(p.detach().cpu().to(torch.long)).values, torch.arange(size)):
        raise ValueError(f"{name} must be a permutation of 0..{size - 1}")


def _records_view(encoded: torch.Tensor, rate_axis: RateAxis) -> torch.Tensor:
    """[24, tiles_per_record, 256] view-order of the records (a copy for the n axis)."""
    if rate_axis == "k":
        return encoded.reshape(RECORDS_PER_EXPERT, -1, TILE_VALUES)
    k_tiles = encoded.shape[0]
    return (encoded.reshape(k_tiles, RECORDS_PER_EXPERT, TILES_PER_RECORD_AXIS, TILE_VALUES)
            .permute(1, 0, 2, 3).reshape(RECORDS_PER_EXPERT, -1, TILE_VALUES))


def _from_records(records: torch.Tensor, shape, rate_axis: RateAxis) -> torch.Tensor:
    if rate_axis == "k":
        return records.reshape(shape).contiguous()
    k_tiles, n_tiles, _ = shape
    return (records.reshape(RECORDS_PER_EXPERT, k_tiles, TILES_PER_RECORD_AXIS, TILE_VALUES)
            .permute(1, 0, 2, 3).reshape(shape).contiguous())


def repack_encoded_records(encoded: torch.Tensor, record_order: torch.Tensor, rate_axis: RateAxis) -> torch.Tensor:
    """Reorder whole 128-channel records of [K/16, N/16, 256] states (destination -> source record)."""
    _validate_encoded_shape(encoded, rate_axis)
    _validate_permutation(record_order, RECORDS_PER_EXPERT, "record_order")
    order = record_order.to(device=encoded.device, dtype=torch.long)
    recs = _records_view(encoded, rate_axis).index_select(0, order)
    return _from_records(recs, encoded.shape, rate_axis)


def _record_groups(bits: tuple[int, ...]):
    return {b: [r for r, x in enumerate(bits) if x == b] for b in sorted(set(bits))}


def _pack_records(records: torch.Tensor, bits: tuple[int, ...]) -> torch.Tensor:
    """[24, T, 256] int16 states -> payload (records in order, each T*16*K words)."""
    T = records.shape[1]
    packed_by_record: dict[int, torch.Tensor] = {}
    for b, recs in _record_groups(bits).items():
        idx = torch.tensor(recs, dtype=torch.long, device=records.device)
        words = _native.pack_trellis(records.index_select(0, idx).contiguous(), b)   # [R, T, 16b]
        for i, r in enumerate(recs):
            packed_by_record[r] = words[i].reshape(-1)
    return torch.cat([packed_by_record[r] for r in range(len(bits))]).contiguous()


def _unpack_records(payload: torch.Tensor, bits: tuple[int, ...], T: int) -> torch.Tensor:
    """payload -> [24, T, 256] int16 cyclic states."""
    offsets, cur = [], 0
    for b in bits:
        offsets.append(cur)
        cur += T * TILE_CHANNELS * b
    if cur != payload.numel():
        raise ValueError("QSRT trellis payload has trailing data")
    out = torch.empty((len(bits), T, TILE_VALUES), dtype=torch.int16, device=payload.device)
    for b, recs in _record_groups(bits).items():
        words = torch.stack([payload.narrow(0, offsets[r], T * 16 * b).reshape(T, 16 * b) for r in recs])
        states = _native.unpack_trellis_states(words.contiguous(), b)
        out[torch.tensor(recs, dtype=torch.long, device=payload.device)] = states
    return out


def pack_qsrt_trellis(encoded: torch.Tensor, mode, *, rate_axis: RateAxis, schema: str = SCHEMA,
                      validate_states: bool = True) -> PackedQSRTTrellis:
    """Pack a complete matrix into its record payload; optionally prove the states close."""
    _validate_encoded_shape(encoded, rate_axis)
    spec = resolve_mode(mode)
    desc = QSRTTrellisDescriptor(mode_id=spec.mode_id, rate_axis=rate_axis, k_tiles=encoded.shape[0],
                                 n_tiles=encoded.shape[1], schema=schema)
    states = encoded.to(torch.int16)
    if not states.is_cuda:
        raise ValueError("pack_qsrt_trellis requires CUDA states (kquant_b200 has no CPU path)")
    bits = record_bits(spec)
    records = _records_view(states.contiguous(), rate_axis).contiguous()
    payload = _pack_records(records, bits)
    if validate_states and not torch.equal(_unpack_records(payload, bits, records.shape[1]), records):
        raise ValueError("encoded input is not a closed cyclic trellis path")
    packed = PackedQSRTTrellis(desc, payload)
    packed.validate()
    return packed


def unpack_qsrt_trellis_states(packed: PackedQSRTTrellis) -> torch.Tensor:
    """Payload -> physical-order 16-bit cyclic states [K/16, N/16, 256]."""
    packed.validate()
    d = packed.descriptor
    recs = _unpack_records(packed.payload, record_bits(d.mode), d.tiles_per_record)
    return _from_records(recs, (d.k_tiles, d.n_tiles, TILE_VALUES), d.rate_axis)


def unpack_qsrt_trellis_edges(packed: PackedQSRTTrellis) -> torch.Tensor:
    """Payload -> physical-order K-bit edge symbols (the low K bits of each state)."""
    d = packed.descriptor
    states = unpack_qsrt_trellis_states(packed)
    bits = torch.tensor(record_bits(d.mode), device=states.device).repeat_interleave(TILES_PER_RECORD_AXIS)
    masks = (1 << bits) - 1
    masks = masks[:, None, None] if d.rate_axis == "k" else masks[None, :, None]
    return (states.to(torch.int32) & masks).to(torch.int16)


def decode_qsrt_exl3_weight(packed: PackedQSRTTrellis, suh: torch.Tensor, svh: torch.Tensor, *,
                            codebook: str = SQG_XOR_CHEB_T12) -> torch.Tensor:
    """Decode a complete payload to the physical EXL-oriented [K, N] weight."""
    from .exl3_encoder_backend import tensor_core_perm_i
    packed.validate()
    if codebook not in QSRT_CODEBOOKS:
        raise ValueError(f"unsupported QSRT codebook: {codebook}")
    d = packed.descriptor
    k, n = d.k_tiles * TILE_CHANNELS, d.n_tiles * TILE_CHANNELS
    for name, v, size in (("suh", suh, k), ("svh", svh, n)):
        if v.ndim != 1 or v.numel() != size:
            raise ValueError(f"{name} must have {size} entries")
    states = unpack_qsrt_trellis_states(packed).to(torch.int64) & 0xFFFF
    dev = states.device
    vals = torch.empty(states.shape, dtype=torch.float32, device=dev)
    rec = torch.tensor(record_bits(d.mode), device=dev).repeat_interleave(TILES_PER_RECORD_AXIS)
    for b in sorted(set(record_bits(d.mode))):
        lab = sqg_codebook(b, codebook, rate_axis=d.rate_axis, device=dev).float()
        sel = rec == b
        if d.rate_axis == "k":
            vals[sel] = lab[states[sel]]
        else:
            vals[:, sel] = lab[states[:, sel]]
    vals = vals[..., tensor_core_perm_i(dev)]
    w = vals.reshape(d.k_tiles, d.n_tiles, 16, 16).permute(0, 2, 1, 3).reshape(k, n)
    return _native.reconstruct_rotated(w.contiguous(), suh.to(device=dev), svh.to(device=dev))
