"""Pin the CPU oracle and the codebook tables to the reference's own golden vectors (CPU only)."""
import hashlib

import numpy as np
import pytest
import torch

from kquant_b200 import codebooks as cb

# Reference golden values: tests/test_sqg_e4m3.py:32-37 and tests/test_qsrt.py:213-231.
SQG_XOR_CHEB_T12_SHA256 = {
    "t12": "cca11fe5744c9c93a34f4217f342fbc0f74ecc8a007c076582424a505fc9da5e",
    2: "62027916386245a84c86156a0a08b6cf07e41548871af0e56fb40780558f6293",
    3: "afe7b3633e7d243b00b379b18ec4dca573722b3727cafef47fcb6470d7e7e6c9",
    4: "5a9620f0c4d8f0a60d0b6fbea921dcecbd193e6febf31043aaa6403c20389c2f",
}
PACK_PREFIX = {
    2: [6939] * 6,
    3: [30469, 1337, 1337, 14711, 14711, 30469],
    4: [17767, 291, -12817, -30293, 17767, 291],
}


def _sha(t: torch.Tensor) -> str:
    return hashlib.sha256(t.contiguous().numpy().tobytes()).hexdigest()


def test_t12_rank_table_sha256():
    assert _sha(cb.sqg_xor_cheb_t12_rank_lut_bytes()) == SQG_XOR_CHEB_T12_SHA256["t12"]


@pytest.mark.parametrize("bits", [2, 3, 4])
def test_t12_labels_sha256(bits):
    labels = cb.sqg_xor_cheb_t12_bytes(bits)
    assert _sha(labels) == SQG_XOR_CHEB_T12_SHA256[bits]
    ranks = cb.sqg_xor_rank_permutation(bits)
    assert torch.equal(torch.sort(ranks).values, torch.arange(1 << 16))


@pytest.mark.parametrize("bits", [2, 3, 4])
def test_oracle_pack_golden_prefix(oracle_mod, bits):
    states = (np.arange(256) % (1 << bits)).astype(np.int16)[None]
    packed = oracle_mod.pack_trellis(states, bits)
    assert packed.shape == (1, 16 * bits)
    assert packed[0, :6].tolist() == PACK_PREFIX[bits]
    assert np.array_equal(oracle_mod.unpack_trellis(packed, bits), states)


@pytest.mark.parametrize("bits", [1, 2, 3, 4, 5, 8])
def test_oracle_pack_roundtrip_low_bits(oracle_mod, bits):
    rng = np.random.default_rng(100 + bits)
    states = rng.integers(-32768, 32768, (7, 256)).astype(np.int16)
    edges = oracle_mod.unpack_trellis(oracle_mod.pack_trellis(states, bits), bits)
    assert np.array_equal(edges.astype(np.int32), states.astype(np.int32) & ((1 << bits) - 1))


@pytest.mark.parametrize("bits", [2, 3, 4])
def test_oracle_states_match_scalar_recurrence(oracle_mod, bits):
    rng = np.random.default_rng(175 + bits)
    edges = rng.integers(0, 1 << bits, (15, 256)).astype(np.int16)
    state = np.zeros(15, np.int64)
    for col in range(256 - ((16 + bits - 1) // bits), 256):
        state = ((state << bits) | edges[:, col]) & 0xFFFF
    expected = []
    for col in range(256):
        state = ((state << bits) | edges[:, col]) & 0xFFFF
        expected.append(state.copy())
    expected = np.stack(expected, 1).astype(np.uint16).view(np.int16)
    assert np.array_equal(oracle_mod.reconstruct_states(edges, bits), expected)


@pytest.mark.parametrize("bits", [2, 3, 4])
def test_oracle_sqg_labels_are_exact_e4m3_widening(oracle_mod, bits):
    lut = cb.sqg_xor_cheb_t12_bytes(bits)
    widened = lut.view(torch.float8_e4m3fn).to(torch.float16).view(torch.int16).numpy().view(np.uint16)
    assert np.array_equal(oracle_mod.labels(oracle_mod.CB_SQG, lut.numpy()), widened)


def test_oracle_viterbi_closes_cyclic_paths(oracle_mod):
    O = oracle_mod
    rng = np.random.default_rng(3)
    tiles = rng.standard_normal((2, 256)).astype(np.float32)
    for K in (2, 3, 4):
        lab = O.labels(O.CB_SQG, cb.sqg_xor_cheb_t12_bytes(K).numpy())
        idx, val, rc = O.viterbi(K, lab, tiles, 128, threads=2)
        assert rc == 0
        edges = (idx & ((1 << K) - 1)).astype(np.int16)
        assert np.array_equal(O.reconstruct_states(edges, K).view(np.uint16), idx)
        assert np.array_equal(val, lab[idx].view(np.float16).astype(np.float32))


@pytest.mark.parametrize("K", [1, 5, 8])
def test_oracle_wide_rates_give_closed_cyclic_paths(oracle_mod, K):
    """K outside 2..4 (the reference template's other rates): every encoded tile is a closed cyclic
    trellis path, state_i = ((state_{i-1} << K) | edge_i) & 0xFFFF, and values are its labels."""
    O = oracle_mod
    lab = O.labels(O.CB_MCG)
    tiles = np.random.default_rng(K).standard_normal((2, 256)).astype(np.float32)
    idx, val, rc = O.viterbi(K, lab, tiles, 32)
    assert rc == 0
    edges = (idx & ((1 << K) - 1)).astype(np.int16)
    assert np.array_equal(O.reconstruct_states(edges, K).view(np.uint16), idx)
    assert np.array_equal(val, lab[idx].view(np.float16).astype(np.float32))
