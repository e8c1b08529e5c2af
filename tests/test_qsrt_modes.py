"""QSRT mode tables and descriptor arithmetic (CPU), against the reference's published values."""
import pytest

from kquant_b200 import qsrt


def test_rate_transfer_modes():
    assert qsrt.record_bits(0) == (3,) * 24
    assert qsrt.pair_kinds("R0") == ("P33",) * 12
    assert qsrt.record_bits(1)[:2] == (2, 4) and qsrt.pair_kinds(1)[0] == "P24"
    assert qsrt.pair_kinds(2)[:2] == ("P24", "P24") and qsrt.pair_kinds(2)[2:] == ("P33",) * 10
    assert all(sum(p) == 6 for p in qsrt.pair_bits(2))
    with pytest.raises(ValueError):
        qsrt.resolve_mode(3)
    with pytest.raises(ValueError, match="monotone"):
        qsrt.ModeSpec(1, "bad", (4,) + (3,) * 22 + (2,))


def test_descriptor_sizes():
    d = qsrt.QSRTTrellisDescriptor(mode_id=0, rate_axis="k", k_tiles=192, n_tiles=224)
    assert d.payload_words == 192 * 224 * 256 * 3 // 16
    assert d.words_per_pair * qsrt.PAIRS_PER_EXPERT == d.payload_words
    with pytest.raises(ValueError, match="3072"):
        qsrt.QSRTTrellisDescriptor(mode_id=0, rate_axis="n", k_tiles=192, n_tiles=224)
    assert qsrt.matrix_rate_axis("w2") == "k" and qsrt.matrix_rate_axis("w1") == "n"
