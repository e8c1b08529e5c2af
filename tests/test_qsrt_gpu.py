"""QSRT payload closure on the GPU against the reference kquant.qsrt fixtures."""
import hashlib
import json
from pathlib import Path

import pytest
import torch

from kquant_b200 import qsrt
from tests.golden.qsrt_cases import CASES, SHAPES, legal_states, scales

pytestmark = pytest.mark.gpu
GOLD = json.loads((Path(__file__).resolve().parent / "golden" / "qsrt_payloads.json").read_text())


@pytest.mark.parametrize("mode,axis", CASES)
def test_payload_bytes_and_decode_match_reference(cuda_device, mode, axis):
    gold = GOLD[f"R{mode}_{axis}"]
    shape = SHAPES[axis]
    states = legal_states(shape, qsrt.record_bits(mode), axis, 300 + 10 * mode + (axis == "n")).to(cuda_device)
    packed = qsrt.pack_qsrt_trellis(states, mode, rate_axis=axis)
    assert packed.descriptor.to_manifest() == gold["manifest"]
    assert hashlib.sha256(packed.payload.cpu().numpy().tobytes()).hexdigest() == gold["payload_sha256"]
    assert torch.equal(qsrt.unpack_qsrt_trellis_states(packed), states)
    edges = qsrt.unpack_qsrt_trellis_edges(packed)
    bits = torch.tensor(qsrt.record_bits(mode), device=cuda_device).repeat_interleave(8)
    masks = (1 << bits) - 1
    masks = masks[:, None, None] if axis == "k" else masks[None, :, None]
    assert torch.equal(edges.to(torch.int32), states.to(torch.int32) & masks)
    suh, svh = scales(shape[0] * 16, shape[1] * 16, 7 + mode)
    w = qsrt.decode_qsrt_exl3_weight(packed, suh.to(cuda_device), svh.to(cuda_device))
    sample = w.flatten()[::gold["decode_sample_stride"]].cpu()
    assert torch.allclose(sample, torch.tensor(gold["decode_sample"]), atol=1e-4, rtol=1e-5)


def test_rejects_noncyclic_states_and_repacks_records(cuda_device):
    bad = torch.zeros(SHAPES["k"], dtype=torch.int16, device=cuda_device)
    bad[..., 0] = 1
    with pytest.raises(ValueError, match="closed cyclic trellis path"):
        qsrt.pack_qsrt_trellis(bad, 2, rate_axis="k")
    states = legal_states(SHAPES["n"], qsrt.record_bits(0), "n", 5).to(cuda_device)
    order = torch.randperm(24)
    moved = qsrt.repack_encoded_records(states, order, "n")
    for dst, src in enumerate(order.tolist()):
        assert torch.equal(moved[:, 8 * dst:8 * dst + 8], states[:, 8 * src:8 * src + 8])
