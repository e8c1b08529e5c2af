"""Golden QSRT payload hashes and decode samples from the REFERENCE kquant.qsrt (run here, CPU).

Usage: python tests/golden/make_qsrt_fixtures.py /path/to/reference  -> tests/golden/qsrt_payloads.json
"""
import hashlib
import json
import sys
from pathlib import Path

import torch

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parents[1]))
from tests.golden.qsrt_cases import CASES, SHAPES, legal_states, scales  # noqa: E402


def main():
    if len(sys.argv) < 2:
        raise SystemExit("usage: make_qsrt_fixtures.py REFERENCE_ROOT")
    sys.path.insert(0, sys.argv[1])
    from kquant import qsrt
    out = {}
    for mode, axis in CASES:
        shape = SHAPES[axis]
        states = legal_states(shape, qsrt.record_bits(mode), axis, 300 + 10 * mode + (axis == "n"))
        packed = qsrt.pack_qsrt_trellis(states, mode, rate_axis=axis)
        suh, svh = scales(shape[0] * 16, shape[1] * 16, 7 + mode)
        w = qsrt.decode_qsrt_exl3_weight(packed, suh, svh)
        flat = w.flatten()
        out[f"R{mode}_{axis}"] = {
            "payload_sha256": hashlib.sha256(packed.payload.numpy().tobytes()).hexdigest(),
            "payload_words": packed.payload.numel(),
            "manifest": packed.descriptor.to_manifest(),
            "decode_sample_stride": 9973,
            "decode_sample": flat[::9973].tolist(),
            "decode_sum": float(w.double().sum()),
        }
        print(mode, axis, out[f"R{mode}_{axis}"]["payload_sha256"][:16])
    (HERE / "qsrt_payloads.json").write_text(json.dumps(out))


if __name__ == "__main__":
    main()
