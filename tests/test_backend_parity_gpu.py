"""End-to-end parity of the backend against fixtures made by the reference backend itself.

tests/golden/make_backend_fixtures.py ran the reference's exl3_encoder_backend
(CPU, C-oracle tile quantizer) on these seeded inputs.  Here the same inputs go
through kquant_b200 on the GPU, with the sign draws taken from the same CPU
generator.  Criteria from the north star: proxy error within 1% relative, and,
where the rotated inputs agree (identical fp16 scales), bit-exact codes and
reconstruction within 1e-3 max-abs.  A case whose fp32 host maths rounds one
fp16 scale differently (CPU vs GPU summation order) legitimately diverges in the
codes downstream of it; it is still held to the proxy criterion.
"""
import json
from pathlib import Path

import numpy as np
import pytest
import torch

from kquant_b200 import exl3_encoder_backend as be
from kquant_b200.ldlq import make_shared_h
from tests.golden.backend_cases import CASES, UNIFORM_CASES, make_inputs, make_uniform_inputs

pytestmark = pytest.mark.gpu
GOLDEN = Path(__file__).resolve().parent / "golden"


@pytest.fixture
def cpu_sign_draws(monkeypatch):
    real = torch.randn

    def randn(*size, device=None, **kw):
        out = real(*size, **kw)
        return out.to(device) if device is not None else out

    monkeypatch.setattr(torch, "randn", randn)


@pytest.mark.parametrize("name", sorted(CASES))
def test_backend_matches_reference_fixture(cuda_device, cpu_sign_draws, name):
    ref = np.load(GOLDEN / f"backend_{name}.npz")
    w, h, args = make_inputs(CASES[name], cuda_device)
    wq, proxy, out = be.quantize_qsrt(w.clone(), make_shared_h(w.shape[0], cuda_device, h), args, True)
    torch.cuda.synchronize()
    ref_proxy = float(ref["proxy"])
    states = be._native.unpack_trellis_states(out["trellis"], args["K"]).cpu().numpy()
    stats = {
        "proxy": proxy, "ref_proxy": ref_proxy, "proxy_rel": abs(proxy - ref_proxy) / ref_proxy,
        "g_scale": args["g_scale"], "ref_g_scale": float(ref["g_scale"]),
        "suh_equal": float((out["suh"].cpu().numpy() == ref["suh"]).mean()),
        "svh_equal": float((out["svh"].cpu().numpy() == ref["svh"]).mean()),
        "states_equal": float((states == ref["states"]).mean()),
        "recon_maxabs": float(np.abs(wq.cpu().numpy() - ref["weight_q"]).max()),
        "recon_rel": float(np.linalg.norm(wq.cpu().numpy() - ref["weight_q"]) / np.linalg.norm(ref["weight_q"])),
    }
    print(name, json.dumps(stats))
    assert stats["proxy_rel"] < 0.01
    assert abs(stats["g_scale"] - stats["ref_g_scale"]) / stats["ref_g_scale"] < 1e-3
    assert stats["suh_equal"] > 0.99 and stats["svh_equal"] > 0.99
    if stats["suh_equal"] == 1.0 and stats["svh_equal"] == 1.0:
        # identical rotated inputs: codes bit-exact and reconstruction within 1e-3
        assert stats["states_equal"] == 1.0
        assert stats["recon_maxabs"] < 1e-3


@pytest.mark.parametrize("name", sorted(UNIFORM_CASES))
def test_uniform_batch_matches_reference_fixture(cuda_device, cpu_sign_draws, name):
    """quantize_uniform_batch (the LDLQ chain engine) against the reference's quantize_uniform_batch."""
    ref = np.load(GOLDEN / f"backend_{name}.npz")
    ws, hs, args = make_uniform_inputs(UNIFORM_CASES[name], cuda_device)
    shared = make_shared_h(ws[0].shape[0], cuda_device, hs[0])
    H_datas = [shared, shared] if hs[1] is hs[0] else [shared, make_shared_h(ws[1].shape[0], cuda_device, hs[1])]
    res = be.quantize_uniform_batch([w.clone() for w in ws], H_datas, args)
    torch.cuda.synchronize()
    for t, (proxy, out) in enumerate(res):
        ref_proxy = float(ref[f"proxy{t}"])
        states = be._native.unpack_trellis_states(out["trellis"], args[t]["K"]).cpu().numpy()
        stats = {
            "proxy_rel": abs(proxy - ref_proxy) / ref_proxy,
            "g_scale_rel": abs(args[t]["g_scale"] - float(ref[f"g_scale{t}"])) / float(ref[f"g_scale{t}"]),
            "suh_equal": float((out["suh"].cpu().numpy() == ref[f"suh{t}"]).mean()),
            "svh_equal": float((out["svh"].cpu().numpy() == ref[f"svh{t}"]).mean()),
            "states_equal": float((states == ref[f"states{t}"]).mean()),
        }
        print(name, t, json.dumps(stats))
        assert stats["proxy_rel"] < 0.01
        assert stats["g_scale_rel"] < 1e-4
        # The global scale comes from a parabola through fp32 MSE sums, summed in a
        # different order on the CPU (fixture) than on the GPU; on a flat MSE curve
        # (uniform_distinct_k4 member 0: 2e-5 relative) that flips the fp16 rounding
        # of a few percent of the suh = su / g entries, and the codes downstream of them.
        # A global scale a few ulp off (uniform_distinct_k4 member 1: 4e-7) changes
        # W * g in the last bits, and the LDLQ feedback carries the resulting code
        # differences up the matrix; codes are bit-exact when all scales agree exactly.
        assert stats["suh_equal"] > 0.9 and stats["svh_equal"] > 0.9
        assert stats["states_equal"] > 0.8
        if stats["suh_equal"] == 1.0 and stats["svh_equal"] == 1.0 and stats["g_scale_rel"] == 0.0:
            assert stats["states_equal"] == 1.0
