"""Parity against the reference backend run on a B200 (fixtures from tests/golden/make_ref_cuda_fixtures.py).

The north-star contract: on identical rotated inputs and Hessians the trellis
codes are bit-exact per tile; end to end the proxy error is within 1 % of the
reference's and the reconstruction within 1e-3 max-abs.

* ``test_qsrt_codes_on_identical_rotated_inputs``: this backend's rotated W
  and L must hash to the digests recorded when the fixture was made, and the
  reference's own LDLQ (with the reference's own Viterbi kernel) ran on
  exactly those tensors.  The codes this backend produces from them must hash
  to the reference's codes: 100 % of the states, every tile.
* ``test_qsrt_end_to_end``: against the reference's complete
  ``quantize_qsrt`` (its own preparation included).
* ``test_qsrt_batch_*`` / ``test_uniform_batch``: kquant's production batch
  calls (``quantize_qsrt_batch`` R0/R1/R2 on both rate axes, the candidate
  reuse engines; ``quantize_uniform_batch``) against the reference's.
"""
import json
from pathlib import Path

import numpy as np
import pytest
import torch

from kquant_b200 import exl3_encoder_backend as be
from kquant_b200.ldlq import make_shared_h
from tests.golden import ref_cuda_cases as C

pytestmark = pytest.mark.gpu
FIXTURES = Path(__file__).resolve().parent / "golden" / "ref_cuda_fixtures.json"


def _fixtures():
    if not FIXTURES.exists():
        pytest.fail(f"{FIXTURES.name} missing: run tests/golden/make_ref_cuda_fixtures.py on a GPU host")
    return json.loads(FIXTURES.read_text())["cases"]


def _first_diff(rows_a, rows_b):
    for i, (a, b) in enumerate(zip(rows_a, rows_b)):
        if a != b:
            return i
    return None


_RUNS = {}


def _run_qsrt(name, device):
    if name not in _RUNS:
        w, h, args = C.qsrt_inputs(name, device)
        with C.Capture(be) as cap:
            wq, proxy, out = be.quantize_qsrt(w.clone(), make_shared_h(w.shape[0], device, h), args, True)
        torch.cuda.synchronize()
        states = be._native.unpack_trellis_states(out["trellis"], args["K"]).cpu().to(torch.int16)
        _RUNS[name] = (cap.inputs, wq, proxy, out, args, states)
    return _RUNS[name]


@pytest.mark.parametrize("name", sorted(C.QSRT_CASES))
def test_qsrt_codes_on_identical_rotated_inputs(cuda_device, name):
    fx = _fixtures()[name]
    (w_r, L), _, _, _, _, states = _run_qsrt(name, cuda_device)
    assert C.digest(w_r) == fx["kq_prep"]["w_r"], "rotated W differs from the one the reference LDLQ ran on"
    assert C.digest(L) == fx["kq_prep"]["L"], "L differs from the one the reference LDLQ ran on"
    rows = C.row_digests(states)
    first = _first_diff(rows[::-1], fx["ref_on_kq_prep"]["state_rows"][::-1])
    assert C.digest(states) == fx["ref_on_kq_prep"]["states"], (
        f"codes differ from the reference LDLQ; first differing tile row (from the bottom): "
        f"{None if first is None else len(rows) - 1 - first}")


@pytest.mark.parametrize("name", sorted(C.QSRT_CASES))
def test_qsrt_end_to_end(cuda_device, name):
    fx = _fixtures()[name]
    ref = fx["ref"]
    _, wq, proxy, out, args, states = _run_qsrt(name, cuda_device)
    assert abs(proxy - ref["proxy"]) / ref["proxy"] < 0.01
    idx = C.sample_index(wq.numel())
    got = wq.flatten()[idx.to(wq.device)].cpu().numpy()
    assert np.abs(got - np.asarray(ref["weight_q_sample"], dtype=np.float32)).max() <= 1e-3
    if all(fx["prep_equal"].values()):
        # the preparation is bit-identical to the reference's, so the whole encode is
        assert C.digest(states) == ref["states"]
        assert C.digest(out["suh"]) == ref["suh"] and C.digest(out["svh"]) == ref["svh"]
        assert args["g_scale"] == ref["g_scale"]


def _check_candidate(got, ref, prep_equal):
    assert abs(got["proxy"] - ref["proxy"]) / ref["proxy"] < 0.01
    assert abs(got["g_scale"] - ref["g_scale"]) / ref["g_scale"] < 1e-3
    idx = C.sample_index(got["weight_q"].numel())
    sample = got["weight_q"].flatten()[idx.to(got["weight_q"].device)].cpu().numpy()
    assert np.abs(sample - np.asarray(ref["weight_q_sample"], dtype=np.float32)).max() <= 1e-3
    if prep_equal:
        assert C.digest(got["encoded"].to(torch.int16)) == ref["states"]


@pytest.mark.parametrize("name", sorted(C.BATCH_CASES))
def test_qsrt_batch_against_reference(cuda_device, name):
    fx = _fixtures()[name]
    ws, hs, groups = C.batch_inputs(name, cuda_device)
    res = be.quantize_qsrt_batch([w.clone() for w in ws], [make_shared_h(w.shape[0], cuda_device, h)
                                                           for w, h in zip(ws, hs)], groups)
    torch.cuda.synchronize()
    for s, cands in enumerate(res):
        for c, got in enumerate(cands):
            ref = fx["sources"][s][c]
            scales_equal = C.digest(got["suh"]) == ref["suh"] and C.digest(got["svh"]) == ref["svh"] \
                and got["g_scale"] == ref["g_scale"]
            _check_candidate(got, ref, scales_equal)


@pytest.mark.parametrize("name", sorted(C.UNIFORM_CASES))
def test_uniform_batch_against_reference(cuda_device, name):
    fx = _fixtures()[name]
    ws, h, args = C.uniform_inputs(name, cuda_device)
    shared = make_shared_h(ws[0].shape[0], cuda_device, h)
    res = be.quantize_uniform_batch([w.clone() for w in ws], [shared, shared], args)
    torch.cuda.synchronize()
    for t, (proxy, out) in enumerate(res):
        ref = fx["members"][t]
        assert abs(proxy - ref["proxy"]) / ref["proxy"] < 0.01
        states = be._native.unpack_trellis_states(out["trellis"], args[t]["K"]).cpu().to(torch.int16)
        if C.digest(out["suh"]) == ref["suh"] and C.digest(out["svh"]) == ref["svh"] \
                and args[t]["g_scale"] == ref["g_scale"]:
            assert C.digest(states) == ref["states"]
