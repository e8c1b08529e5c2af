"""Record fixtures from the REFERENCE backend running on a CUDA GPU (test infrastructure).

The reference's ``kquant/exl3_encoder_backend.py`` is loaded with its own loader
(``kquant.exl3_loader.load_qsrt_encoder``) and its own SQG quantizer hook
(``kquant.sqg_quantizer.install_sqg_quantizer``).  The hook's CUDA extension is
the reference's kernel compiled from its sources into ``oracle/_ref`` (the
reference's JIT loader is replaced by that prebuilt module).  Only the
un-vendored ExLlamaV3 helpers are stubbed, as the decoder contract defines
them: a Sylvester Hadamard normalised 1/sqrt(n) (kquant/exl3_reference.py:195-212)
and ``pack_trellis`` = ``kquant.qsrt.pack_trellis_edges``.

For every case of ``tests/golden/ref_cuda_cases.py`` the script records, as
digests and scalars:

* ``ref``: the reference's own end-to-end result (its rotated W and L at the
  LDLQ call, fp16 scales, g_scale, states, proxy, a sample of the
  reconstruction);
* ``kq_prep``: the digests of this backend's rotated W and L for the same
  inputs (so a test can prove it feeds identical inputs);
* ``ref_on_kq_prep``: the reference's LDLQ run on exactly this backend's
  rotated W and L (codes that this backend must reproduce bit for bit).

Usage (on a GPU host, the reference package importable from KQ_REFERENCE_ROOT):
    KQ_REFERENCE_ROOT=baseline/_ref python tests/golden/make_ref_cuda_fixtures.py OUT.json [case ...]
"""
from __future__ import annotations

import json
import os
import sys
import tempfile
import types
from pathlib import Path

import torch

HERE = Path(__file__).resolve().parent
ROOT = HERE.parents[1]
sys.path.insert(0, str(ROOT))

from tests.golden import ref_cuda_cases as C  # noqa: E402


def load_reference_backend(ref_root: Path):
    sys.path.insert(0, str(ref_root))
    from kquant import qsrt, sqg_quantizer
    from kquant.exl3_loader import load_qsrt_encoder
    from oracle import build_ref

    def had(n, device, dtype, scale):
        h = torch.ones((1, 1), dtype=torch.float64)
        while h.shape[0] < n:
            h = torch.cat((torch.cat((h, h), 1), torch.cat((h, -h), 1)), 0)
        return (h * scale).to(device=device, dtype=dtype)

    stubs = {
        "exllamav3.ext": types.SimpleNamespace(exllamav3_ext=types.SimpleNamespace()),
        "exllamav3.util.hadamard": types.SimpleNamespace(get_hadamard_dt=had),
        "exllamav3.util.tensor": types.SimpleNamespace(save_tensor_image=lambda *a, **k: None),
    }
    for name, mod in stubs.items():
        m = types.ModuleType(name)
        m.__dict__.update(vars(mod))
        sys.modules[name] = m
    module = load_qsrt_encoder(Path(tempfile.mkdtemp()))
    if build_ref.HARNESS.exists():
        module.quantize_tiles = _procedural_quantizer(build_ref.load_harness())
    ext = build_ref.load()
    sqg_quantizer._extension = lambda: ext
    sqg_quantizer.install_sqg_quantizer(module)
    module.pack_trellis = _pack_any_k
    return module


def _pack_any_k(enc, qa):
    """pack_trellis stub: kquant.qsrt's restatement for K2..K4 (the only rates it accepts); the C oracle's
    restatement of the same word order (oracle/kq_oracle.c) at other K."""
    from kquant import qsrt
    K = int(qa["K"])
    if K in (2, 3, 4):
        return qsrt.pack_trellis_edges(enc, K)
    from oracle import oracle as O
    return torch.from_numpy(O.pack_trellis(enc.cpu().numpy(), K)).to(enc.device)


def _procedural_quantizer(harness):
    """The reference backend's plain (non-SQG) tile quantiser, served by the reference kernel template at any K.

    Upstream EXL3 calls ext.quantize_tiles with the MCG / MUL1 flags taken from
    the key presence of ``mcg`` / ``mul1`` (kquant/exl3_encoder_backend.py:81-111);
    that extension is not vendored, so the reference's own kernel
    (oracle/ref_harness.cu) stands in for it.
    """
    def quantize_tiles(tiles, quant_args):
        if "mcg" in quant_args:
            cb = 1
        elif "mul1" in quant_args:
            cb = 2
        else:
            raise NotImplementedError("3INST tiles have no reference kernel here")
        tiles = tiles.contiguous()
        K, n, dev = int(quant_args["K"]), tiles.shape[0], tiles.device
        sms = torch.cuda.get_device_properties(dev).multi_processor_count
        mb = max(1, min(n, sms))
        costs = torch.zeros((mb, 2, 65536 >> K), dtype=torch.float16, device=dev)
        edges = torch.empty(mb * harness.kqref_decision_bytes_per_tile(K), dtype=torch.uint8, device=dev)
        out = torch.empty_like(tiles)
        idx = torch.empty((n, 256), dtype=torch.int16, device=dev)
        rc = harness.kqref_quantize_procedural(tiles.data_ptr(), out.data_ptr(), idx.data_ptr(), costs.data_ptr(),
                                               edges.data_ptr(), n, mb, K, cb,
                                               int(quant_args.get("tailbite_context", 128)),
                                               torch.cuda.current_stream(dev).cuda_stream)
        if rc != 0:
            raise RuntimeError(f"reference harness failed: {rc}")
        return out, idx
    return quantize_tiles


def _states(module_qsrt, trellis, K):
    if K in (2, 3, 4):
        return module_qsrt.unpack_trellis_states(trellis.cpu(), K).to(torch.int16)
    from oracle import oracle as O
    edges = O.unpack_trellis(trellis.cpu().numpy(), K)
    return torch.from_numpy(O.reconstruct_states(edges, K)).to(torch.int16)


def run_qsrt_case(name, ref, kq, device):
    from kquant import qsrt as ref_qsrt
    from kquant.ldlq import make_shared_h as ref_shared
    from kquant_b200.ldlq import make_shared_h as kq_shared
    out = {}
    # reference end to end
    w, h, args = C.qsrt_inputs(name, device)
    with C.Capture(ref) as cap:
        wq, proxy, tens = ref.quantize_qsrt(w.clone(), ref_shared(w.shape[0], device, h), args, True)
    torch.cuda.synchronize()
    states = _states(ref_qsrt, tens["trellis"], args["K"])
    idx = C.sample_index(wq.numel())
    out["ref"] = {"w_r": C.digest(cap.inputs[0]), "L": C.digest(cap.inputs[1]), "suh": C.digest(tens["suh"]),
                  "svh": C.digest(tens["svh"]), "g_scale": float(args["g_scale"]), "proxy": float(proxy),
                  "states": C.digest(states), "state_rows": C.row_digests(states),
                  "trellis": C.digest(tens["trellis"]), "weight_q": C.digest(wq),
                  "weight_q_sample": wq.flatten()[idx.to(device)].cpu().tolist()}
    ref_inputs = cap.inputs
    # this backend's preparation on the same inputs
    w, h, args = C.qsrt_inputs(name, device)
    with C.Capture(kq) as kcap:
        kwq, kproxy, ktens = kq.quantize_qsrt(w.clone(), kq_shared(w.shape[0], device, h), args, True)
    torch.cuda.synchronize()
    kstates = _states(ref_qsrt, ktens["trellis"], args["K"])
    out["kq_prep"] = {"w_r": C.digest(kcap.inputs[0]), "L": C.digest(kcap.inputs[1]),
                      "suh": C.digest(ktens["suh"]), "svh": C.digest(ktens["svh"]),
                      "g_scale": float(args["g_scale"])}
    out["prep_equal"] = {key: out["ref"][key] == out["kq_prep"][key] for key in ("w_r", "L", "suh", "svh")}
    # the reference's LDLQ on this backend's rotated inputs
    _, _, args = C.qsrt_inputs(name, device)
    rwq, renc = ref.ldlq(kcap.inputs[0].clone(), kcap.inputs[1].clone(), args)
    torch.cuda.synchronize()
    renc = renc.to(torch.int16)
    out["ref_on_kq_prep"] = {"states": C.digest(renc), "state_rows": C.row_digests(renc),
                             "weight_q": C.digest(rwq)}
    # informational: how this run of this backend compared (the test repeats it)
    out["kq_check"] = {"states_equal_ref_on_kq_prep": C.digest(kstates) == out["ref_on_kq_prep"]["states"],
                       "proxy": float(kproxy),
                       "proxy_rel": abs(float(kproxy) - float(proxy)) / float(proxy)}
    del ref_inputs
    return out


def run_batch_case(name, ref, kq, device):
    from kquant.ldlq import make_shared_h as ref_shared
    ws, hs, groups = C.batch_inputs(name, device)
    res = ref.quantize_qsrt_batch([w.clone() for w in ws], [ref_shared(w.shape[0], device, h)
                                                             for w, h in zip(ws, hs)], groups)
    torch.cuda.synchronize()
    out = {"sources": []}
    for s, cands in enumerate(res):
        rows = []
        for c in cands:
            idx = C.sample_index(c["weight_q"].numel())
            rows.append({"states": C.digest(c["encoded"].to(torch.int16)), "suh": C.digest(c["suh"]),
                         "svh": C.digest(c["svh"]), "proxy": float(c["proxy"]), "g_scale": float(c["g_scale"]),
                         "weight_q_sample": c["weight_q"].flatten()[idx.to(device)].cpu().tolist()})
        out["sources"].append(rows)
    return out


def run_uniform_case(name, ref, kq, device):
    from kquant import qsrt as ref_qsrt
    from kquant.ldlq import make_shared_h as ref_shared
    ws, h, args = C.uniform_inputs(name, device)
    shared = ref_shared(ws[0].shape[0], device, h)
    res = ref.quantize_uniform_batch([w.clone() for w in ws], [shared, shared], args)
    torch.cuda.synchronize()
    out = {"members": []}
    for t, (proxy, tens) in enumerate(res):
        states = _states(ref_qsrt, tens["trellis"], args[t]["K"])
        out["members"].append({"states": C.digest(states), "suh": C.digest(tens["suh"]),
                               "svh": C.digest(tens["svh"]), "proxy": float(proxy),
                               "g_scale": float(args[t]["g_scale"])})
    return out


def main():
    if len(sys.argv) < 2:
        raise SystemExit(__doc__)
    root = os.environ.get("KQ_REFERENCE_ROOT")
    if not root:
        raise SystemExit("set KQ_REFERENCE_ROOT to the directory that holds the reference's kquant package")
    out_path = Path(sys.argv[1])
    only = set(sys.argv[2:])
    device = torch.device("cuda:0")
    torch.cuda.set_device(device)
    ref = load_reference_backend(Path(root).resolve())
    from kquant_b200 import exl3_encoder_backend as kq
    fixtures = {"device": torch.cuda.get_device_name(device), "torch": torch.__version__, "cases": {}}
    runners = [(C.QSRT_CASES, run_qsrt_case), (C.BATCH_CASES, run_batch_case), (C.UNIFORM_CASES, run_uniform_case)]
    for cases, runner in runners:
        for name in cases:
            if only and name not in only:
                continue
            fixtures["cases"][name] = runner(name, ref, kq, device)
            print(name, json.dumps({k: v for k, v in fixtures["cases"][name].items()
                                    if k in ("prep_equal", "kq_check")}), flush=True)
    out_path.parent.mkdir(parents=True, exist_ok=True)
    out_path.write_text(json.dumps(fixtures, indent=1))
    print("wrote", out_path)


if __name__ == "__main__":
    main()
