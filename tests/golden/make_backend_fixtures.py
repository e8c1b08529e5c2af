"""Generate end-to-end golden fixtures from the REFERENCE backend (run here, on CPU).

The reference's own ``kquant/exl3_encoder_backend.py`` is loaded with its own
loader (``kquant.exl3_loader.load_qsrt_encoder``).  The missing ExLlamaV3 pieces
are stubbed as the decoder contract defines them: a Sylvester Hadamard
normalised 1/sqrt(n) (``kquant/exl3_reference.py:195-212``) and pack_trellis =
``kquant.qsrt.pack_trellis_edges``.  CUDA synchronisation and streams become
no-ops, and the tile quantizer is the C oracle (a restatement of the reference
Viterbi kernel, pinned against it bit for bit on the GPU).  Random sign draws
use the CPU generator; the GPU test reproduces them the same way.

Usage: python tests/golden/make_backend_fixtures.py /path/to/reference [case ...]
Writes tests/golden/backend_<case>.npz (quantize_qsrt cases and the
quantize_uniform_batch cases).
"""
from __future__ import annotations

import math
import sys
import tempfile
import types
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
ROOT = HERE.parents[1]
sys.path.insert(0, str(ROOT))

from tests.golden.backend_cases import CASES, UNIFORM_CASES, make_inputs, make_uniform_inputs  # noqa: E402


def _load_reference_backend(ref_root: Path):
    sys.path.insert(0, str(ref_root))
    from kquant import qsrt
    from kquant.exl3_loader import load_qsrt_encoder
    from oracle import oracle as O

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
    module.get_quant_stream = lambda device: None
    labels = {}

    def quantize_tiles(tiles, quant_args):
        bits = int(quant_args["K"])
        lut = quant_args["sqg_e4m3_luts_by_bits"][bits]
        key = (bits, id(lut))
        if key not in labels:
            labels[key] = O.labels(O.CB_SQG, lut.numpy())
        idx, val, rc = O.viterbi(bits, labels[key], tiles.numpy(), int(quant_args.get("tailbite_context", 128)))
        assert rc == 0
        return torch.from_numpy(val), torch.from_numpy(idx.view(np.int16))

    module.quantize_tiles = quantize_tiles
    # On CUDA, block_ldl returns (L in H's storage, a host copy of the damped
    # H) because H.cpu() copies.  On CPU H.cpu() aliases H, so the copy is
    # overwritten by L; clone first to keep the CUDA semantics.
    ldl = module.block_ldl

    def block_ldl(H, b, quant_args, verbose):
        keep = H.clone()
        L, _ = ldl(H, b, quant_args, verbose)
        return L, keep

    module.block_ldl = block_ldl
    module.pack_trellis = lambda enc, qa: qsrt.pack_trellis_edges(enc, qa["K"])
    torch.cuda.synchronize = lambda *a, **k: None
    return module


def main():
    if len(sys.argv) < 2:
        raise SystemExit("usage: make_backend_fixtures.py REFERENCE_ROOT [case ...]")
    ref_root = Path(sys.argv[1])
    be = _load_reference_backend(ref_root)
    only = set(sys.argv[2:])
    for name, case in CASES.items():
        if only and name not in only:
            continue
        w, h, args = make_inputs(case, "cpu")
        from kquant.ldlq import make_shared_h
        H_data = make_shared_h(w.shape[0], torch.device("cpu"), h)
        wq, proxy, out = be.quantize_qsrt(w.clone(), H_data, args, True)
        # unpacked states come from the reference's ldlq in the same run; recover them by unpacking
        from kquant.qsrt import unpack_trellis_states
        np.savez_compressed(
            HERE / f"backend_{name}.npz",
            weight_q=wq.numpy(), proxy=np.array(proxy), suh=out["suh"].numpy(), svh=out["svh"].numpy(),
            trellis=out["trellis"].numpy(), g_scale=np.array(args["g_scale"]),
            states=unpack_trellis_states(out["trellis"], args["K"]).numpy())
        print(name, "proxy", proxy, "g_scale", args["g_scale"])
    for name, case in UNIFORM_CASES.items():
        if only and name not in only:
            continue
        ws, hs, args = make_uniform_inputs(case, "cpu")
        from kquant.ldlq import make_shared_h
        from kquant.qsrt import unpack_trellis_states
        shared = make_shared_h(ws[0].shape[0], torch.device("cpu"), hs[0])
        H_datas = [shared, shared] if hs[1] is hs[0] else [shared, make_shared_h(ws[1].shape[0], torch.device("cpu"), hs[1])]
        res = be.quantize_uniform_batch([w.clone() for w in ws], H_datas, args)
        fields = {}
        for t, (proxy, out) in enumerate(res):
            fields.update({f"proxy{t}": np.array(proxy), f"suh{t}": out["suh"].numpy(), f"svh{t}": out["svh"].numpy(),
                           f"g_scale{t}": np.array(args[t]["g_scale"]),
                           f"states{t}": unpack_trellis_states(out["trellis"], args[t]["K"]).numpy()})
            print(name, t, "proxy", proxy, "g_scale", args[t]["g_scale"])
        np.savez_compressed(HERE / f"backend_{name}.npz", **fields)


if __name__ == "__main__":
    main()
