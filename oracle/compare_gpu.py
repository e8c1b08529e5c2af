"""Side-by-side timing of this build against the reference's own code on one GPU (test infrastructure).

Not part of the product and not the benchmark line: it times the reference's
CUDA tile kernel (compiled from its sources into oracle/_ref) and the
reference's whole encoder backend (its Python package installed in
baseline/_ref, with that kernel as its tile quantiser) next to this build, on
the same GPU and the same inputs, and prints one JSON object.

* ``tile_kernel``: tiles/s of the tile encoder alone, 4,736 N(0, 1) tiles
  (32 tiles per SM), C = 128: K2..K4 with the production SQG codebook against
  the reference binding ``quantize_tiles_sqg``; K1 and K5..K8 with MCG against
  the reference kernel at those K (oracle/ref_harness.cu).
* ``triplet_encode``: one Kimi-class expert triplet (gate, up [7168 x 2048]
  sharing H13; down [2048 x 7168] with H2; K=3, SQG, C=128) encoded by the
  reference's ``quantize_uniform_batch`` and by this build's
  ``quantize_uniform_batches``; weights/s from CUDA events.

Usage: python oracle/compare_gpu.py [--skip-encode]
"""
from __future__ import annotations

import json
import sys
from pathlib import Path

import torch

ROOT = Path(__file__).resolve().parents[1]
# run as a script, this file's directory would shadow the ``oracle`` package with oracle/oracle.py
sys.path[:] = [str(ROOT)] + [p for p in sys.path if Path(p or ".").resolve() != Path(__file__).resolve().parent]


def _events(fn, reps=1):
    fn()
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(reps):
        fn()
    b.record()
    torch.cuda.synchronize()
    return a.elapsed_time(b) / 1e3 / reps


def tile_kernels(dev):
    from kquant_b200 import _native
    from kquant_b200.codebooks import sqg_xor_cheb_t12_bytes
    from oracle import build_ref
    sms = torch.cuda.get_device_properties(dev).multi_processor_count
    n = 32 * sms
    tiles = torch.randn((n, 256), generator=torch.Generator(device=dev).manual_seed(3), device=dev)
    out = {}
    ext = build_ref.load() if build_ref.OUT.exists() else None
    harness = build_ref.load_harness() if build_ref.HARNESS.exists() else None
    for K in range(1, 9):
        row = {}
        if K in (2, 3, 4):
            lut = sqg_xor_cheb_t12_bytes(K).to(dev)
            labels = _native.build_labels(_native.KQ_CB_SQG, lut, dev)
        else:
            labels = _native.build_labels(_native.KQ_CB_MCG, None, dev)
        t = _events(lambda: _native.viterbi_encode(tiles, K, labels, 128), reps=2)
        row["kq_tiles_per_s"] = round(n / t)
        if K in (2, 3, 4) and ext is not None:
            edges = 65536 >> K
            dec = edges // (4 if K == 2 else 2)
            mb = max(256, 3 * sms)
            costs = torch.zeros((mb, 2, edges), dtype=torch.float16, device=dev)
            tb = torch.empty((mb, 256, dec), dtype=torch.uint8, device=dev)
            lut_t = lut.reshape(1 << K, edges // 2, 2).permute(1, 0, 2).contiguous().reshape(-1)
            o = torch.empty_like(tiles)
            i = torch.empty((n, 256), dtype=torch.int16, device=dev)
            t = _events(lambda: ext.quantize_tiles_sqg(tiles, o, i, costs, tb, lut_t, K, 128), reps=2)
            row["reference_tiles_per_s"] = round(n / t)
        elif harness is not None:
            mb = sms
            costs = torch.zeros((mb, 2, 65536 >> K), dtype=torch.float16, device=dev)
            edges = torch.empty(mb * harness.kqref_decision_bytes_per_tile(K), dtype=torch.uint8, device=dev)
            o = torch.empty_like(tiles)
            i = torch.empty((n, 256), dtype=torch.int16, device=dev)
            st = torch.cuda.current_stream(dev).cuda_stream
            t = _events(lambda: harness.kqref_quantize_procedural(tiles.data_ptr(), o.data_ptr(), i.data_ptr(),
                                                                  costs.data_ptr(), edges.data_ptr(), n, mb, K, 1,
                                                                  128, st))
            row["reference_tiles_per_s"] = round(n / t)
        if "reference_tiles_per_s" in row:
            row["speedup"] = round(row["kq_tiles_per_s"] / row["reference_tiles_per_s"], 2)
        out[f"K{K}"] = row
    return out


def triplet_encode(dev):
    import bench
    from kquant_b200 import exl3_encoder_backend as kq
    from kquant_b200.ldlq import make_shared_h
    from tests.golden.make_ref_cuda_fixtures import load_reference_backend
    ref_root = ROOT / "baseline" / "_ref"
    if not (ref_root / "kquant").exists():
        return {"unavailable": "reference package not installed in baseline/_ref"}
    ref = load_reference_backend(ref_root)
    from kquant.ldlq import make_shared_h as ref_shared
    hf, h13, h2 = bench.make_triplet(dev, seed=1234)
    exl = [bench.to_exl(w) for w in hf]

    def ref_step():
        s13 = ref_shared(bench.HIDDEN, dev, h13)
        ref.quantize_uniform_batch([exl[0].clone(), exl[1].clone()], [s13, s13],
                                   [bench.quant_args("w1", dev), bench.quant_args("w3", dev)])
        ref.quantize_uniform_batch([exl[2].clone()], [ref_shared(bench.INTER, dev, h2)], [bench.quant_args("w2", dev)])

    def kq_step():
        s13 = make_shared_h(bench.HIDDEN, dev, h13)
        kq.quantize_uniform_batches([
            ([exl[0].clone(), exl[1].clone()], [s13, s13], [bench.quant_args("w1", dev), bench.quant_args("w3", dev)]),
            ([exl[2].clone()], [make_shared_h(bench.INTER, dev, h2)], [bench.quant_args("w2", dev)])])

    weights = 3 * bench.HIDDEN * bench.INTER
    t_kq = _events(kq_step)
    t_ref = _events(ref_step)
    return {"weights": weights, "kq_s": round(t_kq, 3), "reference_s": round(t_ref, 3),
            "kq_mweights_per_s": round(weights / t_kq / 1e6, 2),
            "reference_mweights_per_s": round(weights / t_ref / 1e6, 2), "speedup": round(t_ref / t_kq, 2)}


def main():
    dev = torch.device("cuda:0")
    torch.cuda.set_device(dev)
    res = {"device": torch.cuda.get_device_name(dev), "tile_kernel": tile_kernels(dev)}
    if "--skip-encode" not in sys.argv:
        res["triplet_encode"] = triplet_encode(dev)
    print(json.dumps(res, indent=1))


if __name__ == "__main__":
    main()
