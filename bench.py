"""Benchmark: EXL3/QSRT encode of one Kimi-class MoE expert triplet per GPU.

Workload: gate_proj and up_proj (HF [2048, 7168],
EXL [7168, 2048]) share H13 = X^T X / 8192 from 8192 synthetic tokens of
hidden 7168; down_proj (HF [7168, 2048], EXL [2048, 7168]) uses H2 from the
2048 SiLU-gated activations.  Every matrix is encoded at K=3 with the
production SQG codebook (sqg_xor_cheb_t12), tail-biting context 128.

One step is the complete encode of the triplet through the public plugin API
(``quantize_uniform_batch``): H finalisation, regularisation, global scale
search, block-LDLQ with the sm_100a Viterbi kernel, packing and proxy error.
Under torchrun each rank encodes its own triplet (weak scaling).  NCCL carries
only the per-step reduce of the proxy statistics.

``value`` times K steps with inputs resident in HBM.  ``e2e`` times the same
call with the bf16 weights and fp32 Hessians starting in pinned host memory
and the packed trellis, scales and proxies read back to the host.
``--impl reference`` times the CPU restatement of the reference tile encoder
(the reference has no CPU implementation of its own) on a bounded sample of
the same workload.
"""

from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import tempfile
import time
from pathlib import Path

import torch

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "EXL3 encoded Mweights/s (K=3, expert triplet)"
UNIT = "Mweights/s"
HIDDEN, INTER, TOKENS, K_BITS, CTX = 7168, 2048, 8192, 3, 128
CONFIG = {"workload": "kimi_expert_triplet_k3", "matrices": "gate,up [7168x2048] + down [2048x7168] (EXL k x n)",
          "K": K_BITS, "codebook": "sqg_xor_cheb_t12", "tailbite_context": CTX, "tokens": TOKENS,
          "l2": "inputs larger than L2 (bf16 weights 88 MB + H 222 MB per step)"}


def _set_rate(K: int) -> None:
    """Run the triplet at another rate (BASELINE's metric is quoted at 2/3/4 bpw; configs[1] is K=3)."""
    global K_BITS, METRIC, CONFIG
    if K not in (2, 3, 4):
        raise SystemExit("the trellis kernel supports K2--K4")
    K_BITS = K
    METRIC = f"EXL3 encoded Mweights/s (K={K}, expert triplet)"
    CONFIG = dict(CONFIG, K=K, workload=f"kimi_expert_triplet_k{K}")


def _dist():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import torch.distributed as dist
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", device_id=torch.device("cuda", local))
    return world, rank, local


def make_triplet_weights(device: torch.device, seed: int):
    """Synthetic bf16 expert weights (HF orientation): N(0, 0.015^2) entries, rows scaled by |Student-t(4)|
    normalised to unit median.  Returns ((gate, up, down), the generator to continue from, None)."""
    g = torch.Generator(device=device).manual_seed(seed)

    def weight(rows, cols):
        w = torch.randn((rows, cols), generator=g, device=device) * 0.015
        z = torch.randn((rows, 5), generator=g, device=device)
        t = z[:, 0] / torch.sqrt((z[:, 1:] ** 2).sum(1) / 4)
        s = t.abs() / t.abs().median()
        return (w * s.unsqueeze(1)).to(torch.bfloat16)

    return (weight(INTER, HIDDEN), weight(INTER, HIDDEN), weight(HIDDEN, INTER)), g, None


def make_triplet(device: torch.device, seed: int):
    """Synthetic bf16 expert weights (HF orientation) and the two fp32 Hessians."""
    (gate, up, down), g, _ = make_triplet_weights(device, seed)
    chan = torch.exp(torch.randn(HIDDEN, generator=g, device=device))
    x = torch.randn((TOKENS, HIDDEN), generator=g, device=device) * chan
    h13 = (x.T @ x) / TOKENS
    act = torch.nn.functional.silu(x @ gate.float().T) * (x @ up.float().T)
    h2 = (act.T @ act) / TOKENS
    del x, act
    return (gate, up, down), h13.contiguous(), h2.contiguous()


def quant_args(matrix: str, device: torch.device, layer: int = 1):
    from kquant_b200.codebooks import sqg_xor_cheb_t12_bytes
    idx = ("w1", "w3", "w2").index(matrix)
    seed = layer * 1_000_000 + idx
    args = {"K": K_BITS, "seed": seed, "sv_seed": seed + 499_979, "sigma_reg": 0.025, "devices": [str(device)],
            "device_ratios": None, "apply_out_scales": False, "ldlq_tf32": False, "tailbite_context": CTX,
            "sqg_e4m3_luts_by_bits": {b: sqg_xor_cheb_t12_bytes(b) for b in (2, 3, 4)}}
    if matrix in ("w1", "w3"):
        args["g_scale_into_sv"] = True
    return args


def encode_triplet(weights_exl, h13, h2, device):
    """One step: encode gate+up (shared H13) and down (H2), their LDLQ traversals overlapped; returns outputs."""
    from kquant_b200 import exl3_encoder_backend as be
    from kquant_b200.ldlq import make_shared_h
    gate, up, down = weights_exl
    shared = make_shared_h(HIDDEN, device, h13)
    r13, r2 = be.quantize_uniform_batches([
        ([gate, up], [shared, shared], [quant_args("w1", device), quant_args("w3", device)]),
        ([down], [make_shared_h(INTER, device, h2)], [quant_args("w2", device)]),
    ])
    return r13 + r2


def to_exl(w_hf: torch.Tensor) -> torch.Tensor:
    """bf16 HF [out, in] -> fp32 EXL [in, out] on the transposing load kernel."""
    from kquant_b200 import _native
    return _native.bf16_to_f32_transposed(w_hf)


class ClockSampler:
    def __init__(self, index: int):
        self.index = index
        self.proc = None
        self.path = None

    def __enter__(self):
        fd, self.path = tempfile.mkstemp(suffix=".csv")
        os.close(fd)
        q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
             "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
             "clocks_event_reasons.sw_power_cap")
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--id={self.index}", f"--query-gpu={q}",
                                          "--format=csv,noheader,nounits", "-lms", "200"],
                                         stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except OSError:
            self.proc = None
        return self

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self):
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        try:
            for line in open(self.path):
                parts = [p.strip() for p in line.split(",")]
                if len(parts) < 9:
                    continue
                try:
                    sm.append(float(parts[1]))
                    mx = float(parts[2])
                except ValueError:
                    continue
                for name, flag in zip(names, parts[5:9]):
                    if flag.lower() == "active":
                        reasons.add(name)
        except OSError:
            pass
        finally:
            try:
                os.unlink(self.path)
            except OSError:
                pass
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm)}


def _allreduce_max(x: float, world: int) -> float:
    if world == 1:
        return x
    import torch.distributed as dist
    t = torch.tensor([x], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def _reduce_proxy(results, world):
    """Per-step NCCL reduce of the per-tensor proxy statistics; slot = rank * 3 + tensor."""
    from kquant_b200.sharding import reduce_proxy_stats
    rank = int(os.environ.get("RANK", "0"))
    num = torch.zeros(3 * world, dtype=torch.float64, device="cuda")
    den = torch.zeros(3 * world, dtype=torch.float64, device="cuda")
    num[3 * rank:3 * rank + 3] = torch.tensor([r[0] for r in results], dtype=torch.float64)
    den[3 * rank:3 * rank + 3] = 1.0
    return reduce_proxy_stats(num, den)


def cpu_tile_rate(seconds_target: float = 15.0):
    """Oracle (CPU restatement of the reference tile encoder) on all host cores: tiles/s and sample."""
    import numpy as np
    from kquant_b200.codebooks import sqg_xor_cheb_t12_bytes
    from oracle import oracle as O
    cores = os.cpu_count() or 1
    lab = O.labels(O.CB_SQG, sqg_xor_cheb_t12_bytes(K_BITS).numpy())
    rng = np.random.default_rng(0)
    n = cores
    t0 = time.perf_counter()
    O.viterbi(K_BITS, lab, rng.standard_normal((n, 256)).astype(np.float32), CTX, threads=cores)
    dt = time.perf_counter() - t0
    reps = max(1, int(seconds_target / max(dt, 1e-3)))
    n2 = n * reps
    tiles = rng.standard_normal((n2, 256)).astype(np.float32)
    t0 = time.perf_counter()
    O.viterbi(K_BITS, lab, tiles, CTX, threads=cores)
    dt = time.perf_counter() - t0
    return n2 / dt, cores, n2


def weights_per_step():
    return 3 * HIDDEN * INTER


def run_reference(args, world, rank):
    """CPU arm: the oracle restatement of the reference tile encoder on the host cores."""
    if rank != 0:
        return
    # tile encodes per step of the GPU arm: every weight tile once, plus the scale search
    tiles_per_step = weights_per_step() / 256 * 1.22
    values = []
    cores = os.cpu_count() or 1
    sample = ""
    for i in range(args.warmup + args.steps):
        rate, cores, n = cpu_tile_rate(seconds_target=6.0 if i < args.warmup else 12.0)
        if i >= args.warmup:
            values.append(rate / tiles_per_step * weights_per_step() / 1e6)
            sample = f"{n} tiles of K={K_BITS} tail-biting Viterbi (C={CTX}) per step, extrapolated to the triplet"
    v = statistics.median(values)
    line = {"metric": METRIC, "value": v, "unit": UNIT, "n_gpus": args.gpus, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": weights_per_step() / (v * 1e6) * 1e3, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f16", "data": "synthetic", "config": CONFIG,
            "impl": "reference",
            "cpu_baseline": {"value": v, "unit": UNIT, "cores": cores, "kind": "port", "sample": sample},
            "e2e": {"value": v, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def run_viterbi_case(args, local):
    """Tile kernel alone on random N(0,1) tiles: the small case used for ncu captures."""
    from kquant_b200 import _native
    from kquant_b200.codebooks import sqg_xor_cheb_t12_bytes
    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    labels = _native.build_labels(_native.KQ_CB_SQG, sqg_xor_cheb_t12_bytes(args.K).to(device), device)
    g = torch.Generator(device=device).manual_seed(5)
    tiles = torch.randn((args.tiles, 256), generator=g, device=device)
    for _ in range(args.warmup):
        _native.viterbi_encode(tiles, args.K, labels, CTX)
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(args.steps):
        _native.viterbi_encode(tiles, args.K, labels, CTX)
    b.record()
    torch.cuda.synchronize()
    sec = a.elapsed_time(b) / 1e3 / max(args.steps, 1)
    rate = _native.measure_hfma2_rate(device)
    relax = args.tiles * (2 * CTX + 256) * 65536
    print(json.dumps({"case": "viterbi", "K": args.K, "tiles": args.tiles, "ms_per_launch": sec * 1e3,
                      "tiles_per_s": args.tiles / sec, "frac_of_fp16_alu_peak": 3 * relax / sec / (2 * rate)}))


def run_trace_case(args, local):
    """Proxy numerator tr(E^T H E) of the gate/up encode (k=7168, n=4096) on the tcgen05 trace kernel."""
    from kquant_b200 import _native
    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    k, n = HIDDEN, 2 * INTER
    g = torch.Generator(device=device).manual_seed(9)
    H = torch.randn((k, k), generator=g, device=device)
    Et = torch.randn((n, k), generator=g, device=device)
    for _ in range(args.warmup):
        _native.trace_abt(Et, H, Et)
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(args.steps):
        _native.trace_abt(Et, H, Et)
    b.record()
    torch.cuda.synchronize()
    _native.check_trace_errors()
    sec = a.elapsed_time(b) / 1e3 / max(args.steps, 1)
    flops = 2.0 * n * k * k
    print(json.dumps({"case": "trace", "M": n, "N": k, "Kd": k, "ms_per_launch": sec * 1e3,
                      "tflops": flops / sec / 1e12, "algorithmic_bytes": 4 * (k * k + 2 * n * k)}))


def _hbm_peak():
    try:
        return float(json.loads((ROOT / "MEASURED_PEAKS.json").read_text())["hbm_gbs"]), "measured"
    except (OSError, ValueError, KeyError):
        return 6650.0, "fallback"


def _peaks():
    try:
        return json.loads((ROOT / "MEASURED_PEAKS.json").read_text())
    except (OSError, ValueError):
        return {}


def _time(fn, steps, warmup):
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(steps):
        fn()
    b.record()
    torch.cuda.synchronize()
    return a.elapsed_time(b) / 1e3 / max(steps, 1)


def run_pack_case(args, local):
    """Trellis pack / unpack+closure over the triplet's tiles (HBM-bound rows P and S)."""
    from kquant_b200 import _native
    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    n = weights_per_step() // 256
    K = args.K
    states = torch.randint(-32768, 32767, (n, 256), dtype=torch.int16, device=device)
    packed = _native.pack_trellis(states, K)
    peak, src = _hbm_peak()
    out = {"case": "pack", "K": K, "tiles": n, "hbm_peak_gbs": peak, "peak_source": src}
    t = _time(lambda: _native.pack_trellis(states, K), args.steps, args.warmup)
    byt = n * (512 + 32 * K)
    out.update(pack_ms=t * 1e3, pack_gbs=byt / t / 1e9, pack_frac=byt / t / 1e9 / peak)
    t = _time(lambda: _native.unpack_trellis_states(packed, K), args.steps, args.warmup)
    out.update(unpack_ms=t * 1e3, unpack_gbs=byt / t / 1e9, unpack_frac=byt / t / 1e9 / peak)
    print(json.dumps(out))


def run_load_case(args, local):
    """bf16 HF -> fp32 EXL weight load of the triplet (gate, up, down), plain and with a row gather."""
    from kquant_b200 import _native
    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    g = torch.Generator(device=device).manual_seed(3)
    ws = [torch.randn(s, generator=g, device=device).to(torch.bfloat16)
          for s in ((INTER, HIDDEN), (INTER, HIDDEN), (HIDDEN, INTER))]
    perms = [torch.randperm(w.shape[0], generator=g, device=device) for w in ws]
    peak, src = _hbm_peak()
    byt = sum(w.numel() for w in ws) * (2 + 4)
    t = _time(lambda: [_native.bf16_to_f32_transposed(w) for w in ws], args.steps, args.warmup)
    tp = _time(lambda: [_native.bf16_to_f32_transposed(w, p) for w, p in zip(ws, perms)], args.steps, args.warmup)
    tt = _time(lambda: [w.float().T.contiguous() for w in ws], args.steps, args.warmup)
    print(json.dumps({"case": "load", "weights": sum(w.numel() for w in ws), "bytes": byt, "hbm_peak_gbs": peak,
                      "peak_source": src, "ms": t * 1e3, "gbs": byt / t / 1e9, "frac": byt / t / 1e9 / peak,
                      "gather_ms": tp * 1e3, "gather_gbs": byt / tp / 1e9,
                      "torch_float_T_contiguous_ms": tt * 1e3}))


def run_hessian_case(args, local):
    """Hessian accumulation (kquant/capture.py:713-730) of --tokens samples of width --dim on the tensor cores.

    Reports the whole call (operand kernel + GEMM), the GEMM launch alone timed with CUDA events on its
    stream, the tensor work it performs (upper-triangle tiles only; 3 products for 3xTF32) against the
    TF32 peak (half the measured bf16 figure), and torch's FP32 addmm of the reference on the same data.
    """
    from kquant_b200 import _native
    from kquant_b200.capture import accumulate_hessian
    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    T, d = args.tokens, args.dim
    g = torch.Generator(device=device).manual_seed(4)
    x = torch.randn((T, d), generator=g, device=device)
    w = torch.rand(T, generator=g, device=device) + 0.5
    H = torch.zeros((d, d), device=device)
    dpad = -(-d // 256) * 256
    nt = dpad // 256
    tile_frac = nt * (nt + 1) * 128 * 256 / (dpad * dpad)
    peak = _peaks().get("bf16_tflops", 1590.0) / 2
    out = {"case": "hessian", "tokens": T, "dim": d, "tf32_peak_tflops": peak,
           "upper_tile_fraction": round(tile_frac, 4)}
    for prec, split in (("tf32", 1), ("3xtf32", 3)):
        t = _time(lambda: accumulate_hessian(x, w, device=device, chunk_rows=T, precision=prec),
                  args.steps, args.warmup)
        ws = _native.accumulate_hessian(x, w, H, split)
        t_all = _time(lambda: _native.accumulate_hessian(x, w, H, split, ws), args.steps, args.warmup)
        performed = 2.0 * T * dpad * dpad * tile_frac * split
        out[f"{prec}_call_ms"] = round(t * 1e3, 4)
        out[f"{prec}_kernels_ms"] = round(t_all * 1e3, 4)
        out[f"{prec}_tensor_tflops"] = round(performed / t_all / 1e12, 1)
        out[f"{prec}_frac_of_tf32_peak"] = round(performed / t_all / 1e12 / peak, 3)
    acc = torch.zeros((d, d), device=device)
    torch.backends.cuda.matmul.allow_tf32 = False
    t = _time(lambda: acc.addmm_(x.T, x * w.unsqueeze(1)), args.steps, args.warmup)
    out["torch_fp32_addmm_ms"] = round(t * 1e3, 4)
    print(json.dumps(out))


def run_experts_case(args, local):
    """A bounded slice of BASELINE configs[2]: --experts Kimi-class experts on one GPU, per-expert Hessians from
    64 routed tokens (top-8 of 384 over 8192 synthetic tokens), per-tensor K in {2,3,4} drawn with probabilities
    (0.2, 0.4, 0.4) (3.2 bpw on average), all encoded by one quantize_uniform_batches call per step."""
    from kquant_b200 import _native
    from kquant_b200 import exl3_encoder_backend as be
    from kquant_b200.ldlq import make_shared_h
    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    _native.load()
    E = args.experts
    g = torch.Generator(device=device).manual_seed(77)
    chan = torch.exp(torch.randn(HIDDEN, generator=g, device=device))
    x_all = torch.randn((TOKENS, HIDDEN), generator=g, device=device) * chan
    logits = torch.randn((TOKENS, 384), generator=g, device=device)
    routed = torch.zeros((TOKENS, 384), dtype=torch.bool, device=device)
    routed.scatter_(1, logits.topk(8, dim=1).indices, True)
    kg = torch.Generator().manual_seed(78)
    ks = [[(2, 3, 4)[int(torch.multinomial(torch.tensor([0.2, 0.4, 0.4]), 1, generator=kg))] for _ in range(3)]
          for _ in range(E)]
    experts = []
    for e in range(E):
        (gate, up, down), _, _ = make_triplet_weights(device, seed=5000 + e)
        tok = torch.nonzero(routed[:, e]).flatten()[:64]
        x = x_all[tok]
        h13 = (x.T @ x) / x.shape[0]
        act = torch.nn.functional.silu(x @ gate.float().T) * (x @ up.float().T)
        h2 = (act.T @ act) / x.shape[0]
        experts.append(([to_exl(w) for w in (gate, up, down)], h13.contiguous(), h2.contiguous()))
    del x_all

    def groups():
        out = []
        for e, (ws, h13, h2) in enumerate(experts):
            qa = [quant_args(m, device, layer=e + 1) for m in ("w1", "w3", "w2")]
            for q, K in zip(qa, ks[e]):
                q["K"] = K
            s13 = make_shared_h(HIDDEN, device, h13)
            if ks[e][0] == ks[e][1]:
                out.append(([ws[0].clone(), ws[1].clone()], [s13, s13], qa[:2]))
            else:
                out.append(([ws[0].clone()], [s13], qa[:1]))
                out.append(([ws[1].clone()], [s13], qa[1:2]))
            out.append(([ws[2].clone()], [make_shared_h(INTER, device, h2)], qa[2:]))
        return out

    weights = E * 3 * HIDDEN * INTER
    for _ in range(args.warmup):
        be.quantize_uniform_batches(groups())
    torch.cuda.synchronize()
    _native.stats.reset(timing=True)
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(args.steps):
        res = be.quantize_uniform_batches(groups())
    b.record()
    torch.cuda.synchronize()
    t = a.elapsed_time(b) / 1e3 / args.steps
    vl, vbusy, vtiles, vrelax, vsum = _native.stats.viterbi_summary()
    peak = 2.0 * _native.measure_hfma2_rate(device) / 1e12
    proxies = [p for r in res for p, _ in r]
    flat = [k for row in ks for k in row]
    print(json.dumps({
        "case": "experts", "experts": E, "weights_per_step": weights, "bpw_mean": sum(flat) / len(flat),
        "k_counts": {k: flat.count(k) for k in (2, 3, 4)}, "ms_per_step": t * 1e3,
        "mweights_per_s": weights / t / 1e6, "viterbi_launches_per_step": vl // max(args.steps, 1),
        "viterbi_busy_share": vbusy / (t * args.steps),
        "viterbi_frac_of_fp16_peak": 3.0 * vrelax / vbusy / 1e12 / peak if vbusy else None,
        "proxy_max": max(proxies), "data": "synthetic"}))


def run_qsrt_case(args, local):
    """kquant's production call (kquant/pack/qsrt_encoder.py:824-832): quantize_qsrt_batch over --experts experts
    x the three rate-transfer modes R0/R1/R2, once for gate ([7168 x 2048], n-axis records) and once for down
    ([2048 x 7168], k-axis records), per-expert Hessians from 64 routed tokens.  Reports source weights/s (each
    source encoded at all three candidate rates) and candidate weights/s."""
    from kquant_b200 import _native
    from kquant_b200 import exl3_encoder_backend as be
    from kquant_b200 import qsrt
    from kquant_b200.ldlq import make_shared_h
    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    _native.load()
    E = args.experts
    g = torch.Generator(device=device).manual_seed(79)
    chan = torch.exp(torch.randn(HIDDEN, generator=g, device=device))
    srcs = {"w1": [], "w2": []}
    hs = {"w1": [], "w2": []}
    for e in range(E):
        (gate, up, down), _, _ = make_triplet_weights(device, seed=6000 + e)
        x = torch.randn((64, HIDDEN), generator=g, device=device) * chan
        act = torch.nn.functional.silu(x @ gate.float().T) * (x @ up.float().T)
        srcs["w1"].append(to_exl(gate))
        srcs["w2"].append(to_exl(down))
        hs["w1"].append(((x.T @ x) / 64).contiguous())
        hs["w2"].append(((act.T @ act) / 64).contiguous())

    def groups(matrix):
        axis = qsrt.matrix_rate_axis(matrix)
        out = []
        for e in range(E):
            base = quant_args(matrix, device, layer=e + 1)
            cands = []
            for mode in qsrt.RATE_TRANSFER_MODES:
                # the modes' record maps cover 24 records of 128 channels; this expert's intermediate
                # size holds INTER / 128 of them (records come in K2/K4 pairs, so the cut keeps 3 bpw)
                rec = qsrt.record_bits(mode)[:INTER // 128]
                bits = tuple(b for b in rec for _ in range(8))
                cands.append(dict(base, mixed_rate_axis=axis, mixed_tile_bits=bits))
            out.append(cands)
        return out

    def step():
        for matrix, k in (("w1", HIDDEN), ("w2", INTER)):
            be.quantize_qsrt_batch([w.clone() for w in srcs[matrix]],
                                   [make_shared_h(k, device, h) for h in hs[matrix]], groups(matrix))

    for _ in range(max(args.warmup, 1)):
        step()
    torch.cuda.synchronize()
    _native.stats.reset(timing=True)
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(args.steps):
        step()
    b.record()
    torch.cuda.synchronize()
    t = a.elapsed_time(b) / 1e3 / args.steps
    vl, vbusy, vtiles, vrelax, vsum = _native.stats.viterbi_summary()
    peak = 2.0 * _native.measure_hfma2_rate(device) / 1e12
    weights = E * 2 * HIDDEN * INTER
    print(json.dumps({"case": "qsrt", "experts": E, "matrices": "gate (n-axis) + down (k-axis)", "modes": "R0,R1,R2",
                      "ms_per_step": t * 1e3, "source_mweights_per_s": weights / t / 1e6,
                      "candidate_mweights_per_s": 3 * weights / t / 1e6,
                      "viterbi_launches_per_step": vl // max(args.steps, 1),
                      "viterbi_busy_share": vbusy / (t * args.steps),
                      "viterbi_frac_of_fp16_peak": 3.0 * vrelax / vbusy / 1e12 / peak if vbusy else None}))


def run_chain_case(args, local):
    """The LDLQ chain engine alone on the triplet's shapes (gate+up [7168 x 4096] and down [2048 x 7168], K=--K):
    synthetic W, unit-lower-triangular L and zero feedback state, every step of every chain.  Reports launches,
    mean launch time (CUDA events) and tiles/s; the profiling case for pair_kernel<K, ChainIO>."""
    from kquant_b200 import _native
    from kquant_b200 import exl3_encoder_backend as be
    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    _native.load()
    g = torch.Generator(device=device).manual_seed(9)

    def member(k, n):
        W = torch.randn((k, n), generator=g, device=device) * 0.5
        L = torch.tril(torch.randn((k, k), generator=g, device=device) * 0.01, -1) + torch.eye(k, device=device)
        qa = quant_args("w1", device)
        qa["K"] = args.K
        return be._ChainMember(W, L, torch.empty_like(W),
                               torch.empty((k // 16, n // 16, 256), dtype=torch.int16, device=device), qa)

    shapes = [(HIDDEN, 2 * INTER), (INTER, HIDDEN)]
    for _ in range(max(args.warmup, 1)):
        be._chain_traverse([member(k, n) for k, n in shapes], device)
    members = [member(k, n) for k, n in shapes]
    torch.cuda.synchronize()
    _native.stats.reset(timing=True)
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    be._chain_traverse(members, device)
    b.record()
    torch.cuda.synchronize()
    vl, vbusy, vtiles, vrelax, vsum = _native.stats.viterbi_summary()
    peak = 2.0 * _native.measure_hfma2_rate(device) / 1e12
    print(json.dumps({"case": "chain", "K": args.K, "launches": vl, "tiles": vtiles,
                      "ms_total": a.elapsed_time(b), "ms_per_launch": vsum / vl * 1e3,
                      "tiles_per_s": vtiles / vbusy, "frac_of_fp16_alu_peak": 3.0 * vrelax / vbusy / 1e12 / peak}))


def run_profile_case(args, local):
    """Kernel list of one warm triplet step (torch.profiler / CUPTI device times): every launch of the step with
    its device time, grouped by kernel, as a launch list without a replaying profiler."""
    from torch.profiler import ProfilerActivity, profile
    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    hf, h13, h2 = make_triplet(device, seed=1234)
    exl = [to_exl(w) for w in hf]
    for _ in range(max(args.warmup, 1)):
        encode_triplet([w.clone() for w in exl], h13, h2, device)
    torch.cuda.synchronize()
    with profile(activities=[ProfilerActivity.CUDA]) as prof:
        encode_triplet([w.clone() for w in exl], h13, h2, device)
        torch.cuda.synchronize()
    rows = sorted(prof.key_averages(), key=lambda e: -e.device_time_total)
    total = sum(e.device_time_total for e in rows)
    print(json.dumps({"case": "profile", "device_ms": total / 1e3, "kernels": [
        {"name": e.key[:120], "launches": e.count, "ms": e.device_time_total / 1e3,
         "share": e.device_time_total / total} for e in rows[:args.top]]}, indent=1))


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=3)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="kq", choices=["kq", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--e2e-steps", type=int, default=2)
    ap.add_argument("--case", default="triplet",
                    choices=["triplet", "experts", "qsrt", "chain", "viterbi", "trace", "pack", "load", "hessian",
                             "profile"],
                    help="viterbi: only the tile kernel on --tiles random tiles (profiling case)")
    ap.add_argument("--tiles", type=int, default=1184)
    ap.add_argument("--K", type=int, default=K_BITS)
    ap.add_argument("--tokens", type=int, default=TOKENS, help="hessian case: samples per call")
    ap.add_argument("--dim", type=int, default=HIDDEN, help="hessian case: sample width")
    ap.add_argument("--experts", type=int, default=8, help="experts case: experts per GPU")
    ap.add_argument("--top", type=int, default=25, help="profile case: kernels listed")
    args = ap.parse_args()
    if args.case == "triplet" and args.K != K_BITS:
        _set_rate(args.K)
    world, rank, local = _dist()
    if args.case == "experts":
        run_experts_case(args, local)
        return
    if args.case == "profile":
        run_profile_case(args, local)
        return
    if args.case == "chain":
        run_chain_case(args, local)
        return
    if args.case == "qsrt":
        run_qsrt_case(args, local)
        return
    if args.case == "viterbi":
        run_viterbi_case(args, local)
        return
    if args.case == "trace":
        run_trace_case(args, local)
        return
    if args.case == "pack":
        run_pack_case(args, local)
        return
    if args.case == "load":
        run_load_case(args, local)
        return
    if args.case == "hessian":
        run_hessian_case(args, local)
        return
    if args.impl == "reference":
        run_reference(args, world, rank)
        if world > 1:
            torch.distributed.barrier()
            torch.distributed.destroy_process_group()
        return
    from kquant_b200 import _native
    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    _native.load()

    hf, h13, h2 = make_triplet(device, seed=1234 + rank)
    exl = [to_exl(w) for w in hf]

    def step_resident():
        return encode_triplet([w.clone() for w in exl], h13, h2, device)

    for _ in range(args.warmup):
        res = step_resident()
    torch.cuda.synchronize()
    if world > 1:
        torch.distributed.barrier()
    _native.stats.reset(timing=True)
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clk:
        torch.cuda.synchronize()
        start.record()
        for _ in range(args.steps):
            res = step_resident()
            proxies = _reduce_proxy(res, world)
        end.record()
        torch.cuda.synchronize()
    if world > 1:
        torch.distributed.barrier()
    elapsed = _allreduce_max(start.elapsed_time(end) / 1e3, world)
    launches = _native.stats.launches
    vl, vsec, vtiles, vrelax, vsum = _native.stats.viterbi_summary()
    sizes = sorted(n for _, _, n, _ in _native.stats.events)
    median_tiles = sizes[len(sizes) // 2] if sizes else 0
    _native.stats.reset(timing=False)
    clocks = clk.summary()

    # end-to-end: host (pinned) inputs -> device -> encode -> host outputs
    host_w = [w.cpu().pin_memory() for w in hf]
    host_h = [h13.cpu().pin_memory(), h2.cpu().pin_memory()]
    h2d = sum(t.numel() * t.element_size() for t in host_w + host_h)
    torch.cuda.synchronize()
    if world > 1:
        torch.distributed.barrier()
    def step_e2e():
        dw = [w.to(device, non_blocking=True) for w in host_w]
        dh13, dh2 = (h.to(device, non_blocking=True) for h in host_h)
        out = encode_triplet([to_exl(w) for w in dw], dh13, dh2, device)
        host_out = [{k: v.cpu() for k, v in o[1].items()} for o in out]
        proxy_host = _reduce_proxy(out, world).cpu()
        return sum(v.numel() * v.element_size() for o in host_out for v in o.values()) + proxy_host.numel() * 8

    if args.e2e_steps > 0:
        step_e2e()                       # untimed: first-use allocations of the host-input path
        torch.cuda.synchronize()
    es, ee = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    es.record()
    d2h = 0
    for _ in range(max(args.e2e_steps, 0)):
        d2h = step_e2e()
    ee.record()
    torch.cuda.synchronize()
    e_elapsed = max(_allreduce_max(es.elapsed_time(ee) / 1e3, world), 1e-9)

    total_weights = weights_per_step() * world
    value = total_weights * args.steps / elapsed / 1e6
    e2e = total_weights * args.e2e_steps / e_elapsed / 1e6
    hfma2 = _native.measure_hfma2_rate(device)
    peak_ops = 2.0 * hfma2 / 1e12                       # fp16 ops/s (two lanes per HFMA2)
    achieved_ops = 3.0 * vrelax / vsec / 1e12 if vsec > 0 else None
    traffic = None
    tpath = ROOT / "profiles" / "viterbi_dram_bytes_per_tile.txt"
    if tpath.exists() and vl:
        try:
            # per launch of the dominant kernel (the LDLQ chain launches, the median launch size)
            traffic = float(tpath.read_text().split()[0]) * median_tiles
        except (ValueError, IndexError):
            traffic = None
    line = {
        "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": elapsed / args.steps * 1e3, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f16 trellis / f32 LDLQ", "data": "synthetic",
        "config": {**CONFIG, "parallelism": f"expert-sharded x{world}"},
        "e2e": {"value": e2e, "unit": UNIT, "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h},
        "gpu_launches": launches,
        "roofline": {"bound": "alu", "kernel": "kq viterbi_kernel", "achieved": achieved_ops, "peak": peak_ops,
                     "unit": "Tops/s fp16 (3 ops per relaxation)",
                     "frac": (achieved_ops / peak_ops) if achieved_ops else None,
                     "traffic": traffic, "launches": vl, "avg_launch_ms": vsum / vl * 1e3 if vl else None,
                     "busy_ms": vsec * 1e3,
                     "timing": "achieved = relaxations / union of the Viterbi launch intervals (CUDA events "
                               "on the launching stream)",
                     "peak_source": "measured HFMA2 rate (kq_probe_hfma2) x 2 lanes, this GPU, this run"},
        "viterbi_share_of_step": vsec / elapsed if elapsed else None,
        "clocks": clocks,
    }
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        rate, cores, n = cpu_tile_rate()
        tiles_per_step = vtiles / args.steps
        cpu_v = rate / tiles_per_step * weights_per_step() / 1e6
        line["cpu_baseline"] = {"value": cpu_v, "unit": UNIT, "cores": cores, "kind": "port",
                                "sample": f"{n} tiles of the K={K_BITS} C={CTX} Viterbi on {cores} threads, "
                                          f"scaled by the GPU step's {tiles_per_step:.0f} tile encodes"}
    if rank == 0:
        print(json.dumps(line), flush=True)
    if world > 1:
        torch.distributed.destroy_process_group()


if __name__ == "__main__":
    main()
