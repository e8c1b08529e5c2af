"""Benchmark: EXL3/QSRT trellis encode of Kimi-class MoE experts, one process per GPU.

Default workload (``--case slice``): a slice of the full-layer configuration.
Each rank encodes ``--experts`` experts of its shard of a 384-expert layer
(``sharding.shard_experts``: 48 experts per GPU at 8 GPUs).  Every expert is a
gate/up/down triplet (HF gate, up [2048, 7168], down [7168, 2048]; EXL [k, n] =
the transpose) of bf16 weights ~ N(0, 0.015^2) with Student-t(4) row scales.
Per-expert Hessians come from the expert's first 64 routed tokens (top-8 of
384 over 8192 synthetic tokens of width 7168).  Per-tensor K in {2, 3, 4} is a
seeded allocation over the layer with exactly 20 / 40 / 40 % of the tensors
(3.2 bits per weight).  Production SQG codebook (sqg_xor_cheb_t12), C = 128.

One step is the complete encode of the rank's experts through the public
plugin API (``quantize_uniform_batches``: H finalisation, regularisation,
global scale search, block-LDLQ on the sm_100a kernels, packing, proxy error).
Ranks share no data; the per-tensor proxy statistics are reduced over NCCL
once, after the timed steps.

``--case triplet`` is the single expert triplet at one K (``--K``, default 3);
``--case layer`` encodes the whole layer (384 experts + the shared expert)
once across the ranks and reports its wall time.

``value`` times K steps with inputs resident in HBM.  ``e2e`` times the same
call with the bf16 weights and fp32 Hessians starting in pinned host memory
and the packed trellis, scales and proxies read back to the host.
``--impl reference`` times the reference's own LDLQ (CPU torch) with the CPU
restatement of its tile encoder on all host cores (the reference has no CPU
tile encoder of its own) on a bounded slice of the same workload.
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

METRIC = "EXL3 encoded Mweights/s at 2/3/4 bpw"
UNIT = "Mweights/s"
HIDDEN, INTER, TOKENS, K_BITS, CTX = 7168, 2048, 8192, 3, 128
LAYER_EXPERTS, ROUTED_TOKENS, TOP_K = 384, 64, 8
SHARED = LAYER_EXPERTS                   # index of the shared expert


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


def quant_args(matrix: str, device: torch.device, layer: int = 1, K: int = K_BITS):
    from kquant_b200.codebooks import sqg_xor_cheb_t12_bytes
    idx = ("w1", "w3", "w2").index(matrix)
    seed = layer * 1_000_000 + idx
    args = {"K": K, "seed": seed, "sv_seed": seed + 499_979, "sigma_reg": 0.025, "devices": [str(device)],
            "device_ratios": None, "apply_out_scales": False, "ldlq_tf32": False, "tailbite_context": CTX,
            "sqg_e4m3_luts_by_bits": {b: sqg_xor_cheb_t12_bytes(b) for b in (2, 3, 4)}}
    if matrix in ("w1", "w3"):
        args["g_scale_into_sv"] = True
    return args


def encode_triplet(weights_exl, h13, h2, device, K: int = K_BITS):
    """One step: encode gate+up (shared H13) and down (H2), their LDLQ traversals overlapped; returns outputs."""
    from kquant_b200 import exl3_encoder_backend as be
    from kquant_b200.ldlq import make_shared_h
    gate, up, down = weights_exl
    shared = make_shared_h(HIDDEN, device, h13)
    r13, r2 = be.quantize_uniform_batches([
        ([gate, up], [shared, shared], [quant_args("w1", device, K=K), quant_args("w3", device, K=K)]),
        ([down], [make_shared_h(INTER, device, h2)], [quant_args("w2", device, K=K)]),
    ])
    return r13 + r2


def layer_rates(seed: int = 78) -> list[list[int]]:
    """Seeded per-tensor K of the layer's 384 routed experts and the shared expert (row 384), [gate, up, down]:
    exactly 20 % K2, 40 % K3 and 40 % K4 of the 1155 tensors, i.e. 3.2 bits per weight."""
    n = (LAYER_EXPERTS + 1) * 3
    n2 = n // 5
    n3 = (n - n2) // 2
    ks = torch.tensor([2] * n2 + [3] * n3 + [4] * (n - n2 - n3))
    ks = ks[torch.randperm(n, generator=torch.Generator().manual_seed(seed))]
    return ks.view(LAYER_EXPERTS + 1, 3).tolist()


class Layer:
    """Synthetic MoE layer on one rank: the routing activations (identical on every rank, one seed), and the
    rank's experts with their bf16 HF weights and fp32 Hessians resident on the device.

    Expert e's Hessians come from its first 64 routed tokens (top-8 routing of 8192 tokens over 384
    experts): H13 = X_e^T X_e / 64 and H2 = A_e^T A_e / 64 with A_e = SiLU(X_e gate^T) * (X_e up^T).
    The shared expert (index 384) sees all 8192 tokens.
    """

    def __init__(self, device: torch.device, experts: list[int], seed: int = 77, layer: int = 0):
        self.device = device
        self.layer = layer
        self.rates = layer_rates(78 + layer)
        g = torch.Generator(device=device).manual_seed(seed)
        chan = torch.exp(torch.randn(HIDDEN, generator=g, device=device))
        x_all = torch.randn((TOKENS, HIDDEN), generator=g, device=device) * chan
        logits = torch.randn((TOKENS, LAYER_EXPERTS), generator=g, device=device)
        routed = torch.zeros((TOKENS, LAYER_EXPERTS), dtype=torch.bool, device=device)
        routed.scatter_(1, logits.topk(TOP_K, dim=1).indices, True)
        self.experts = []
        for e in experts:
            (gate, up, down), _, _ = make_triplet_weights(device, seed=5000 + 1000 * layer + e)
            if e == SHARED:
                x = x_all
            else:
                x = x_all[torch.nonzero(routed[:, e]).flatten()[:ROUTED_TOKENS]]
            h13 = (x.T @ x) / x.shape[0]
            act = torch.nn.functional.silu(x @ gate.float().T) * (x @ up.float().T)
            h2 = (act.T @ act) / x.shape[0]
            self.experts.append((e, (gate, up, down), h13.contiguous(), h2.contiguous()))
        del x_all, routed, logits

    @property
    def weights(self) -> int:
        return len(self.experts) * 3 * HIDDEN * INTER

    def groups(self, exl: dict) -> list:
        """quantize_uniform_batches groups of the given experts ({e: ([gate, up, down] EXL fp32, h13, h2)})."""
        from kquant_b200.ldlq import make_shared_h
        out = []
        for e, (ws, h13, h2) in exl.items():
            ks = self.rates[e]
            qa = [quant_args(m, self.device, layer=1000 * self.layer + e + 1, K=k)
                  for m, k in zip(("w1", "w3", "w2"), ks)]
            s13 = make_shared_h(HIDDEN, self.device, h13)
            if ks[0] == ks[1]:
                out.append(([ws[0], ws[1]], [s13, s13], qa[:2]))
            else:
                out.append(([ws[0]], [s13], qa[:1]))
                out.append(([ws[1]], [s13], qa[1:2]))
            out.append(([ws[2]], [make_shared_h(INTER, self.device, h2)], qa[2:]))
        return out

    def encode(self, experts=None, batch: int = 0):
        """Encode (a subset of) the rank's experts; returns [(expert, matrix, proxy)] and the outputs."""
        from kquant_b200 import exl3_encoder_backend as be
        todo = self.experts if experts is None else experts
        batch = batch or len(todo)
        proxies, outs = [], []
        for i in range(0, len(todo), batch):
            part = todo[i:i + batch]
            exl = {e: ([to_exl(w) for w in hf], h13, h2) for e, hf, h13, h2 in part}
            res = be.quantize_uniform_batches(self.groups(exl))
            flat = [r for grp in res for r in grp]
            for j, (e, _, _, _) in enumerate(part):
                proxies += [(e, m, flat[3 * j + m][0]) for m in range(3)]
            outs += flat
        return proxies, outs


def reduce_proxies(proxies, world: int) -> torch.Tensor:
    """One NCCL reduce of the per-tensor proxies into global slots (expert * 3 + matrix)."""
    from kquant_b200.sharding import reduce_proxy_stats
    slots = (LAYER_EXPERTS + 1) * 3
    num = torch.zeros(slots, dtype=torch.float64, device="cuda")
    den = torch.zeros(slots, dtype=torch.float64, device="cuda")
    if proxies:
        idx = torch.tensor([e * 3 + m for e, m, _ in proxies], device="cuda")
        num[idx] = torch.tensor([p for _, _, p in proxies], dtype=torch.float64, device="cuda")
        den[idx] = 1.0
    return reduce_proxy_stats(num, den)


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


def tile_encodes(k: int, n: int) -> int:
    """Tile encodes of one [k, n] matrix: every tile once, plus the global-scale search of
    ``sample_scale_tiles`` / ``g_scale_search_batch`` (10 coarse scales on a 1/3 subsample, 5 fine)."""
    tk, tn = k // 16, n // 16
    diag = max(tk, tn)
    samples = 3 * diag + 2 * min(max(8, 3 * diag // 16), (tk * tn + 1) // 2)
    return tk * tn + 10 * -(-samples // 3) + 5 * samples


def encodes_per_weight() -> float:
    """Tile encodes per weight of an expert triplet (gate, up [7168 x 2048], down [2048 x 7168])."""
    return (2 * tile_encodes(HIDDEN, INTER) + tile_encodes(INTER, HIDDEN)) / (3 * HIDDEN * INTER)


def cpu_tile_rate(seconds_target: float = 15.0, K: int = K_BITS):
    """Oracle (CPU restatement of the reference tile encoder) on all host cores: tiles/s and sample size."""
    import numpy as np
    from kquant_b200.codebooks import sqg_xor_cheb_t12_bytes
    from oracle import oracle as O
    cores = os.cpu_count() or 1
    lab = O.labels(O.CB_SQG, sqg_xor_cheb_t12_bytes(K).numpy())
    rng = np.random.default_rng(0)
    n = cores
    t0 = time.perf_counter()
    O.viterbi(K, lab, rng.standard_normal((n, 256)).astype(np.float32), CTX, threads=cores)
    dt = time.perf_counter() - t0
    reps = max(1, int(seconds_target / max(dt, 1e-3)))
    n2 = n * reps
    tiles = rng.standard_normal((n2, 256)).astype(np.float32)
    t0 = time.perf_counter()
    O.viterbi(K, lab, tiles, CTX, threads=cores)
    dt = time.perf_counter() - t0
    return n2 / dt, cores, n2


def _reference_cpu_backend():
    """The reference's encoder backend on the CPU (baseline/_ref), tile quantiser = the C oracle; or None."""
    ref = ROOT / "baseline" / "_ref"
    if not (ref / "kquant" / "exl3_encoder_backend.py").exists():
        return None
    from tests.golden.make_backend_fixtures import _load_reference_backend
    return _load_reference_backend(ref)


def run_reference(args, world, rank):
    """CPU arm.  Each step runs the reference's own block-LDLQ (``ldlq``: CPU torch feedback GEMMs, tile
    gather/scatter) over a 128 x 256 slice of an expert matrix with the C restatement of the reference tile
    encoder on all host threads, K cycling 2, 3, 4.  The rate is charged the workload's global-scale search
    (its tile encodes per weight, the same count the GPU arm performs).  Falls back to the tile encoder alone
    when the reference package is not installed in baseline/_ref."""
    if rank != 0:
        return
    from kquant_b200.codebooks import sqg_xor_cheb_t12_bytes
    cores = os.cpu_count() or 1
    be = _reference_cpu_backend()
    k, n = 128, 256
    scale_search = encodes_per_weight() * 256          # tile encodes per tile of the workload (>= 1)
    times, weights = [], 0
    g = torch.Generator().manual_seed(11)
    for i in range(args.warmup + args.steps):
        K = (2, 3, 4)[i % 3]
        W = torch.randn((k, n), generator=g)
        x = torch.randn((4 * k, k), generator=g)
        H = x.T @ x / x.shape[0] + 1e-2 * torch.eye(k)
        qa = {"K": K, "devices": ["cpu"], "tailbite_context": CTX,
              "sqg_e4m3_luts_by_bits": {b: sqg_xor_cheb_t12_bytes(b) for b in (2, 3, 4)}}
        t0 = time.perf_counter()
        if be is not None:
            L, _ = be.block_ldl(H.clone(), 16, qa, False)
            L[torch.arange(k), torch.arange(k)] = 0
            be.ldlq(W, L, qa)
        else:
            cpu_tile_rate(seconds_target=0.0, K=K)
        dt = time.perf_counter() - t0
        if i >= args.warmup:
            times.append(dt)
            weights += k * n
    sec = sum(times)
    v = weights / (sec * scale_search) / 1e6
    sample = (f"reference ldlq (CPU torch) + C tile encoder on {cores} threads over a {k}x{n} slice per step, "
              f"K cycling 2/3/4; charged {scale_search:.3f} tile encodes per tile (the workload's scale search)"
              if be is not None else f"C tile encoder on {cores} threads, {cores} tiles per step")
    line = {"metric": METRIC, "value": v, "unit": UNIT, "n_gpus": args.gpus, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": sec / max(len(times), 1) * 1e3, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f16 trellis / f32 LDLQ", "data": "synthetic",
            "config": {"workload": "moe_layer_slice", "sample": f"{k}x{n} per step"},
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
    if args.K in (2, 3, 4):
        labels = _native.build_labels(_native.KQ_CB_SQG, sqg_xor_cheb_t12_bytes(args.K).to(device), device)
    else:
        labels = _native.build_labels(_native.KQ_CB_MCG, None, device)
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


def run_microbench_case(args, local):
    """configs[3] tile microbench: --tiles (default 1,048,576) independent N(0, 1) tiles at each K = 1..8
    (production SQG codebook at K2..K4, procedural MCG elsewhere), identity Hessian (tile encoder only), C=128.
    One warm-up launch on 16 tiles per SM, then one timed launch of all tiles per K."""
    from kquant_b200 import _native
    from kquant_b200.codebooks import sqg_xor_cheb_t12_bytes
    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    g = torch.Generator(device=device).manual_seed(5)
    tiles = torch.randn((args.tiles, 256), generator=g, device=device)
    out = torch.empty_like(tiles)
    states = torch.empty((args.tiles, 256), dtype=torch.int16, device=device)
    sms = torch.cuda.get_device_properties(device).multi_processor_count
    peak = 2.0 * _native.measure_hfma2_rate(device)
    rows = {}
    for K in range(1, 9):
        if K in (2, 3, 4):
            labels = _native.build_labels(_native.KQ_CB_SQG, sqg_xor_cheb_t12_bytes(K).to(device), device)
        else:
            labels = _native.build_labels(_native.KQ_CB_MCG, None, device)
        _native.viterbi_encode(tiles[:16 * sms], K, labels, CTX)
        torch.cuda.synchronize()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        _native.viterbi_encode(tiles, K, labels, CTX, out=out, states=states)
        b.record()
        torch.cuda.synchronize()
        sec = a.elapsed_time(b) / 1e3
        relax = args.tiles * (2 * CTX + 256) * 65536
        rows[f"K{K}"] = {"s": round(sec, 3), "tiles_per_s": round(args.tiles / sec),
                         "mweights_per_s": round(args.tiles * 256 / sec / 1e6, 1),
                         "frac_of_fp16_alu_peak": round(3 * relax / sec / peak, 3)}
    print(json.dumps({"case": "microbench", "tiles": args.tiles, "tailbite_context": CTX,
                      "peak_fp16_ops": peak, "per_K": rows}))


def run_mla_case(args, local):
    """MLA attention projections at K=5 (procedural MCG codebook): q_b_proj 1536 -> 12288, kv_b_proj
    512 -> 16384 and o_proj 8192 -> 7168 (HF [out, in]; EXL [in, out]), bf16 weights with Student-t rows,
    Hessians from 8192 synthetic tokens of each input width (per-channel lognormal scales).  One step
    encodes all three through quantize_uniform_batches."""
    from kquant_b200 import _native
    from kquant_b200 import exl3_encoder_backend as be
    from kquant_b200.ldlq import make_shared_h
    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    _native.load()
    g = torch.Generator(device=device).manual_seed(31)
    shapes = {"q_b_proj": (12288, 1536), "kv_b_proj": (16384, 512), "o_proj": (7168, 8192)}
    mats = []
    for i, (name, (out_f, in_f)) in enumerate(shapes.items()):
        w = torch.randn((out_f, in_f), generator=g, device=device) * 0.015
        z = torch.randn((out_f, 5), generator=g, device=device)
        t = z[:, 0] / torch.sqrt((z[:, 1:] ** 2).sum(1) / 4)
        w = (w * (t.abs() / t.abs().median()).unsqueeze(1)).to(torch.bfloat16)
        x = torch.randn((TOKENS, in_f), generator=g, device=device) * torch.exp(torch.randn(in_f, generator=g,
                                                                                              device=device))
        h = ((x.T @ x) / TOKENS).contiguous()
        del x
        mats.append((name, to_exl(w), h, i))

    def step():
        groups = []
        for name, w, h, i in mats:
            qa = {"K": args.K, "mcg": True, "seed": 9000 + i, "sv_seed": 9500 + i, "sigma_reg": 0.025,
                  "devices": [str(device)], "apply_out_scales": False, "tailbite_context": CTX}
            groups.append(([w.clone()], [make_shared_h(w.shape[0], device, h)], [qa]))
        return be.quantize_uniform_batches(groups)

    for _ in range(max(args.warmup, 1)):
        step()
    torch.cuda.synchronize()
    _native.stats.reset(timing=True)
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(args.steps):
        res = step()
    b.record()
    torch.cuda.synchronize()
    t = a.elapsed_time(b) / 1e3 / args.steps
    vl, vbusy, vtiles, vrelax, vsum = _native.stats.viterbi_summary()
    peak = 2.0 * _native.measure_hfma2_rate(device) / 1e12
    weights = sum(w.numel() for _, w, _, _ in mats)
    print(json.dumps({"case": "mla", "K": args.K, "codebook": "mcg", "matrices": {n: list(s) for n, s in shapes.items()},
                      "weights": weights, "ms_per_step": t * 1e3, "mweights_per_s": weights / t / 1e6,
                      "proxies": {n: r[0][0] for (n, _, _, _), r in zip(mats, res)},
                      "viterbi_launches_per_step": vl // max(args.steps, 1),
                      "viterbi_busy_share": vbusy / (t * args.steps),
                      "viterbi_frac_of_fp16_peak": 3.0 * vrelax / vbusy / 1e12 / peak if vbusy else None}))


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
    n = 3 * HIDDEN * INTER // 256
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


def run_reconstruct_case(args, local):
    """Row W: the original-basis reconstruction of the triplet's three matrices on the Walsh-Hadamard kernel
    (HBM-bound: one read and one write of each matrix), against the matmul form (two fp32 block GEMMs and
    two scalings, as kquant/exl3_encoder_backend.py:2211-2216 computes it)."""
    from kquant_b200 import _native
    from kquant_b200 import exl3_encoder_backend as be
    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    g = torch.Generator(device=device).manual_seed(3)
    mats = [(torch.randn(s, generator=g, device=device), torch.randn(s[0], generator=g, device=device),
             torch.randn(s[1], generator=g, device=device)) for s in ((HIDDEN, INTER), (HIDDEN, INTER),
                                                                       (INTER, HIDDEN))]
    peak, src = _hbm_peak()
    byt = sum(w.numel() for w, _, _ in mats) * 8
    t = _time(lambda: [_native.reconstruct_rotated(w, u, v) for w, u, v in mats], args.steps, args.warmup)

    def matmul_form():
        for w, u, v in mats:
            x = be.preapply_had_l(w, 128)
            x *= u.unsqueeze(1)
            x = be.preapply_had_r(x, 128)
            x *= v.unsqueeze(0)

    tm = _time(matmul_form, args.steps, args.warmup)
    print(json.dumps({"case": "reconstruct", "weights": sum(w.numel() for w, _, _ in mats), "bytes": byt,
                      "ms": t * 1e3, "gbs": byt / t / 1e9, "frac_of_hbm": byt / t / 1e9 / peak, "peak_source": src,
                      "matmul_form_ms": tm * 1e3}))


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
    """Kernel list of one warm step of the default workload (torch.profiler / CUPTI device times): every launch
    of the step with its device time, grouped by kernel, plus the step's wall time (CUDA events), so the
    device-idle share is visible; a launch list without a replaying profiler."""
    from torch.profiler import ProfilerActivity, profile
    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    from kquant_b200 import _native
    _native.load()
    wl = SliceWorkload(args, 1, 0, device)
    for _ in range(max(args.warmup, 1)):
        wl.step()
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with profile(activities=[ProfilerActivity.CUDA]) as prof:
        a.record()
        wl.step()
        b.record()
        torch.cuda.synchronize()
    rows = sorted(prof.key_averages(), key=lambda e: -e.device_time_total)
    total = sum(e.device_time_total for e in rows)
    wall = a.elapsed_time(b)
    # the longest device-idle gaps between consecutive kernels (where the host held the GPU back)
    evs = sorted((e.time_range.start, e.time_range.end, e.name) for e in prof.events()
                 if e.device_type.name == "CUDA" and e.time_range.end > e.time_range.start)
    gaps, last_end, last_name = [], None, None
    for st, en, name in evs:
        if last_end is not None and st > last_end:
            gaps.append((st - last_end, last_name[:60], name[:60]))
        if last_end is None or en > last_end:
            last_end, last_name = en, name
    gaps.sort(reverse=True)
    print(json.dumps({"case": "profile", "workload": wl.config["workload"], "step_ms": wall,
                      "gap_total_ms": sum(g for g, _, _ in gaps) / 1e3,
                      "top_gaps_us": [[round(g, 1), x, y] for g, x, y in gaps[:12]],
                      "device_busy_ms": total / 1e3, "idle_share": 1 - total / 1e3 / wall, "kernels": [
                          {"name": e.key[:120], "launches": e.count, "ms": e.device_time_total / 1e3,
                           "share": e.device_time_total / total} for e in rows[:args.top]]}, indent=1))


class SliceWorkload:
    """The default step: this rank's first ``experts`` experts of its shard of the layer."""

    def __init__(self, args, world, rank, device):
        from kquant_b200.sharding import shard_experts
        mine = shard_experts([1.0] * LAYER_EXPERTS, world, rank)[:args.experts]
        self.layer = Layer(device, mine)
        self.device = device
        self.weights = self.layer.weights
        self.exl = {e: [to_exl(w) for w in hf] for e, hf, _, _ in self.layer.experts}
        ks = [k for e in mine for k in self.layer.rates[e]]
        self.config = {"workload": "moe_layer_slice", "experts_per_gpu": len(mine),
                       "experts": f"{mine[0]}..{mine[-1]} of {LAYER_EXPERTS} (shard of rank {rank})",
                       "matrices": "gate,up [7168x2048] + down [2048x7168] per expert (EXL k x n)",
                       "K_per_tensor": ks, "bpw_layer": 3.2, "hessian_tokens_per_expert": ROUTED_TOKENS,
                       "codebook": "sqg_xor_cheb_t12", "tailbite_context": CTX,
                       "l2": "inputs larger than L2 (per expert: bf16 weights 88 MB + H 222 MB)"}

    def step(self):
        from kquant_b200 import exl3_encoder_backend as be
        exl = {e: ([w.clone() for w in self.exl[e]], h13, h2) for e, _, h13, h2 in self.layer.experts}
        res = be.quantize_uniform_batches(self.layer.groups(exl))
        flat = [r for grp in res for r in grp]
        return [(e, m, flat[3 * i + m][0]) for i, (e, _, _, _) in enumerate(self.layer.experts) for m in range(3)], flat

    def host_inputs(self):
        w = [w.cpu().pin_memory() for _, hf, _, _ in self.layer.experts for w in hf]
        h = [t.cpu().pin_memory() for _, _, h13, h2 in self.layer.experts for t in (h13, h2)]
        return w, h

    def step_e2e(self, host):
        """Pinned host bf16 weights + fp32 Hessians -> device -> encode -> packed outputs back on the host."""
        from kquant_b200 import exl3_encoder_backend as be
        hw, hh = host
        exl = {}
        for i, (e, _, _, _) in enumerate(self.layer.experts):
            ws = [to_exl(w.to(self.device, non_blocking=True)) for w in hw[3 * i:3 * i + 3]]
            exl[e] = (ws, hh[2 * i].to(self.device, non_blocking=True), hh[2 * i + 1].to(self.device, non_blocking=True))
        res = be.quantize_uniform_batches(self.layer.groups(exl))
        flat = [r for grp in res for r in grp]
        host_out = [{k: v.cpu() for k, v in o[1].items()} for o in flat]
        proxies = torch.tensor([o[0] for o in flat], dtype=torch.float64)
        return sum(v.numel() * v.element_size() for o in host_out for v in o.values()) + proxies.numel() * 8


class TripletWorkload:
    """configs[1]-style single triplet at one K, Hessians from 8192 tokens."""

    def __init__(self, args, world, rank, device, K=None):
        self.K = K or args.K
        self.device = device
        self.hf, self.h13, self.h2 = make_triplet(device, seed=1234 + rank)
        self.exl = [to_exl(w) for w in self.hf]
        self.weights = 3 * HIDDEN * INTER
        self.config = {"workload": f"kimi_expert_triplet_k{self.K}",
                       "matrices": "gate,up [7168x2048] + down [2048x7168] (EXL k x n)", "K": self.K,
                       "codebook": "sqg_xor_cheb_t12", "tailbite_context": CTX, "tokens": TOKENS,
                       "l2": "inputs larger than L2 (bf16 weights 88 MB + H 222 MB per step)"}

    def step(self):
        res = encode_triplet([w.clone() for w in self.exl], self.h13, self.h2, self.device, K=self.K)
        return [(0, m, r[0]) for m, r in enumerate(res)], res

    def host_inputs(self):
        return [w.cpu().pin_memory() for w in self.hf], [self.h13.cpu().pin_memory(), self.h2.cpu().pin_memory()]

    def step_e2e(self, host):
        hw, hh = host
        dw = [w.to(self.device, non_blocking=True) for w in hw]
        dh13, dh2 = (h.to(self.device, non_blocking=True) for h in hh)
        out = encode_triplet([to_exl(w) for w in dw], dh13, dh2, self.device, K=self.K)
        host_out = [{k: v.cpu() for k, v in o[1].items()} for o in out]
        proxies = torch.tensor([o[0] for o in out], dtype=torch.float64)
        return sum(v.numel() * v.element_size() for o in host_out for v in o.values()) + proxies.numel() * 8


def per_k_rates(args, device) -> dict:
    """Triplet (configs[1] shapes) Mweights/s at K = 2, 3, 4: one warm-up and one timed step each."""
    out = {}
    for K in (2, 3, 4):
        wl = TripletWorkload(args, 1, 0, device, K=K)
        wl.step()
        torch.cuda.synchronize()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        wl.step()
        b.record()
        torch.cuda.synchronize()
        out[f"K{K}"] = round(wl.weights / (a.elapsed_time(b) / 1e3) / 1e6, 2)
        del wl
    return out


def run_encode(args, world, rank, local):
    """The measured encode: K timed steps of the workload (HBM-resident), then the end-to-end leg."""
    from kquant_b200 import _native
    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    _native.load()
    wl = TripletWorkload(args, world, rank, device) if args.case == "triplet" else \
        SliceWorkload(args, world, rank, device)
    for _ in range(args.warmup):
        wl.step()
    torch.cuda.synchronize()
    if world > 1:
        torch.distributed.barrier()
    _native.stats.reset(timing=True)
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clk:
        torch.cuda.synchronize()
        start.record()
        for _ in range(args.steps):
            proxies, _ = wl.step()
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
    # one reduce of the per-tensor proxy statistics, after the timed steps
    global_proxy = reduce_proxies(proxies, world)
    proxy_max = float(global_proxy.max())

    # end-to-end: pinned host inputs -> device -> encode -> host outputs
    host = wl.host_inputs()
    h2d = sum(t.numel() * t.element_size() for part in host for t in part)
    if args.e2e_steps > 0:
        wl.step_e2e(host)                 # untimed: first-use allocations of the host-input path
    torch.cuda.synchronize()
    if world > 1:
        torch.distributed.barrier()
    es, ee = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    es.record()
    d2h = 0
    for _ in range(max(args.e2e_steps, 0)):
        d2h = wl.step_e2e(host)
    ee.record()
    torch.cuda.synchronize()
    e_elapsed = max(_allreduce_max(es.elapsed_time(ee) / 1e3, world), 1e-9)

    total_weights = wl.weights * world
    value = total_weights * args.steps / elapsed / 1e6
    e2e = total_weights * args.e2e_steps / e_elapsed / 1e6
    hfma2 = _native.measure_hfma2_rate(device)
    peak_ops = 2.0 * hfma2 / 1e12                       # fp16 ops/s (two lanes per HFMA2)
    achieved_ops = 3.0 * vrelax / vsec / 1e12 if vsec > 0 else None
    traffic = None
    tpath = ROOT / "profiles" / "viterbi_dram_bytes_per_tile.txt"
    if tpath.exists() and vl:
        try:
            traffic = float(tpath.read_text().split()[0]) * median_tiles
        except (ValueError, IndexError):
            traffic = None
    line = {
        "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": elapsed / args.steps * 1e3, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f16 trellis / f32 LDLQ", "data": "synthetic",
        "config": {**wl.config, "parallelism": f"expert-sharded x{world}"},
        "e2e": {"value": e2e, "unit": UNIT, "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h},
        "gpu_launches": launches,
        "roofline": {"bound": "alu", "kernel": "kq pair_kernel (Viterbi)", "achieved": achieved_ops,
                     "peak": peak_ops, "unit": "Tops/s fp16 (3 ops per relaxation)",
                     "frac": (achieved_ops / peak_ops) if achieved_ops else None,
                     "traffic": traffic,
                     "traffic_source": "ncu dram bytes per tile of one chain launch (profiles/"
                                       "viterbi_dram_bytes_per_tile.txt) x the median launch's tiles",
                     "launches": vl, "avg_launch_ms": vsum / vl * 1e3 if vl else None,
                     "busy_ms": vsec * 1e3,
                     "timing": "achieved = relaxations / union of the Viterbi launch intervals (CUDA events "
                               "on the launching stream)",
                     "peak_source": "measured HFMA2 rate (kq_probe_hfma2) x 2 lanes, this GPU, this run"},
        "viterbi_share_of_step": vsec / elapsed if elapsed else None,
        "proxy_max": proxy_max,
        "clocks": clocks,
    }
    if world == 1 and args.case != "triplet" and not args.no_per_k:
        line["per_K_triplet_mweights_s"] = per_k_rates(args, device)
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        rate, cores, n = cpu_tile_rate()
        cpu_v = rate / encodes_per_weight() / 1e6
        line["cpu_baseline"] = {"value": cpu_v, "unit": UNIT, "cores": cores, "kind": "port",
                                "sample": f"{n} tiles of the K={K_BITS} C={CTX} Viterbi (C oracle) on {cores} "
                                          f"threads, charged {encodes_per_weight() * 256:.3f} tile encodes per "
                                          f"tile (the workload's scale search)"}
    if rank == 0:
        print(json.dumps(line), flush=True)


def run_layer_case(args, world, rank, local):
    """The whole layer once: 384 routed experts + the shared expert over the ranks (48 + 1 at 8 GPUs), encoded
    in batches of --experts; reports the wall time (device events, max over ranks) and Mweights/s.  With one
    process and --layer-ranks N, that process encodes the last (longest) of the N shards alone: the ranks share
    no data, so an N-GPU run's wall time is its slowest shard's."""
    from kquant_b200 import _native
    from kquant_b200.sharding import shard_experts
    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    _native.load()
    ranks = args.layer_ranks or world
    if world not in (1, ranks):
        raise SystemExit("--layer-ranks must equal the number of processes (or run one process)")
    # one process standing in for rank ranks-1 of a ranks-GPU run: that shard only (it also holds the
    # shared expert, so it is the longest); the layer's wall time on `ranks` GPUs is this shard's time
    shard = rank if world == ranks else ranks - 1
    mine = shard_experts([1.0] * LAYER_EXPERTS, ranks, shard)
    if shard == ranks - 1:
        mine = mine + [SHARED]
    layer = Layer(device, mine)
    layer.encode(layer.experts[:1])            # warm-up: one expert
    torch.cuda.synchronize()
    if world > 1:
        torch.distributed.barrier()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clk:
        a.record()
        proxies, _ = layer.encode(batch=args.experts)
        b.record()
        torch.cuda.synchronize()
    if world > 1:
        torch.distributed.barrier()
    t = _allreduce_max(a.elapsed_time(b) / 1e3, world)
    gp = reduce_proxies(proxies, world)
    total = (LAYER_EXPERTS + 1) * 3 * HIDDEN * INTER
    if rank == 0:
        ks = [k for row in layer.rates for k in row]
        print(json.dumps({"case": "layer", "experts": LAYER_EXPERTS + 1, "weights": total, "n_gpus": world,
                          "layer_ranks": ranks, "one_shard_on_one_gpu": world != ranks,
                          "experts_per_gpu": len(mine), "bpw_mean": sum(ks) / len(ks),
                          "wall_s": t, "mweights_per_s": total / t / 1e6,
                          "proxy_mean": float(gp.mean()), "proxy_max": float(gp.max()),
                          "clocks": clk.summary(), "data": "synthetic"}), flush=True)


def run_stream_case(args, world, rank, local):
    """configs[4]-style streaming: --layers consecutive MoE layers, each rank encoding --experts experts of its
    shard of every layer.  Layer l+1's synthetic weights and Hessians are generated on the device, from a seed,
    on a side stream while layer l encodes; each layer's packed trellis and scales go back to pinned host
    memory on a third stream.  Reports sustained encoded weights/s over the whole stream (device events,
    max over ranks)."""
    from kquant_b200 import _native
    from kquant_b200 import exl3_encoder_backend as be
    from kquant_b200.sharding import shard_experts
    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    _native.load()
    main_stream = torch.cuda.current_stream(device)
    gen_stream, out_stream = torch.cuda.Stream(device), torch.cuda.Stream(device)
    mine = shard_experts([1.0] * LAYER_EXPERTS, world, rank)[:args.experts]

    def generate(layer):
        with torch.cuda.stream(gen_stream):
            lay = Layer(device, mine, layer=layer)
            exl = {e: ([to_exl(w) for w in hf], h13, h2) for e, hf, h13, h2 in lay.experts}
            ready = gen_stream.record_event()
        return lay, exl, ready

    warm = Layer(device, mine[:1], layer=args.layers)        # warm-up: one expert of a layer outside the stream
    warm.encode()
    del warm
    torch.cuda.synchronize()
    if world > 1:
        torch.distributed.barrier()
    host_out, pending = [], []
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clk:
        a.record()
        nxt = generate(0)
        for layer in range(args.layers):
            lay, exl, ready = nxt
            main_stream.wait_event(ready)
            for ws, h13, h2 in exl.values():
                for t in (*ws, h13, h2):
                    t.record_stream(main_stream)
            if layer + 1 < args.layers:
                nxt = generate(layer + 1)
            res = be.quantize_uniform_batches(lay.groups(exl))
            done = main_stream.record_event()
            with torch.cuda.stream(out_stream):
                out_stream.wait_event(done)
                for grp in res:
                    for _, tens in grp:
                        for v in tens.values():
                            v.record_stream(out_stream)
                            dst = torch.empty(v.shape, dtype=v.dtype, pin_memory=True)
                            dst.copy_(v, non_blocking=True)
                            host_out.append(dst)
            pending.append(res)
        main_stream.wait_stream(out_stream)
        b.record()
        torch.cuda.synchronize()
    if world > 1:
        torch.distributed.barrier()
    t = _allreduce_max(a.elapsed_time(b) / 1e3, world)
    weights = args.layers * len(mine) * 3 * HIDDEN * INTER * world
    proxies = [p for res in pending for grp in res for p, _ in grp]
    if rank == 0:
        print(json.dumps({"case": "stream", "layers": args.layers, "experts_per_gpu_per_layer": len(mine),
                          "n_gpus": world, "weights": weights, "wall_s": t,
                          "sustained_mweights_per_s": weights / t / 1e6,
                          "d2h_bytes": sum(x.numel() * x.element_size() for x in host_out),
                          "proxy_max": max(proxies), "clocks": clk.summary(),
                          "data": "synthetic, generated on the device per layer"}), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=3)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="kq", choices=["kq", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-per-k", action="store_true")
    ap.add_argument("--e2e-steps", type=int, default=2)
    ap.add_argument("--case", default="slice",
                    choices=["slice", "triplet", "layer", "stream", "qsrt", "chain", "viterbi", "microbench", "mla", "trace",
                             "pack", "load", "hessian", "profile", "reconstruct"],
                    help="viterbi: only the tile kernel on --tiles random tiles (profiling case)")
    ap.add_argument("--tiles", type=int, default=None, help="viterbi: 1184; microbench: 1,048,576")
    ap.add_argument("--K", type=int, default=K_BITS)
    ap.add_argument("--tokens", type=int, default=TOKENS, help="hessian case: samples per call")
    ap.add_argument("--dim", type=int, default=HIDDEN, help="hessian case: sample width")
    ap.add_argument("--experts", type=int, default=4, help="slice: experts per GPU; layer: experts per batch")
    ap.add_argument("--top", type=int, default=25, help="profile case: kernels listed")
    ap.add_argument("--layers", type=int, default=8, help="stream case: consecutive layers")
    ap.add_argument("--layer-ranks", type=int, default=0,
                    help="layer case: GPUs the layer is sharded over; one process runs the last shard alone")
    args = ap.parse_args()
    if args.tiles is None:
        args.tiles = 1 << 20 if args.case == "microbench" else 1184
    if args.case == "mla" and args.K == K_BITS:
        args.K = 5
    world, rank, local = _dist()
    cases = {"profile": run_profile_case, "chain": run_chain_case, "qsrt": run_qsrt_case,
             "viterbi": run_viterbi_case, "trace": run_trace_case, "pack": run_pack_case, "load": run_load_case,
             "hessian": run_hessian_case, "microbench": run_microbench_case, "mla": run_mla_case,
             "reconstruct": run_reconstruct_case}
    if args.case in cases:
        cases[args.case](args, local)
    elif args.impl == "reference":
        run_reference(args, world, rank)
    elif args.case == "layer":
        run_layer_case(args, world, rank, local)
    elif args.case == "stream":
        run_stream_case(args, world, rank, local)
    else:
        run_encode(args, world, rank, local)
    if world > 1:
        torch.distributed.barrier()
        torch.distributed.destroy_process_group()


if __name__ == "__main__":
    main()
