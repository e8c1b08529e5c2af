"""Seeded problems of the CUDA reference fixtures (shared by the generator and the GPU tests).

The reference backend and this backend both run on a B200 with these exact
inputs: weights and activations are drawn from a CPU ``torch.Generator``
(bit-identical on every host) and moved to the device; Hessians are formed on
the device with fp32 cuBLAS (TF32 off), which is deterministic for one shape
on one GPU model.  ``digest`` hashes a tensor's bytes; the fixture file
records digests and a few scalars instead of the (large) tensors themselves.

Shapes follow the benchmark configurations of the encode path:

* ``cfg0_2048_k4``: the single dense linear, W 2048 x 2048 ~ N(0, 0.02) with
  0.1 % outliers x10, H from 4096 tokens with per-channel lognormal scales plus
  1e-2 mean-diagonal damping, K=4, production SQG codebook, C=128.
* ``cfg1_slice_7168_k3``: a 256-column slice of the gate projection of one
  expert triplet (EXL k = 7168: 448 LDLQ steps, 56 buffers), Student-t rows,
  H from 8192 tokens, K=3.
* ``mla_kvb_slice_k5``: a 1024-column slice of an MLA kv_b_proj (EXL k = 512)
  at K=5 on the procedural MCG codebook, H from 2048 tokens.  The reference
  host rejects K=5, so its tile quantiser here is the reference kernel
  template launched at K=5 (oracle/ref_harness.cu).
* ``batch_n_r012`` / ``batch_k_r012``: kquant's production call
  ``quantize_qsrt_batch`` over two sources x the rate-transfer modes
  R0/R1/R2, along n (gate-like, the n-axis candidate reuse) and along k
  (down-like, the k-axis prefix trie).
* ``uniform_pair_1024_k3``: ``quantize_uniform_batch`` of two matrices that
  share one Hessian (gate/up).
"""
from __future__ import annotations

import hashlib

import torch

from kquant_b200.codebooks import sqg_xor_cheb_t12_bytes

QSRT_CASES = {
    "cfg0_2048_k4": {"kind": "dense", "k": 2048, "n": 2048, "K": 4, "tokens": 4096, "seed": 21},
    "cfg1_slice_7168_k3": {"kind": "triplet_slice", "k": 7168, "n": 256, "K": 3, "tokens": 8192, "seed": 22},
    # MLA kv_b_proj-like slice (EXL k = 512 latent rows) at K=5 on the procedural MCG codebook
    "mla_kvb_slice_k5": {"kind": "dense", "k": 512, "n": 1024, "K": 5, "tokens": 2048, "seed": 23,
                         "codebook": "mcg"},
}

BATCH_CASES = {
    "batch_n_r012": {"axis": "n", "k": 1024, "n": 1024, "sources": 2, "tokens": 256, "seed": 31},
    "batch_k_r012": {"axis": "k", "k": 1024, "n": 512, "sources": 2, "tokens": 256, "seed": 32},
}

UNIFORM_CASES = {
    "uniform_pair_1024_k3": {"k": 1024, "n": 512, "K": 3, "tokens": 2048, "seed": 41},
}


def digest(t: torch.Tensor) -> str:
    """SHA-256 of a tensor's bytes (contiguous, on the host)."""
    return hashlib.sha256(t.detach().contiguous().cpu().numpy().tobytes()).hexdigest()


def row_digests(states: torch.Tensor) -> list[str]:
    """Short digest per tile row of [k/16, n/16, 256] states (where a divergence starts)."""
    s = states.detach().contiguous().cpu()
    return [hashlib.sha256(s[i].numpy().tobytes()).hexdigest()[:12] for i in range(s.shape[0])]


def sample_index(numel: int, count: int = 1024, seed: int = 5) -> torch.Tensor:
    g = torch.Generator().manual_seed(seed)
    return torch.randint(0, numel, (count,), generator=g)


def _hessian(x_cpu: torch.Tensor, device, damp: float | None) -> torch.Tensor:
    previous = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    try:
        x = x_cpu.to(device)
        h = (x.T @ x) / x.shape[0]
        if damp:
            h += damp * h.diagonal().mean() * torch.eye(h.shape[0], device=device)
        return h.contiguous()
    finally:
        torch.backends.cuda.matmul.allow_tf32 = previous


def _student_rows(g: torch.Generator, rows: int, cols: int, std: float) -> torch.Tensor:
    w = torch.randn((rows, cols), generator=g) * std
    z = torch.randn((rows, 5), generator=g)
    t = z[:, 0] / torch.sqrt((z[:, 1:] ** 2).sum(1) / 4)
    return w * (t.abs() / t.abs().median()).unsqueeze(1)


def base_args(K: int, seed: int, device, codebook: str = "sqg") -> dict:
    args = {"K": K, "seed": 1000 + seed, "sv_seed": 2000 + seed, "sigma_reg": 0.025, "devices": [str(device)],
            "apply_out_scales": None, "tailbite_context": 128}
    if codebook == "sqg":
        args["sqg_e4m3_luts_by_bits"] = {b: sqg_xor_cheb_t12_bytes(b) for b in (2, 3, 4)}
    else:
        args[codebook] = True
    return args


def qsrt_inputs(name: str, device):
    """(W [k, n] fp32 on device, H [k, k] fp32 on device, quant_args) of a quantize_qsrt case."""
    c = QSRT_CASES[name]
    g = torch.Generator().manual_seed(c["seed"])
    k, n = c["k"], c["n"]
    if c["kind"] == "dense":
        w = torch.randn((k, n), generator=g) * 0.02
        w[torch.rand((k, n), generator=g) < 0.001] *= 10
        w = w.to(torch.bfloat16).float()
        x = torch.randn((c["tokens"], k), generator=g) * torch.exp(torch.randn(k, generator=g))
        h = _hessian(x, device, 1e-2)
    else:
        # HF gate [n_out, 7168] rows ~ N(0, 0.015) x |t4|; EXL orientation is its transpose
        w = _student_rows(g, n, k, 0.015).to(torch.bfloat16).float().T.contiguous()
        x = torch.randn((c["tokens"], k), generator=g) * torch.exp(torch.randn(k, generator=g))
        h = _hessian(x, device, None)
    return w.to(device), h, base_args(c["K"], c["seed"], device, c.get("codebook", "sqg"))


def batch_inputs(name: str, device):
    """(sources [k, n] list, Hessians list, quant_args_groups) of a quantize_qsrt_batch case (R0/R1/R2)."""
    from kquant_b200 import qsrt
    c = BATCH_CASES[name]
    g = torch.Generator().manual_seed(c["seed"])
    k, n = c["k"], c["n"]
    ws, hs, groups = [], [], []
    for s in range(c["sources"]):
        ws.append((torch.randn((k, n), generator=g) * 0.02).to(torch.bfloat16).float().to(device))
        x = torch.randn((c["tokens"], k), generator=g) * torch.exp(torch.randn(k, generator=g))
        hs.append(_hessian(x, device, 1e-2))
        base = base_args(3, c["seed"] * 10 + s, device)
        extent = (n if c["axis"] == "n" else k) // 128
        cands = []
        for mode in qsrt.RATE_TRANSFER_MODES:
            rec = qsrt.record_bits(mode)[:extent]
            if len(rec) < extent:
                raise ValueError("rate map shorter than the matrix")
            bits = tuple(b for b in rec for _ in range(8))
            cands.append(dict(base, mixed_rate_axis=c["axis"], mixed_tile_bits=bits))
        groups.append(cands)
    return ws, hs, groups


def uniform_inputs(name: str, device):
    """([w1, w2], shared H, [args1, args2]) of a quantize_uniform_batch case (two matrices, one Hessian)."""
    c = UNIFORM_CASES[name]
    g = torch.Generator().manual_seed(c["seed"])
    k, n = c["k"], c["n"]
    ws = [(torch.randn((k, n), generator=g) * 0.02).to(torch.bfloat16).float().to(device) for _ in range(2)]
    x = torch.randn((c["tokens"], k), generator=g) * torch.exp(torch.randn(k, generator=g))
    h = _hessian(x, device, 1e-2)
    a1 = base_args(c["K"], c["seed"], device)
    a2 = dict(a1, sv_seed=a1["sv_seed"] + 1)
    return ws, h, [a1, a2]


class Capture:
    """Wraps a module's ``ldlq``/``ldlq_mixed`` and keeps the first call's rotated inputs."""

    def __init__(self, module):
        self.module = module
        self.saved = {}
        self.inputs = None

    def __enter__(self):
        for name in ("ldlq", "ldlq_mixed"):
            fn = getattr(self.module, name)
            self.saved[name] = fn

            def wrapped(weight, L, quant_args, pb=None, _fn=fn):
                if self.inputs is None:
                    self.inputs = (weight.detach().clone(), L.detach().clone())
                return _fn(weight, L, quant_args, pb)

            setattr(self.module, name, wrapped)
        return self

    def __exit__(self, *exc):
        for name, fn in self.saved.items():
            setattr(self.module, name, fn)
