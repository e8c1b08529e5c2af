"""Seeded inputs of the end-to-end backend fixtures (shared by generator and tests)."""
import torch

from kquant_b200.codebooks import sqg_xor_cheb_t12_bytes

CASES = {
    "k4_uniform": {"k": 256, "n": 256, "K": 4, "ctx": 32, "seed": 11},
    "k3_c128": {"k": 256, "n": 128, "K": 3, "ctx": 128, "seed": 12},
}


def make_inputs(case, device):
    g = torch.Generator().manual_seed(case["seed"])
    k, n = case["k"], case["n"]
    w = torch.randn((k, n), generator=g) * 0.02
    w[torch.rand((k, n), generator=g) < 0.001] *= 10
    x = torch.randn((4 * k, k), generator=g) * torch.exp(torch.randn(k, generator=g))
    h = x.T @ x / x.shape[0]
    h += 1e-2 * h.diagonal().mean() * torch.eye(k)
    args = {"K": case["K"], "seed": 1000 + case["seed"], "sv_seed": 2000 + case["seed"], "sigma_reg": 0.025,
            "devices": [str(device)], "apply_out_scales": None, "tailbite_context": case["ctx"],
            "sqg_e4m3_luts_by_bits": {b: sqg_xor_cheb_t12_bytes(b) for b in (2, 3, 4)}}
    return w.to(device), h.to(device), args


# quantize_uniform_batch fixtures: two matrices sharing one H (gate/up style), and
# two matrices with distinct Hessians (stacked members)
UNIFORM_CASES = {
    "uniform_pair_k3": {"k": 256, "n": 256, "K": 3, "ctx": 128, "seed": 13},
    "uniform_distinct_k4": {"k": 256, "n": 128, "K": 4, "ctx": 32, "seed": 14, "distinct": True},
}


def make_uniform_inputs(case, device):
    """([w1, w2], [h1, h2], [args1, args2]); h2 is h1 unless the case has distinct Hessians."""
    w1, h1, a1 = make_inputs(case, device)
    w2, h2, _ = make_inputs(dict(case, seed=case["seed"] + 100), device)
    a2 = dict(a1, sv_seed=a1["sv_seed"] + 1)
    a2["sqg_e4m3_luts_by_bits"] = a1["sqg_e4m3_luts_by_bits"]
    return [w1, w2], [h1, h2 if case.get("distinct") else h1], [a1, a2]
