"""Expert/tensor sharding of the encode across the GPUs of one box.

The encode shards with no data-path exchange (one process per GPU, each
encoding its own experts; kquant's own driver does the same with OS processes,
scripts/pack_qsrt_candidates.py:1558-1733).  Two small cross-rank couplings
remain, both over torch.distributed (NCCL on GPUs, gloo in CPU tests):

* the per-tensor proxy statistics (numerator / denominator of
  tr(dW H dW^T) / tr(W H W^T)) are summed once at the end;
* optionally, the layer-shared input-scale profile (``shared_input_scales_key``,
  kquant/exl3_encoder_backend.py:1964-1973) is computed by the rank that owns
  the layer's first expert and broadcast as one [k, 1] vector, instead of
  every rank re-encoding that expert as a primer.
"""

from __future__ import annotations

import torch
import torch.distributed as dist


def shard_experts(expert_costs: list[float], world: int, rank: int) -> list[int]:
    """Contiguous expert ranges with balanced total cost (greedy prefix split).

    Equal costs give equal contiguous blocks (384 experts / 8 GPUs = 48 each).
    Every expert is assigned to exactly one rank.
    """
    if world < 1 or not 0 <= rank < world:
        raise ValueError("rank must be in [0, world)")
    n = len(expert_costs)
    if any(c <= 0 for c in expert_costs):
        raise ValueError("expert costs must be positive")
    total = float(sum(expert_costs))
    bounds = [0]
    acc = 0.0
    for i, c in enumerate(expert_costs):
        acc += c
        # close a shard once its share of the total is reached, keeping enough experts for the rest
        while len(bounds) < world and acc >= total * len(bounds) / world and n - (i + 1) >= world - len(bounds):
            bounds.append(i + 1)
    while len(bounds) < world:
        bounds.append(n)
    bounds.append(n)
    return list(range(bounds[rank], bounds[rank + 1]))


def reduce_proxy_stats(numerators: torch.Tensor, denominators: torch.Tensor, group=None) -> torch.Tensor:
    """Sum per-tensor proxy numerators/denominators over ranks; returns the global proxy per tensor slot.

    Each rank passes vectors indexed by a global tensor slot, with zeros for
    tensors it does not own.
    """
    stats = torch.stack((numerators.double(), denominators.double()))
    if dist.is_available() and dist.is_initialized():
        dist.all_reduce(stats, op=dist.ReduceOp.SUM, group=group)
    return stats[0] / stats[1].clamp_min(1e-8)


def broadcast_shared_input_scales(key, scales: torch.Tensor | None, src: int, shape, device, group=None):
    """Publish one rank's input-scale profile under ``key`` on every rank."""
    from .exl3_encoder_backend import _SHARED_INPUT_SCALES
    buf = scales.detach().to(device=device, dtype=torch.float32).contiguous() if scales is not None else \
        torch.empty(shape, dtype=torch.float32, device=device)
    if dist.is_available() and dist.is_initialized():
        dist.broadcast(buf, src=src, group=group)
    _SHARED_INPUT_SCALES[key] = buf
    return buf
