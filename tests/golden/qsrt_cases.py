"""Seeded legal QSRT matrices shared by the fixture generator and the GPU tests."""
import numpy as np
import torch

RECORD_BITS_BY_MODE = None   # filled lazily from the module under test


def legal_states(shape, record_bits, rate_axis, seed):
    """Random K-bit edges per 128-channel record, closed into cyclic 16-bit states."""
    g = torch.Generator().manual_seed(seed)
    states = torch.empty(shape, dtype=torch.int16)
    for r, bits in enumerate(record_bits):
        sl = slice(8 * r, 8 * r + 8)
        sub = (8, shape[1], 256) if rate_axis == "k" else (shape[0], 8, 256)
        edges = torch.randint(0, 1 << bits, sub, generator=g).numpy().astype(np.int64)
        st = np.zeros_like(edges)
        for lag in range((16 + bits - 1) // bits):
            st |= np.roll(edges, lag, axis=-1) << (lag * bits)
        st = torch.from_numpy((st & 0xFFFF).astype(np.uint16).view(np.int16))
        if rate_axis == "k":
            states[sl] = st
        else:
            states[:, sl] = st
    return states


def scales(k, n, seed):
    g = torch.Generator().manual_seed(seed)
    return ((torch.rand(k, generator=g) + 0.5).half(), (torch.rand(n, generator=g) + 0.5).half())


CASES = [(mode, axis) for mode in (0, 1, 2) for axis in ("k", "n")]
SHAPES = {"k": (192, 224, 256), "n": (224, 192, 256)}
