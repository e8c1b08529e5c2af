"""The allocation-free entry point gives the same codes and values as the workspace one.

kq_quantize_tiles_sqg_noalloc exists for callers that cannot allocate device
memory (their host owns the device allocator, or an allocation at that point
would stall them).  It keeps its scratch in a fixed __device__ array, so two
calls in a row reuse the same memory; the second call must not see stale
state from the first.  This file is collected last on purpose.
"""
import ctypes

import pytest
import torch

from kquant_b200 import codebooks as cb

pytestmark = pytest.mark.gpu


def _call_workspace(L, tiles, lut, K, C, stream):
    n = tiles.shape[0]
    vals = torch.empty_like(tiles)
    states = torch.empty((n, 256), dtype=torch.int16, device=tiles.device)
    ws_bytes = L.kq_viterbi_workspace_bytes(K, n)
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device=tiles.device)
    rc = L.kq_quantize_tiles_sqg(tiles.data_ptr(), vals.data_ptr(), states.data_ptr(), n, lut.data_ptr(), K, C,
                                 ws.data_ptr(), ws_bytes, stream)
    assert rc == 0, L.kq_last_error()
    return vals, states


def _call_noalloc(L, tiles, lut, K, C, stream):
    n = tiles.shape[0]
    vals = torch.full_like(tiles, float("nan"))
    states = torch.full((n, 256), -1, dtype=torch.int16, device=tiles.device)
    rc = L.kq_quantize_tiles_sqg_noalloc(tiles.data_ptr(), vals.data_ptr(), states.data_ptr(), n, lut.data_ptr(),
                                         K, C, stream)
    assert rc == 0, L.kq_last_error()
    return vals, states


def test_noalloc_matches_workspace_entry_point_twice(native, cuda_device):
    L = native.load()
    stream = ctypes.c_void_p(torch.cuda.current_stream(cuda_device).cuda_stream)
    g = torch.Generator(device=cuda_device).manual_seed(2024)
    # two calls in a row (other K, odd count, other context), then: one tile and one pair (a single job per
    # CTA, half a pair), K2, and the per-call bound of 4096 tiles
    cases = [(3, 600, 128), (4, 37, 64), (3, 1, 128), (4, 2, 16), (2, 300, 128), (3, 4096, 128)]
    for K, n, C in cases:
        tiles = torch.randn((n, 256), generator=g, device=cuda_device)
        tiles[: n // 3] = torch.round(tiles[: n // 3] * 2) / 2      # tie-heavy tiles
        lut = cb.sqg_xor_cheb_t12_bytes(K).to(cuda_device)
        v_ref, s_ref = _call_workspace(L, tiles, lut, K, C, stream)
        v_na, s_na = _call_noalloc(L, tiles, lut, K, C, stream)
        torch.cuda.synchronize(cuda_device)
        assert torch.equal(s_na, s_ref), f"K{K}: states differ"
        assert torch.equal(v_na, v_ref), f"K{K}: values differ"


def test_noalloc_rejects_oversized_calls(native, cuda_device):
    L = native.load()
    big = 4097
    rc = L.kq_quantize_tiles_sqg_noalloc(None, None, None, big, None, 3, 128, None)
    assert rc != 0
    assert b"4096" in L.kq_last_error()
