"""GPU parity of the trellis pack / unpack kernels against the oracle and the golden prefixes."""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

PACK_PREFIX = {
    2: [6939] * 6,
    3: [30469, 1337, 1337, 14711, 14711, 30469],
    4: [17767, 291, -12817, -30293, 17767, 291],
}


@pytest.mark.parametrize("K", [2, 3, 4])
def test_pack_golden_prefix(native, cuda_device, K):
    states = (torch.arange(256, dtype=torch.int16) % (1 << K))[None].to(cuda_device)
    packed = native.pack_trellis(states, K)
    assert packed[0, :6].tolist() == PACK_PREFIX[K]


@pytest.mark.parametrize("K", [1, 2, 3, 4, 5, 6, 7, 8])
def test_pack_matches_oracle(native, oracle_mod, cuda_device, K):
    rng = np.random.default_rng(300 + K)
    states = rng.integers(-32768, 32768, (3, 5, 256)).astype(np.int16)
    got = native.pack_trellis(torch.from_numpy(states).to(cuda_device), K).cpu().numpy()
    assert np.array_equal(got, oracle_mod.pack_trellis(states, K))


@pytest.mark.parametrize("K", [1, 2, 3, 4, 5, 8])
def test_unpack_states_roundtrip(native, oracle_mod, cuda_device, K):
    rng = np.random.default_rng(400 + K)
    edges = rng.integers(0, 1 << K, (9, 256)).astype(np.int16)
    states = oracle_mod.reconstruct_states(edges, K)
    packed = native.pack_trellis(torch.from_numpy(states).to(cuda_device), K)
    back = native.unpack_trellis_states(packed, K).cpu().numpy()
    assert np.array_equal(back, states)


def test_pack_empty_and_large(native, cuda_device):
    empty = torch.empty((0, 256), dtype=torch.int16, device=cuda_device)
    assert native.pack_trellis(empty, 3).shape == (0, 48)
    big = torch.randint(-32768, 32767, (448, 128, 256), dtype=torch.int16, device=cuda_device)
    packed = native.pack_trellis(big, 3)
    edges = native.unpack_trellis_states(packed, 3) & 7
    assert torch.equal(edges, big & 7)


@pytest.mark.parametrize("rows,cols,perm", [(2048, 7168, False), (7168, 2048, True), (100, 136, True), (64, 8, False)])
def test_bf16_transposed_load(native, cuda_device, rows, cols, perm):
    g = torch.Generator(device=cuda_device).manual_seed(rows + cols)
    src = torch.randn((rows, cols), generator=g, device=cuda_device).to(torch.bfloat16)
    p = torch.randperm(rows, generator=g, device=cuda_device) if perm else None
    got = native.bf16_to_f32_transposed(src, p)
    ref = (src.index_select(0, p) if perm else src).float().T.contiguous()
    assert torch.equal(got, ref)
