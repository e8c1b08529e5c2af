"""GPU parity of the wide-butterfly Viterbi kernel (K1, K5..K8) against the CPU oracle and the reference kernel.

The reference template covers any K (kquant/csrc/qsrt_quantize_tiles_kernel.cuh:14-21);
its host binding rejects K outside 2..4 (kquant/csrc/sqg_quantize.cu:190, 286), so
the reference side here is oracle/ref_harness.cu, the reference's own translation
unit launched at these K.
"""
import numpy as np
import pytest
import torch

from tests.test_viterbi_gpu import KINDS, _labels, _tiles

pytestmark = pytest.mark.gpu

WIDE = [1, 5, 6, 7, 8]


@pytest.fixture(scope="session")
def ref_harness():
    from oracle import build_ref
    if not build_ref.HARNESS.exists():
        pytest.skip("reference harness oracle/_ref/kquant_ref_harness.so not built")
    return build_ref.load_harness()


@pytest.mark.parametrize("K", WIDE)
@pytest.mark.parametrize("tiles_kind,C", [("normal", 128), ("coarse", 128), ("zeros", 7), ("wide", 1),
                                          ("coarse", 37)])
def test_wide_matches_oracle(native, oracle_mod, cuda_device, K, tiles_kind, C):
    O = oracle_mod
    lab_dev, lab_cpu = _labels(native, O, "mcg", K, cuda_device)
    tiles = _tiles(tiles_kind, 2, 300 + K)
    idx_ref, val_ref, rc = O.viterbi(K, lab_cpu, tiles, C)
    assert rc == 0
    vals, states = native.viterbi_encode(torch.from_numpy(tiles).to(cuda_device), K, lab_dev, C)
    torch.cuda.synchronize()
    assert np.array_equal(states.cpu().numpy().view(np.uint16), idx_ref)
    assert np.array_equal(vals.cpu().numpy(), val_ref)


@pytest.mark.parametrize("K", WIDE)
@pytest.mark.parametrize("kind", ["mul1", "3inst"])
def test_wide_other_codebooks_match_oracle(native, oracle_mod, cuda_device, K, kind):
    O = oracle_mod
    lab_dev, lab_cpu = _labels(native, O, kind, K, cuda_device)
    tiles = _tiles("normal", 2, 400 + K)
    idx_ref, val_ref, _ = O.viterbi(K, lab_cpu, tiles, 128)
    vals, states = native.viterbi_encode(torch.from_numpy(tiles).to(cuda_device), K, lab_dev, 128)
    assert np.array_equal(states.cpu().numpy().view(np.uint16), idx_ref)
    assert np.array_equal(vals.cpu().numpy(), val_ref)


@pytest.mark.parametrize("K", WIDE)
def test_wide_multiwave_subset_matches_oracle(native, oracle_mod, cuda_device, K):
    """More tiles than SMs: each CTA loops over tiles; spot-check first, wave-boundary and last tiles."""
    O = oracle_mod
    lab_dev, lab_cpu = _labels(native, O, "mcg", K, cuda_device)
    sms = torch.cuda.get_device_properties(cuda_device).multi_processor_count
    n = 2 * sms + 3
    tiles = _tiles("coarse", n, 50 + K)
    vals, states = native.viterbi_encode(torch.from_numpy(tiles).to(cuda_device), K, lab_dev, 128)
    pick = np.array([0, sms - 1, sms, 2 * sms, n - 1])
    idx_ref, val_ref, _ = O.viterbi(K, lab_cpu, tiles[pick], 128)
    assert np.array_equal(states.cpu().numpy().view(np.uint16)[pick], idx_ref)
    assert np.array_equal(vals.cpu().numpy()[pick], val_ref)


@pytest.mark.parametrize("K", WIDE + [2, 3, 4])
@pytest.mark.parametrize("codebook", [1, 2])
def test_wide_matches_reference_kernel(native, ref_harness, cuda_device, K, codebook):
    """Bit-exact against the reference kernel at scale (300 tiles, half tie-heavy, C = 128 and 16)."""
    n = 300
    g = torch.Generator(device=cuda_device).manual_seed(23 + K)
    tiles = torch.randn((n, 256), generator=g, device=cuda_device)
    tiles[: n // 2] = torch.round(tiles[: n // 2] * 2) / 2
    sms = torch.cuda.get_device_properties(cuda_device).multi_processor_count
    mb = min(n, sms)
    costs = torch.zeros((mb, 2, 65536 >> K), dtype=torch.float16, device=cuda_device)
    edges = torch.empty(mb * ref_harness.kqref_decision_bytes_per_tile(K), dtype=torch.uint8, device=cuda_device)
    lab = native.build_labels(codebook, None, cuda_device)
    for C in (128, 16):
        ref_out = torch.empty_like(tiles)
        ref_idx = torch.empty((n, 256), dtype=torch.int16, device=cuda_device)
        stream = torch.cuda.current_stream(cuda_device).cuda_stream
        rc = ref_harness.kqref_quantize_procedural(tiles.data_ptr(), ref_out.data_ptr(), ref_idx.data_ptr(),
                                                   costs.data_ptr(), edges.data_ptr(), n, mb, K, codebook, C,
                                                   stream)
        assert rc == 0
        vals, states = native.viterbi_encode(tiles, K, lab, C)
        torch.cuda.synchronize()
        assert torch.equal(states, ref_idx), f"K{K} cb{codebook} C{C}"
        assert torch.equal(vals, ref_out)


def test_wide_rate_ldlq_matches_unfused_reference_order(native, cuda_device):
    """K=5 through the public LDLQ entry: codes equal the reference's ldlq loop restated in torch
    (cuBLAS feedback, gather, tile encode, scatter) on the same inputs."""
    from kquant_b200 import exl3_encoder_backend as be
    g = torch.Generator(device=cuda_device).manual_seed(5)
    k, n = 256, 256
    W = torch.randn((k, n), generator=g, device=cuda_device) * 0.5
    L = torch.tril(torch.randn((k, k), generator=g, device=cuda_device) * 0.02, -1)
    args = {"K": 5, "mcg": True, "devices": [str(cuda_device)], "tailbite_context": 128}
    wq, enc = be.ldlq(W, L, args)
    # restated reference loop (kquant/exl3_encoder_backend.py:389-505)
    prod = torch.zeros_like(W)
    ref_wq = torch.zeros_like(W)
    ref_enc = torch.zeros((k // 16, n // 16, 256), dtype=torch.int16, device=cuda_device)
    perm, perm_i = be.tensor_core_perm(cuda_device), be.tensor_core_perm_i(cuda_device)
    torch.backends.cuda.matmul.allow_tf32 = False
    for j in range(k, 0, -128):
        i = j - 128
        bw, bq, bp, bl = W[i:j], ref_wq[i:j], prod[i:j], L[i:j]
        for bj in range(128, 0, -16):
            bi = bj - 16
            err = bw[bj:] - bq[bj:]
            comp = bp[bi:bj]
            comp.addmm_(bl[bj:, i + bi:i + bj].T, err)
            rows = bw[bi:bj] + comp
            tiles = rows.reshape(16, n // 16, 16).permute(1, 0, 2).reshape(n // 16, 256)[:, perm]
            q, idx = be.quantize_tiles(tiles, args)
            bq[bi:bj] = q[:, perm_i].reshape(n // 16, 16, 16).permute(1, 0, 2).reshape(16, n)
            ref_enc[(i + bi) // 16] = idx
        prod.addmm_(bl.T, bw - bq)
    torch.cuda.synchronize()
    assert torch.equal(enc, ref_enc)
    assert torch.equal(wq, ref_wq)


def test_wide_rate_members_on_streams_equal_single_runs(native, cuda_device):
    """Several K1/K5..K8 members of one engine run (stepped in turn on their own streams) give the same codes
    and What, bit for bit, as each member run alone."""
    from kquant_b200 import exl3_encoder_backend as be
    g = torch.Generator(device=cuda_device).manual_seed(6)
    shapes = [(256, 512, 5), (128, 1024, 6), (384, 256, 1)]

    def make():
        out = []
        for k, n, K in shapes:
            W = torch.randn((k, n), generator=g, device=cuda_device) * 0.5
            L = torch.tril(torch.randn((k, k), generator=g, device=cuda_device) * 0.02, -1)
            out.append((W, L, K))
        return out

    probs = make()

    def member(W, L, K):
        args = {"K": K, "mcg": True, "devices": [str(cuda_device)], "tailbite_context": 64}
        k, n = W.shape
        return be._ChainMember(W, L, torch.empty_like(W), torch.empty((k // 16, n // 16, 256), dtype=torch.int16,
                                                                      device=cuda_device), args)

    together = [member(*p) for p in probs]
    be._chain_traverse(together, cuda_device)
    alone = []
    for p in probs:
        m = member(*p)
        be._chain_traverse([m], cuda_device)
        alone.append(m)
    torch.cuda.synchronize()
    for a, b in zip(together, alone):
        assert torch.equal(a.enc, b.enc)
        assert torch.equal(a.wq, b.wq)
