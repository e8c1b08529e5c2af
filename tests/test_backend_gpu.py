"""GPU tests of the plugin-API backend: closure, decode consistency, argument contracts."""
import math

import pytest
import torch

from kquant_b200 import _native, codebooks as cb
from kquant_b200 import exl3_encoder_backend as be
from kquant_b200.ldlq import make_shared_h

pytestmark = pytest.mark.gpu


def _problem(dev, k=256, n=512, seed=0):
    g = torch.Generator(device=dev).manual_seed(seed)
    w = torch.randn((k, n), generator=g, device=dev) * 0.02
    x = torch.randn((4 * k, k), generator=g, device=dev) * torch.exp(torch.randn(k, generator=g, device=dev))
    h = x.T @ x / x.shape[0]
    return w, h


def _args(dev, **kw):
    a = {"K": 3, "seed": 7, "sv_seed": 11, "sigma_reg": 0.025, "devices": [str(dev)], "apply_out_scales": False,
         "tailbite_context": 128, "sqg_e4m3_luts_by_bits": {b: cb.sqg_xor_cheb_t12_bytes(b) for b in (2, 3, 4)}}
    a.update(kw)
    return a


def _decode(states, suh, svh, tile_bits, axis):
    """Decode [k/16, n/16, 256] states with the reference decoder's maths (kquant/exl3_reference.py:146-281)."""
    dev = states.device
    vals = torch.empty(states.shape, dtype=torch.float32, device=dev)
    for bits in sorted(set(tile_bits)):
        lab = cb.sqg_codebook(bits, cb.SQG_XOR_CHEB_T12, device=dev).float()
        v = lab[(states.long() & 0xFFFF)]
        sel = torch.tensor([b == bits for b in tile_bits], device=dev)
        if axis == "k":
            vals[sel] = v[sel]
        else:
            vals[:, sel] = v[:, sel]
    inv = be.tensor_core_perm_i(dev)
    vals = vals[..., inv]
    tk, tn, _ = vals.shape
    w = vals.reshape(tk, tn, 16, 16).permute(0, 2, 1, 3).reshape(tk * 16, tn * 16)
    w = be.preapply_had_l(w, 128) * suh.float().unsqueeze(1)
    return be.preapply_had_r(w, 128) * svh.float().unsqueeze(0)


@pytest.mark.parametrize("axis", ["n", "k"])
def test_qsrt_batch_decodes_to_its_reconstruction(cuda_device, axis):
    dev = cuda_device
    w, h = _problem(dev)
    k, n = w.shape
    ntiles = (n if axis == "n" else k) // 16
    bits = tuple([3] * ntiles)
    alt = tuple((2, 3, 4)[i % 3] for i in range(ntiles))
    groups = [[_args(dev, mixed_rate_axis=axis, mixed_tile_bits=bits), _args(dev, mixed_rate_axis=axis,
                                                                            mixed_tile_bits=alt)]]
    res = be.quantize_qsrt_batch([w.clone()], [make_shared_h(k, dev, h)], groups)
    assert len(res) == 1 and len(res[0]) == 2
    for cand, tb in zip(res[0], (bits, alt)):
        assert math.isfinite(cand["proxy"]) and 0 < cand["proxy"] < 0.5
        dec = _decode(cand["encoded"], cand["suh"], cand["svh"], tb, axis)
        assert torch.allclose(dec, cand["weight_q"], atol=1e-5, rtol=0)
        # every tile is a closed cyclic trellis path at its rate
        for bw in set(tb):
            sel = torch.tensor([b == bw for b in tb], device=dev)
            st = cand["encoded"][sel] if axis == "k" else cand["encoded"][:, sel]
            back = _native.unpack_trellis_states(_native.pack_trellis(st.contiguous(), bw), bw)
            assert torch.equal(back, st)
    # the all-K3 candidate of the reuse path equals a plain single-candidate encode
    w2, h2 = _problem(dev)
    single = be.quantize_qsrt_batch([w2], [make_shared_h(k, dev, h2)], [[_args(dev, mixed_rate_axis=axis,
                                                                              mixed_tile_bits=bits)]])
    assert torch.equal(single[0][0]["encoded"], res[0][0]["encoded"])


def test_quantize_qsrt_packs_closed_trellis(cuda_device):
    dev = cuda_device
    w, h = _problem(dev, k=256, n=256, seed=3)
    args = _args(dev)
    args["sqg_e4m3_lut"] = cb.sqg_xor_cheb_t12_bytes(4)
    del args["sqg_e4m3_luts_by_bits"]
    args["K"] = 4
    wq, proxy, out = be.quantize_qsrt(w.clone(), make_shared_h(256, dev, h), args, True)
    assert out["trellis"].shape == (16, 16, 64)
    assert out["suh"].dtype == torch.half and out["svh"].shape == (256,)
    assert 0 < proxy < 0.1
    assert args["q_fallback"] is False and "g_scale" in args
    rel = (wq - w).square().sum() / w.square().sum()
    assert rel < 0.05


def test_uniform_batch_shared_and_distinct_h(cuda_device):
    dev = cuda_device
    w1, h = _problem(dev, k=256, n=256, seed=5)
    w2, _ = _problem(dev, k=256, n=256, seed=6)
    shared = make_shared_h(256, dev, h)
    a1, a2 = _args(dev, seed=1, sv_seed=2), _args(dev, seed=1, sv_seed=3)
    r = be.quantize_uniform_batch([w1.clone(), w2.clone()], [shared, shared], [a1, a2])
    assert len(r) == 2 and all(0 < p < 0.2 for p, _ in r)
    assert all(o["trellis"].shape == (16, 16, 48) for _, o in r)
    hb = [make_shared_h(256, dev, h), make_shared_h(256, dev, h)]
    r2 = be.quantize_uniform_batch([w1.clone(), w2.clone()], hb, [_args(dev, seed=1, sv_seed=2),
                                                                  _args(dev, seed=1, sv_seed=3)])
    assert all(0 < p < 0.2 for p, _ in r2)


def test_quantize_tiles_dispatch_and_errors(cuda_device):
    dev = cuda_device
    tiles = torch.randn((5, 256), device=dev)
    q, i = be.quantize_tiles(tiles, {"K": 2, "devices": [str(dev)], "sqg_e4m3_luts_by_bits": {2: None, 3: None, 4: None}})
    q2, i2 = be.quantize_tiles(tiles, {"K": 2, "devices": [str(dev)], "mcg": True})
    assert torch.equal(i, i2) and torch.equal(q, q2)
    with pytest.raises(ValueError, match="missing rate-specific SQG K3 LUT"):
        be.quantize_tiles(tiles, {"K": 3, "devices": [str(dev)], "sqg_e4m3_luts_by_bits": {2: None}})
    with pytest.raises(ValueError, match="R44 mode"):
        be.quantize_tiles(tiles, {"K": 3, "devices": [str(dev)], "sqg_e4m3_mode": "other"})
    with pytest.raises(ValueError):
        be.quantize_tiles(tiles[:, :255].contiguous(), {"K": 3, "devices": [str(dev)], "mcg": True})


def test_uniform_batches_overlap_equals_sequential(cuda_device):
    """quantize_uniform_batches (overlapped traversals on prioritised streams) == sequential calls."""
    dev = cuda_device
    w1, h13 = _problem(dev, k=512, n=256, seed=21)
    w3, _ = _problem(dev, k=512, n=256, seed=22)
    w2, h2 = _problem(dev, k=256, n=512, seed=23)

    def groups():
        s13 = make_shared_h(512, dev, h13)
        return [([w1.clone(), w3.clone()], [s13, s13], [_args(dev, seed=1, sv_seed=2), _args(dev, seed=1, sv_seed=3)]),
                ([w2.clone()], [make_shared_h(256, dev, h2)], [_args(dev, seed=4, sv_seed=5)])]

    seq = [be.quantize_uniform_batch(w, h, q) for w, h, q in groups()]
    conc = be.quantize_uniform_batches(groups())
    assert len(conc) == 2
    for rs, rc in zip(seq, conc):
        for (ps, os_), (pc, oc) in zip(rs, rc):
            assert ps == pc
            for key in ("trellis", "suh", "svh"):
                assert torch.equal(os_[key], oc[key]), key


@pytest.mark.parametrize("B,k,n", [(1, 256, 512), (2, 128, 256)])
def test_fused_ldlq_step_equals_unfused(cuda_device, B, k, n):
    """The fused step kernel (kq_ldlq_step_encode) gives the same What/codes as gather + quantize_tiles + scatter."""
    dev = cuda_device
    g = torch.Generator(device=dev).manual_seed(B * 1000 + k)
    W = torch.randn((B, k, n), generator=g, device=dev) * 0.02
    x = torch.randn((B, 4 * k, k), generator=g, device=dev)
    H = x.transpose(1, 2) @ x / x.shape[1] + 0.01 * torch.eye(k, device=dev)
    Ls = torch.stack([torch.linalg.cholesky(h).T.contiguous() for h in H])
    Ls = Ls / torch.diagonal(Ls, dim1=1, dim2=2).unsqueeze(2)      # unit upper-triangular factor, L^T layout
    Ls = Ls.transpose(1, 2).contiguous()
    qa = _args(dev)
    plan = be._RatePlan(3, None, B, n // 16, dev)
    fused = be._ldlq_traverse(W, Ls, qa, plan, buffer_rows=128, tf32=False)
    plain = be._ldlq_traverse(W, Ls, qa, plan, buffer_rows=128, tf32=False,
                              source_indices=torch.arange(B, device=dev))
    assert torch.equal(fused[0], plain[0])
    assert torch.equal(fused[1], plain[1])
    assert torch.equal(fused[2], plain[2])


def test_chain_engine_long_buffers_and_stacked_members(cuda_device):
    """Chain engine with 256-row LDLQ buffers (feedback staged in two chunks) and distinct-H members:
    closed trellises, sane proxies, and uniform_batches == sequential uniform_batch."""
    dev = cuda_device
    w1, h1 = _problem(dev, k=512, n=256, seed=31)
    w2, h2 = _problem(dev, k=512, n=256, seed=32)
    w3, h3 = _problem(dev, k=256, n=384, seed=33)

    def groups():
        return [([w1.clone(), w2.clone()], [make_shared_h(512, dev, h1), make_shared_h(512, dev, h2)],
                 [_args(dev, seed=1, sv_seed=2, buf_size_k=256), _args(dev, seed=1, sv_seed=3, buf_size_k=256)]),
                ([w3.clone()], [make_shared_h(256, dev, h3)], [_args(dev, seed=4, sv_seed=5, K=4)])]

    seq = [be.quantize_uniform_batch(w, h, q) for w, h, q in groups()]
    conc = be.quantize_uniform_batches(groups())
    for rs, rc in zip(seq, conc):
        for (ps, os_), (pc, oc) in zip(rs, rc):
            assert 0 < ps < 0.2 and ps == pc
            assert torch.equal(os_["trellis"], oc["trellis"])
    for res, K in ((seq[0], 3), (seq[1], 4)):
        for _, out in res:
            st = _native.unpack_trellis_states(out["trellis"], K).view(-1, 256).long() & 0xFFFF
            prev = torch.roll(st, 1, dims=1)
            assert torch.equal(((prev << K) | (st & ((1 << K) - 1))) & 0xFFFF, st)


def test_chain_step_against_oracle(cuda_device):
    """One kq_ldlq_chain_step launch (in-kernel feedback) against the oracle, bit for bit (smoke's check)."""
    import numpy as np

    import __graft_entry__
    __graft_entry__._smoke_chain_step(cuda_device, np.random.default_rng(5))


@pytest.mark.parametrize("B,k,n", [(1, 1024, 512), (2, 512, 384)])
def test_chain_engine_equals_cublas_feedback_path(cuda_device, B, k, n):
    """Chain engine (feedback product summed in the kernel) == the fused-step path whose feedback is the
    reference's cuBLAS baddbmm (kquant/exl3_encoder_backend.py:389-505), codes and What bit for bit."""
    dev = cuda_device
    W = torch.stack([_problem(dev, k=k, n=n, seed=40 + b)[0] for b in range(B)]) * 25
    Ls = []
    for b in range(B):
        _, h = _problem(dev, k=k, n=n, seed=50 + b)
        L, _ = be.block_ldl(h.clone(), 16, {"devices": [str(dev)], "sigma_reg": 0.025}, False)
        Ls.append(L)
    Ls = torch.stack(Ls).contiguous()
    qa = _args(dev)
    wq_c = torch.empty_like(W)
    enc_c = torch.empty((B, k // 16, n // 16, 256), dtype=torch.int16, device=dev)
    members = [be._ChainMember(W[b], Ls[b], wq_c[b], enc_c[b], qa) for b in range(B)]
    be._chain_traverse(members, dev)
    plan = be._RatePlan(3, None, B, n // 16, dev)
    wq_s, enc_s, _ = be._ldlq_traverse(W, Ls, qa, plan, buffer_rows=128, tf32=False)
    torch.cuda.synchronize()
    assert torch.equal(enc_c, enc_s)
    assert torch.equal(wq_c, wq_s)


def _mixed_case(dev, axis, seed):
    k, n = 512, 256
    ws, ls = [], []
    for b in range(2):
        w, h = _problem(dev, k=k, n=n, seed=seed + b)
        L, _ = be.block_ldl(h.clone(), 16, {"devices": [str(dev)], "sigma_reg": 0.025}, False)
        ws.append(w * 25)
        ls.append(L)
    return torch.stack(ws).contiguous(), torch.stack(ls).contiguous(), (n if axis == "n" else k) // 16


def _old_path(W, Ls, qal):
    """The unfused traversal (cuBLAS feedback, per-K tile launches): source_indices bypasses the chain engine."""
    idx = torch.arange(W.shape[0], dtype=torch.long, device=W.device)
    return be.ldlq_mixed_batched(W, Ls, qal, source_indices=idx)


@pytest.mark.parametrize("axis", ["n", "k"])
def test_mixed_chain_engine_equals_unfused_path(cuda_device, axis):
    """Mixed-rate LDLQ on the chain engine (K2/K3/K4 chains sharing launches) == the unfused path."""
    dev = cuda_device
    W, Ls, nt = _mixed_case(dev, axis, 60)
    maps = [tuple((2, 3, 4)[(i // 8 + b) % 3] for i in range(nt)) for b in range(2)]
    qal = [_args(dev, mixed_rate_axis=axis, mixed_tile_bits=m) for m in maps]
    wq_c, enc_c = be.ldlq_mixed_batched(W, Ls, qal)
    wq_o, enc_o = _old_path(W, Ls, qal)
    assert torch.equal(enc_c, enc_o)
    assert torch.equal(wq_c, wq_o)


@pytest.mark.parametrize("axis", ["n", "k"])
def test_candidate_reuse_equals_independent_encodes(cuda_device, axis):
    """n-axis reuse (base + replacement columns in one engine run) and k-axis prefix trie (forking chains) ==
    every candidate encoded on its own by the unfused path."""
    dev = cuda_device
    W, Ls, nt = _mixed_case(dev, axis, 70)
    base = tuple([3] * nt)
    if axis == "n":
        cands = [base, tuple([2] * 8 + [4] * 8 + [3] * (nt - 16)), tuple([2] * 8 + [3] * (nt - 8))]
        reuse = be.ldlq_mixed_n_candidates_reuse
    else:
        # maps agree on the bottom buffers and diverge in the top two, in different buffers per candidate
        cands = [base, tuple([2] * 8 + [4] * 8 + [3] * (nt - 16)), tuple([4] * 8 + [2] * 8 + [3] * (nt - 16)),
                 tuple([3] * 8 + [2] * 4 + [4] * 4 + [3] * (nt - 16))]
        reuse = be.ldlq_mixed_k_candidates_prefix_reuse
    groups = [[_args(dev, mixed_rate_axis=axis, mixed_tile_bits=m) for m in cands] for _ in range(2)]
    wq_r, enc_r = reuse(W, Ls, groups)
    f = 0
    for s in range(2):
        for c in range(len(cands)):
            wq_o, enc_o = _old_path(W[s:s + 1].contiguous(), Ls[s:s + 1].contiguous(), [groups[s][c]])
            assert torch.equal(enc_r[f], enc_o[0]), (s, c)
            assert torch.equal(wq_r[f], wq_o[0]), (s, c)
            f += 1


@pytest.mark.parametrize("axis", ["n", "k"])
def test_qsrt_batch_candidates_equal_single_encodes(cuda_device, axis):
    """kquant's production call (quantize_qsrt_batch, reuse engines) == quantize_qsrt per candidate, which the
    reference fixtures pin: scales and codes bit for bit, proxies to float rounding."""
    dev = cuda_device
    k, n = (256, 512) if axis == "n" else (512, 256)
    w, h = _problem(dev, k=k, n=n, seed=90)
    nt = (n if axis == "n" else k) // 16
    maps = [tuple([3] * nt), tuple([2] * 8 + [4] * 8 + [3] * (nt - 16)),
            tuple([2] * 8 + [4] * 8 + [2] * 8 + [4] * 8 + [3] * (nt - 32))]
    group = [_args(dev, mixed_rate_axis=axis, mixed_tile_bits=m) for m in maps]
    batch = be.quantize_qsrt_batch([w.clone()], [make_shared_h(k, dev, h)], [group])[0]
    for m, cand in zip(maps, batch):
        # pack_trellis_fn (kquant/exl3_encoder_backend.py quantize_qsrt) returning the raw states
        _, proxy, out = be.quantize_qsrt(w.clone(), make_shared_h(k, dev, h),
                                         _args(dev, mixed_rate_axis=axis, mixed_tile_bits=m,
                                               pack_trellis_fn=lambda enc, qa: enc.clone()), False)
        assert torch.equal(out["suh"], cand["suh"]) and torch.equal(out["svh"], cand["svh"])
        assert torch.equal(out["trellis"], cand["encoded"])
        assert abs(proxy - cand["proxy"]) <= 1e-6 * max(proxy, 1e-12)


def test_mixed_chain_engine_odd_runs(cuda_device):
    """n-axis maps with single-column K runs (odd-length chains in mixed-K launches) == the unfused path."""
    dev = cuda_device
    W, Ls, nt = _mixed_case(dev, "n", 80)
    maps = [tuple((2, 3, 4, 3, 2, 4, 4, 4)[i % 8] for i in range(nt)),
            tuple((3, 2, 2, 4, 3, 3, 4, 2)[i % 8] for i in range(nt))]
    qal = [_args(dev, mixed_rate_axis="n", mixed_tile_bits=m) for m in maps]
    wq_c, enc_c = be.ldlq_mixed_batched(W, Ls, qal)
    wq_o, enc_o = _old_path(W, Ls, qal)
    assert torch.equal(enc_c, enc_o)
    assert torch.equal(wq_c, wq_o)


@pytest.mark.parametrize("rates", [(3, 3, 3, 3, 3), (2, 3, 4, 3, 2), (2, 3, 4, 3, 2, 4, 3, 2, 3, 4)])
def test_double_wave_chain_launches_equal_single_wave(cuda_device, monkeypatch, rates):
    """Launches of two tile pairs per CTA (uniform K: the grid-stride kernel; mixed K: the per-CTA pair table)
    give the same codes and What, bit for bit, as one-wave launches of the same chains."""
    dev = cuda_device
    k, n = 512, 2048

    def run():
        members, outs = [], []
        for b, K in enumerate(rates):
            w, h = _problem(dev, k=k, n=n, seed=80 + b)
            L, _ = be.block_ldl(h.clone(), 16, {"devices": [str(dev)], "sigma_reg": 0.025}, False)
            wq = torch.empty_like(w)
            enc = torch.empty((k // 16, n // 16, 256), dtype=torch.int16, device=dev)
            members.append(be._ChainMember((w * 25).contiguous(), L, wq, enc, _args(dev, K=K)))
            outs.append((wq, enc))
        be._chain_traverse(members, dev)
        torch.cuda.synchronize()
        return outs

    sizes = []
    real_step = _native.ldlq_chain_step

    def spy(items, ctx, device, max_ctas=0):
        sizes.append(sum(int(i.n_tiles) for i in items))
        return real_step(items, ctx, device, max_ctas)

    monkeypatch.setattr(_native, "ldlq_chain_step", spy)
    double = run()
    sms = torch.cuda.get_device_properties(dev).multi_processor_count
    assert max(sizes) > 2 * sms
    real_select = be._select_launch
    monkeypatch.setattr(be, "_select_launch", lambda cands, cap, s: real_select(cands, min(cap, 2 * s), s))
    single = run()
    for (wq_d, enc_d), (wq_s, enc_s) in zip(double, single):
        assert torch.equal(enc_d, enc_s)
        assert torch.equal(wq_d, wq_s)
