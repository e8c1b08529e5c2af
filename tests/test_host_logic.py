"""Host-side logic of the backend, checked on the CPU (no device work)."""
import math
import sys

import pytest
import torch

from kquant_b200 import _native, codebooks as cb
from kquant_b200 import exl3_encoder_backend as be
from kquant_b200.exl3_loader import load_qsrt_encoder
from kquant_b200.ldlq import SIGMA_REG, make_shared_h
from kquant_b200.sqg_quantizer import install_sqg_quantizer


def test_tensor_core_order_is_the_exl_fragment_layout():
    perm = be.tensor_core_perm("cpu")
    assert sorted(perm.tolist()) == list(range(256))
    # thread t, slot s -> row 2*(t%4) + (s&1) + 8*((s>>1)&1), column t//4 + 8*(s>>2)
    assert perm[:8].tolist() == [0, 16, 128, 144, 8, 24, 136, 152]
    assert perm[8 * 5 + 3].item() == (2 * 1 + 1 + 8) * 16 + 1
    assert torch.equal(perm[be.tensor_core_perm_i("cpu")], torch.arange(256, dtype=perm.dtype))


def test_mixed_rate_spec_validates_like_the_reference():
    assert be.mixed_rate_spec(32, 64, {"mixed_rate_axis": "n", "mixed_tile_bits": [2, 3, 4, 3]}) == ("n", (2, 3, 4, 3))
    with pytest.raises(ValueError, match="mixed_rate_axis"):
        be.mixed_rate_spec(32, 32, {"mixed_rate_axis": "x", "mixed_tile_bits": [3, 3]})
    with pytest.raises(ValueError, match="expected 2"):
        be.mixed_rate_spec(32, 32, {"mixed_rate_axis": "k", "mixed_tile_bits": [3]})
    with pytest.raises(ValueError, match="only integer K2, K3, and K4"):
        be.mixed_rate_spec(32, 32, {"mixed_rate_axis": "k", "mixed_tile_bits": [3, True]})
    with pytest.raises(ValueError, match="required"):
        be.mixed_rate_spec(32, 32, {"mixed_rate_axis": "k"})
    with pytest.raises(ValueError, match="tile aligned"):
        be.mixed_rate_spec(24, 32, {"mixed_rate_axis": "k", "mixed_tile_bits": [3]})


def test_mixed_grouping_orders_by_width_and_inverts():
    order, inverse, slices = be._make_mixed_ldlq_grouping([3, 2, 4, 2, 3], "cpu")
    assert order.tolist() == [1, 3, 0, 4, 2]
    assert slices == ((2, 0, 2), (3, 2, 4), (4, 4, 5))
    assert torch.equal(order[inverse], torch.arange(5))
    assert be._make_mixed_ldlq_grouping([3, 3], "cpu") == (None, None, ((3, 0, 2),))


def test_rate_plan_groups_tiles_per_step():
    plan = be._RatePlan([(2, 3), (3, 3)], "n", 2, 2, "cpu")        # member-major flat tiles
    groups = plan.groups_for(0)
    assert [(b, w.tolist()) for b, w in groups] == [(2, [0]), (3, [1, 2, 3])]
    plan_k = be._RatePlan([(2, 4), (4, 4)], "k", 2, 3, "cpu")
    g0 = plan_k.groups_for(0)
    assert [(b, w.tolist()) for b, w in g0] == [(2, [0, 1, 2]), (4, [3, 4, 5])]
    assert plan_k.groups_for(1) == [(4, None)]
    assert be._RatePlan(3, None, 4, 8, "cpu").groups_for(7) == [(3, None)]


def test_tile_codebook_dispatch_and_errors():
    luts = {b: cb.sqg_xor_cheb_t12_bytes(b) for b in (2, 3, 4)}
    assert be._tile_codebook({"sqg_e4m3_luts_by_bits": luts}, 3) == (_native.KQ_CB_SQG, luts[3])
    assert be._tile_codebook({"sqg_e4m3_luts_by_bits": {2: None, 3: luts[3], 4: None}}, 2) == (_native.KQ_CB_MCG, None)
    assert be._tile_codebook({"mcg": False}, 3) == (_native.KQ_CB_MCG, None)       # key presence, as upstream
    assert be._tile_codebook({"mul1": True}, 3) == (_native.KQ_CB_MUL1, None)
    assert be._tile_codebook({}, 3) == (_native.KQ_CB_3INST, None)
    kind, lut = be._tile_codebook({"sqg_e4m3_mode": "normal"}, 4)
    assert kind == _native.KQ_CB_SQG and torch.equal(lut, cb.sqg_e4m3_bytes(4, "normal"))
    with pytest.raises(ValueError, match="cannot be combined"):
        be._tile_codebook({"sqg_e4m3_luts_by_bits": luts, "sqg_e4m3_lut": luts[3]}, 3)
    with pytest.raises(TypeError, match="mapping"):
        be._tile_codebook({"sqg_e4m3_luts_by_bits": [1, 2]}, 3)
    with pytest.raises(ValueError, match="K2, K3, or K4"):
        be._tile_codebook({"sqg_e4m3_luts_by_bits": {5: None}}, 3)


def test_multigpu_split_sizes():
    assert be._split_sizes(100, ["a", "b", "c"], None) == [33, 33, 34]
    assert be._split_sizes(160, ["a", "b"], [1, 3]) == [32, 128]   # round-half-even of 40/16, as upstream
    assert sum(be._split_sizes(17, ["a"] * 5, [1, 1, 1, 1, 100])) == 17


def test_scale_helpers():
    w = torch.ones(4, 4)
    su, sv = torch.ones(4, 1), torch.ones(1, 4)
    w2, su2, sv2 = be.apply_g_scale(w.clone(), su.clone(), sv.clone(), 2.0)
    assert torch.all(w2 == 2) and torch.all(su2 == 0.5) and torch.all(sv2 == 1)
    w3, su3, sv3 = be.apply_g_scale(w.clone(), su.clone(), sv.clone(), 2.0, into_sv=True)
    assert torch.all(su3 == 1) and torch.all(sv3 == 0.5)
    with pytest.raises(ValueError):
        be.apply_g_scale(w, su, sv, -1.0)
    with pytest.raises(ValueError):
        be.relocate_g_scale_to_sv(su, sv, math.inf)
    x = torch.randn(70, 33)
    assert torch.allclose(be.block_rms(x, 0, True), x.square().mean(0, keepdim=True).sqrt(), rtol=1e-5)
    assert torch.allclose(be.block_rms_n(x), x.square().mean().sqrt(), rtol=1e-5)
    assert be.block_nmse(x, x) == 0.0


def test_shared_h_and_loader_contract():
    h = make_shared_h(32, torch.device("cpu"), torch.eye(32) * 2)
    assert h["count"] == 1 and not h["finalized"] and torch.equal(h["H"], h["error_H"])
    assert h["H"].data_ptr() != h["error_H"].data_ptr()
    assert SIGMA_REG == 0.025
    with pytest.raises(ValueError):
        make_shared_h(16, torch.device("cpu"), torch.eye(32))
    mod = load_qsrt_encoder("/does/not/matter")
    assert mod is be and sys.modules["exllamav3.modules.quant.exl3_lib.kquant_qsrt_encoder"] is be
    install_sqg_quantizer(mod)
    assert mod._kquant_sqg_installed
    other = type(sys)("other_backend")
    other.quantize_tiles = lambda *a: None
    install_sqg_quantizer(other)
    assert other.quantize_tiles is be.quantize_tiles


def test_sample_scale_tiles_shape_and_order():
    w = torch.randn(64, 128)
    tiles = be.sample_scale_tiles(w)
    tk, tn = 4, 8
    diag = max(tk, tn) * 3
    extremes = 2 * min(max(8, diag // 16), (tk * tn + 1) // 2)
    assert tiles.shape == (diag + extremes, 256)
    first = w.view(tk, 16, tn, 16)[0, :, 0, :].reshape(256)[be.tensor_core_perm("cpu")]
    assert torch.equal(tiles[0], first)


def test_no_cpu_path():
    with pytest.raises(ValueError, match="CUDA"):
        be.quantize_tiles(torch.zeros(1, 256), {"K": 3, "devices": ["cpu"], "mcg": True})


@pytest.mark.parametrize("k,n", [(7168, 2048), (2048, 7168), (2048, 2048), (128, 256), (512, 1024)])
def test_tile_encode_count_matches_scale_search_sampling(k, n):
    """bench.tile_encodes (the CPU arm's scale-search charge) equals the encodes the backend performs."""
    import bench
    w = torch.randn((k, n))
    samples = be.sample_scale_tiles(w).shape[0]
    assert bench.tile_encodes(k, n) == (k // 16) * (n // 16) + 10 * len(range(0, samples, 3)) + 5 * samples


def test_layer_rate_allocation_is_3p2_bpw_and_seeded():
    import bench
    ks = bench.layer_rates()
    flat = [k for row in ks for k in row]
    assert len(ks) == bench.LAYER_EXPERTS + 1 and all(len(r) == 3 for r in ks)
    assert {k: flat.count(k) for k in (2, 3, 4)} == {2: 231, 3: 462, 4: 462}
    assert sum(flat) / len(flat) == pytest.approx(3.2)
    assert bench.layer_rates() == ks and bench.layer_rates(seed=1) != ks
