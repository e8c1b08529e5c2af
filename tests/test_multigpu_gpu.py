"""quantize_tiles_multigpu over two or more devices (kquant/exl3_encoder_backend.py:131-228).

The tile batch is split across quant_args["devices"] (by device_ratios when given), each slice encoded on
its own device and gathered on the first; codes and values must equal a single-device encode.  Skipped on
hosts with one GPU.
"""
import pytest
import torch

from kquant_b200 import exl3_encoder_backend as be

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("ratios", [None, [3, 1]])
def test_quantize_tiles_multigpu_equals_single_device(cuda_device, ratios):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    g = torch.Generator(device=cuda_device).manual_seed(8)
    tiles = torch.randn((700, 256), generator=g, device=cuda_device)
    args = {"K": 3, "mcg": True, "devices": ["cuda:0"], "tailbite_context": 128}
    q1, i1 = be.quantize_tiles(tiles, args)
    multi = dict(args, devices=["cuda:0", "cuda:1"], device_ratios=ratios)
    q2, i2 = be.quantize_tiles_multigpu_sync(tiles, multi)
    torch.cuda.synchronize()
    assert q2.device == tiles.device and i2.device == tiles.device
    assert torch.equal(i1, i2)
    assert torch.equal(q1, q2)
