"""The reconstruction kernel (kq_reconstruct_rotated) against the matmul form of the reference.

out = had_r(had_l(What) * su) * sv with 128-block Sylvester Hadamards normalised 1/sqrt(128)
(kquant/exl3_encoder_backend.py:268-285, 2211-2216).  The kernel uses fast Walsh-Hadamard
transforms, so it agrees with the FP64 matmul form to fp32 rounding; the bound here is 2e-6 of the
output's scale (the encoder's reconstruction contract is 1e-3 max-abs).
"""
import pytest
import torch

from kquant_b200 import _native

pytestmark = pytest.mark.gpu


def _had(n, dev):
    h = torch.ones((1, 1), dtype=torch.float64)
    while h.shape[0] < n:
        h = torch.cat((torch.cat((h, h), 1), torch.cat((h, -h), 1)), 0)
    return (h / n ** 0.5).to(dev)


@pytest.mark.parametrize("k,n", [(128, 128), (256, 384), (2048, 7168), (7168, 2048)])
def test_reconstruct_matches_matmul_form(cuda_device, k, n):
    g = torch.Generator(device=cuda_device).manual_seed(k + n)
    wq = torch.randn((k, n), generator=g, device=cuda_device)
    su = torch.randn(k, generator=g, device=cuda_device).sign() * (1 + torch.rand(k, generator=g, device=cuda_device))
    sv = torch.randn(n, generator=g, device=cuda_device).sign() * torch.rand(n, generator=g, device=cuda_device)
    out = _native.reconstruct_rotated(wq, su, sv)
    H = _had(128, cuda_device)
    w = (H @ wq.double().view(k // 128, 128, n)).view(k, n) * su.double().unsqueeze(1)
    w = (w.view(k, n // 128, 128) @ H).view(k, n) * sv.double().unsqueeze(0)
    torch.cuda.synchronize()
    err = (out.double() - w).abs().max().item()
    assert err <= 2e-6 * w.abs().max().item()


def test_reconstruct_rejects_untiled_shapes(cuda_device):
    wq = torch.zeros((100, 128), device=cuda_device)
    with pytest.raises(_native.KQError, match="multiples of 128"):
        _native.reconstruct_rotated(wq, torch.ones(100, device=cuda_device), torch.ones(128, device=cuda_device))
