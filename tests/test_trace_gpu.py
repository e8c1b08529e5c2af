"""tcgen05 fused GEMM + trace kernel (kq_trace_abt) against fp64 torch."""
import pytest
import torch

pytestmark = pytest.mark.gpu


def _ref(A, B, D):
    return float(((A.double() @ B.double().T) * D.double()).sum())


@pytest.mark.parametrize("M,N,Kd", [(128, 256, 32), (256, 512, 96), (384, 768, 512)])
def test_trace_random_matches_fp64(native, cuda_device, M, N, Kd):
    g = torch.Generator(device=cuda_device).manual_seed(M + N + Kd)
    A = torch.randn((M, Kd), generator=g, device=cuda_device)
    B = torch.randn((N, Kd), generator=g, device=cuda_device)
    D = torch.randn((M, N), generator=g, device=cuda_device)
    got = float(native.trace_abt(A, B, D))
    native.check_trace_errors()
    scale = float(((A.double() @ B.double().T).abs() * D.double().abs()).sum())
    assert abs(got - _ref(A, B, D)) <= 2e-3 * scale          # TF32 operands, fp32 accumulation


def test_trace_is_the_proxy_numerator(native, cuda_device):
    g = torch.Generator(device=cuda_device).manual_seed(7)
    k, n = 512, 384
    X = torch.randn((4 * k, k), generator=g, device=cuda_device)
    H = X.T @ X / X.shape[0]
    H = 0.5 * (H + H.T)
    E = torch.randn((k, n), generator=g, device=cuda_device) * 0.01
    Et = E.T.contiguous()
    got = float(native.trace_abt(Et, H, Et))
    ref = float(torch.trace(E.double().T @ H.double() @ E.double()))
    assert abs(got - ref) / ref < 1e-3
