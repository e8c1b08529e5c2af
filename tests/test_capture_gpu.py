"""Hessian accumulation on the tensor cores against fp64 (kquant/capture.py:713-730 contract)."""
import pytest
import torch

from kquant_b200.capture import accumulate_hessian

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("tokens,dim,chunk", [(1000, 512, 300), (4096, 256, 4096), (64, 384, 64), (77, 100, 50),
                                              (3000, 1000, 3000), (5, 7, 2)])
def test_hessian_matches_fp64(cuda_device, tokens, dim, chunk):
    g = torch.Generator().manual_seed(tokens + dim)
    x = torch.randn((tokens, dim), generator=g) * torch.exp(torch.randn(dim, generator=g))
    w = torch.rand(tokens, generator=g) + 0.1
    ref = (x.double().T @ (x.double() * w.double().unsqueeze(1)))
    # The FP32 CUDA-core product (TF32 off) sets the accuracy 3xTF32 must match.
    torch.backends.cuda.matmul.allow_tf32 = False
    xd, wd = x.to(cuda_device), w.to(cuda_device)
    fp32 = (xd.T @ (xd * wd.unsqueeze(1))).double().cpu()
    fp32_err = float((fp32 - ref).abs().max() / ref.abs().max())
    for precision, tol in (("3xtf32", max(2e-6, 4 * fp32_err)), ("tf32", 2e-3)):
        acc, den = accumulate_hessian(x, w, device=cuda_device, chunk_rows=chunk, precision=precision)
        err = (acc.double().cpu() - ref).abs().max() / ref.abs().max()
        assert err < tol, (precision, float(err), fp32_err)
        assert den == pytest.approx(float(w.double().sum()), rel=1e-12)
        assert torch.equal(acc, acc.T)


def test_gemm_abt_beta_and_alpha(native, cuda_device):
    g = torch.Generator(device=cuda_device).manual_seed(1)
    A = torch.randn((256, 64), generator=g, device=cuda_device)
    B = torch.randn((512, 64), generator=g, device=cuda_device)
    C = torch.randn((256, 512), generator=g, device=cuda_device)
    ref = 0.5 * (A.double() @ B.double().T) + 2.0 * C.double()
    native.gemm_abt_tf32(A, B, C, alpha=0.5, beta=2.0)
    native.check_trace_errors()
    assert (C.double() - ref).abs().max() < 2e-3 * ref.abs().max()


def test_hessian_accumulates_into_out_and_empty(cuda_device):
    g = torch.Generator().manual_seed(3)
    x = torch.randn((300, 256), generator=g)
    w = torch.rand(300, generator=g)
    start = torch.eye(256, device=cuda_device)
    acc, den = accumulate_hessian(x, w, device=cuda_device, chunk_rows=128, out=start.clone())
    ref = x.double().T @ (x.double() * w.double().unsqueeze(1)) + torch.eye(256, dtype=torch.float64)
    assert (acc.double().cpu() - ref).abs().max() < 1e-5 * ref.abs().max()
    acc0, den0 = accumulate_hessian(x[:0], w[:0], device=cuda_device, chunk_rows=128)
    assert den0 == 0.0 and not acc0.any()
