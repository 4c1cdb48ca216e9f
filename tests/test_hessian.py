"""Hessian accumulation and factorization (src/liqk_v2.py:207-231, :1074-1088).

CovAccumulator is checked bit for bit against the reference's own sequence (Gram, conversion to fp64, add) on CPU (fp32
batches) and on the GPU (bf16 / fp16 batches on the tensor cores).  tri_inv_lower (leaf inverses + tensor-core merges)
is checked against the reference's triangular solve on Cholesky factors of damped Gram matrices like the pipeline's:
exact zeros above the diagonal, residual |L X - I| and the difference to the solve within fp32 tolerances."""
import pytest
import torch

from ltq_research_b200.hessian import CovAccumulator


def _reference_sequence(batches):
    """The reference's _CovAccumulator arithmetic (src/liqk_v2.py:219-231), restated."""
    H, n = None, 0
    for x in batches:
        x2 = x.reshape(-1, x.shape[-1])
        if x2.dtype in (torch.bfloat16, torch.float16):
            gram = torch.mm(x2.T, x2, out_dtype=torch.float32)
        else:
            x2 = x2.float()
            gram = x2.T @ x2
        if H is None:
            H = torch.zeros((x2.shape[1],) * 2, dtype=torch.float64, device=x2.device)
        H.add_(gram.to(torch.float64))
        n += x2.shape[0]
    return (H / max(n, 1)).to(torch.float32)


def test_cov_accumulator_fp32_batches_cpu():
    g = torch.Generator().manual_seed(1)
    batches = [torch.randn(3, 40, 64, generator=g) * torch.exp(torch.randn(64, generator=g)) for _ in range(4)]
    acc = CovAccumulator()
    for b in batches:
        acc.add(b)
    assert acc.n == 4 * 120
    assert torch.equal(acc.get(), _reference_sequence(batches))
    assert CovAccumulator().n == 0


@pytest.mark.gpu
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32])
def test_cov_accumulator_gpu(dtype, cuda_dev):
    g = torch.Generator(device=cuda_dev).manual_seed(2)
    batches = [(torch.randn(2, 512, 768, device=cuda_dev, generator=g) * 0.5).to(dtype) for _ in range(3)]
    acc = CovAccumulator()
    for b in batches:
        acc.add(b)
    assert torch.equal(acc.get(), _reference_sequence(batches))


def _cholesky_factor(K, seed, dev):
    """L = chol(flip(H_reg)) as the pipeline builds it: H = X^T X / N with per-channel scales, damped by 0.2 mean(diag)."""
    g = torch.Generator(device=dev).manual_seed(seed)
    X = torch.randn(max(2 * K, 1024), K, device=dev, generator=g) * torch.exp(torch.randn(1, K, device=dev, generator=g))
    H = X.T @ X / X.shape[0]
    H.diagonal().add_(0.2 * H.diagonal().mean())
    L, info = torch.linalg.cholesky_ex(H.flip(0, 1))
    assert int(info) == 0
    return L


@pytest.mark.gpu
@pytest.mark.parametrize("K", [256, 768, 1280, 3072])
def test_tri_inv_lower_accuracy(K, cuda_dev):
    """Against the exact (fp64) inverse: normwise residual |L X - I| / (|L| |X|) within 4 u (u = 2^-24; the merges are
    backward stable) and forward error below 1e-5 relative.  Multiplying by inverted blocks loses the extra forward
    accuracy of substitution (the reference's triangular solve reaches ~1e-7 here); the fast mode accepts that, the
    fp32 mode keeps the reference's solve."""
    from ltq_research_b200.hessian import tri_inv_lower
    L = _cholesky_factor(K, K, cuda_dev)
    X = tri_inv_lower(L)
    torch.cuda.synchronize()
    assert X.is_contiguous() and torch.equal(torch.tril(X), X)
    Ld, Xd = L.double(), X.double()
    I = torch.eye(K, device=cuda_dev, dtype=torch.float64)
    exact = torch.linalg.solve_triangular(Ld, I, upper=False)
    normwise = ((Ld @ Xd - I).norm() / (Ld.norm() * Xd.norm())).item()
    assert normwise <= 4 * 2.0 ** -24, normwise
    fwd = ((Xd - exact).norm() / exact.norm()).item()
    assert fwd < 1e-5, fwd


@pytest.mark.gpu
def test_tri_inv_lower_column_major_input(cuda_dev):
    """The factorization returns column-major factors; the inverse reads any layout."""
    from ltq_research_b200.hessian import tri_inv_lower
    L = _cholesky_factor(512, 5, cuda_dev)
    Lt = L.T.contiguous().T  # column-major copy
    assert Lt.stride() != L.contiguous().stride()
    assert torch.equal(tri_inv_lower(Lt), tri_inv_lower(L.contiguous()))
