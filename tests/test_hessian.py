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


def _damped_gram(K, seed, dev, damp=0.2):
    g = torch.Generator(device=dev).manual_seed(seed)
    X = torch.randn(max(2 * K, 1024), K, device=dev, generator=g) * torch.exp(torch.randn(1, K, device=dev, generator=g))
    H = X.T @ X / X.shape[0]
    H.diagonal().add_(damp * H.diagonal().mean())
    return H


@pytest.mark.gpu
@pytest.mark.parametrize("K", [256, 768, 1280, 3072])
def test_cholesky_lower_accuracy(K, cuda_dev):
    """Blocked factorization (leaf kernel + tensor-core panel and trailing products) against the fp64 factor of the
    same matrix: exact zeros above the diagonal; backward error |A - L L^T| / |A| and forward error of L within 4x
    those of torch.linalg.cholesky_ex's own fp32 factor (or 16 u / 1e-5 when the library's are smaller still); info 0;
    the inverse within tri_inv_lower's bounds; the input untouched unless overwrite is asked for."""
    from ltq_research_b200.hessian import cholesky_lower
    A = _damped_gram(K, K + 1, cuda_dev).flip(0, 1).contiguous()
    A0 = A.clone()
    L, info, X = cholesky_lower(A, inverse=True)
    torch.cuda.synchronize()
    assert int(info) == 0 and torch.equal(A, A0)
    assert L.is_contiguous() and torch.equal(torch.tril(L), L) and torch.equal(torch.tril(X), X)
    Ad, Ld = A.double(), L.double()
    exact = torch.linalg.cholesky(Ad)
    Lc = torch.linalg.cholesky_ex(A)[0].double()
    back = ((Ad - Ld @ Ld.T).norm() / Ad.norm()).item()
    back_lib = ((Ad - Lc @ Lc.T).norm() / Ad.norm()).item()
    fwd = ((Ld - exact).norm() / exact.norm()).item()
    fwd_lib = ((Lc - exact).norm() / exact.norm()).item()
    print(f"K={K}: backward {back:.3g} (library {back_lib:.3g}), forward {fwd:.3g} (library {fwd_lib:.3g})")
    assert back <= max(4 * back_lib, 16 * 2.0 ** -24), (back, back_lib)
    assert fwd <= max(4 * fwd_lib, 1e-5), (fwd, fwd_lib)
    I = torch.eye(K, device=cuda_dev, dtype=torch.float64)
    Xd = X.double()
    assert ((Ld @ Xd - I).norm() / (Ld.norm() * Xd.norm())).item() <= 4 * 2.0 ** -24
    inv = torch.linalg.solve_triangular(exact, I, upper=False)
    assert ((Xd - inv).norm() / inv.norm()).item() < 1e-5
    L2, info2, X2 = cholesky_lower(A0, overwrite=True)
    assert X2 is None and L2.data_ptr() == A0.data_ptr() and torch.equal(L2, L) and int(info2) == 0


@pytest.mark.gpu
@pytest.mark.parametrize("K", [256, 1024, 3072])
def test_cholesky_lower_solve_refit_system(K, cuda_dev):
    """The refit system of the fast mode: A = (U^T U) o H + 1e-3 mean(diag) I, factored with the leaves' diagonal-block
    inverses kept and solved by chol_solve (block substitution through those inverses, ltq_chol_solve), against fp64
    and against torch.cholesky_solve on the same factor; the kept blocks invert L's diagonal blocks."""
    from ltq_research_b200.hessian import chol_solve, cholesky_lower
    g = torch.Generator(device=cuda_dev).manual_seed(3)
    U = torch.randn(512, K, device=cuda_dev, generator=g)
    H = _damped_gram(K, 4, cuda_dev)
    A = (U.T @ U) * H
    A.diagonal().add_(1e-3 * A.diagonal().mean())
    b = torch.randn(K, device=cuda_dev, generator=g)
    L, info, D = cholesky_lower(A, diag_inv=True)
    assert int(info) == 0 and D.shape == (K // 256, 256, 256)
    for p in range(K // 256):
        Lp = L[256 * p:256 * (p + 1), 256 * p:256 * (p + 1)].double()
        res = (torch.tril(D[p]).double() @ Lp - torch.eye(256, device=cuda_dev, dtype=torch.float64)).abs().max()
        assert res.item() < 1e-4, (p, res.item())
    x = chol_solve(L, D, b)
    lib = torch.cholesky_solve(b.unsqueeze(1), L).squeeze(1)
    want = torch.linalg.solve(A.double(), b.double())
    err = ((x.double() - want).norm() / want.norm()).item()
    err_lib = ((lib.double() - want).norm() / want.norm()).item()
    assert err < 1e-4 and err < 4 * err_lib + 1e-6, (err, err_lib)
    assert torch.equal(chol_solve(L, D, b), x)  # deterministic
    with pytest.raises(ValueError):
        cholesky_lower(A, inverse=True, diag_inv=True)


@pytest.mark.gpu
@pytest.mark.parametrize("j", [0, 37, 255, 256, 700])
def test_cholesky_lower_info_first_bad_minor(j, cuda_dev):
    """A = T D T^T with T unit lower (small entries) and D = I except D_jj = -1: the leading minor of order m is
    prod_{i < m} D_i, so the first that is not positive has order j + 1 — the blocked factorization reports exactly
    that.  torch.linalg.cholesky_ex (cuSOLVER) agrees except at the last column of a 256-column panel, where it was
    seen to report j + 2."""
    from ltq_research_b200.hessian import cholesky_lower
    K = 768
    g = torch.Generator(device=cuda_dev).manual_seed(j)
    T = torch.tril(torch.randn(K, K, device=cuda_dev, dtype=torch.float64, generator=g) * 0.02, -1)
    T.diagonal().fill_(1.0)
    D = torch.ones(K, device=cuda_dev, dtype=torch.float64)
    D[j] = -1.0
    A = ((T * D) @ T.T).float()
    _, info, _ = cholesky_lower(A)
    _, info_lib = torch.linalg.cholesky_ex(A)
    assert int(info) == j + 1
    assert int(info_lib) == j + 1 or (j % 256 == 255 and int(info_lib) == j + 2)


def test_factorization_entry_checks_cpu():
    """cholesky_lower / tri_inv_lower take square fp32 CUDA matrices with a multiple of 256 rows and raise otherwise
    (there is no CPU path)."""
    from ltq_research_b200.hessian import cholesky_lower, tri_inv_lower
    for bad in (torch.eye(256), torch.eye(256, dtype=torch.float64), torch.zeros(256, 512), torch.eye(200)):
        with pytest.raises(ValueError):
            cholesky_lower(bad)
        with pytest.raises(ValueError):
            tri_inv_lower(bad)
