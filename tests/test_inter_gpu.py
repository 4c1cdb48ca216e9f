"""GPU: the operands of the LDLQ inter-block update (src/liqk_v2.py:972-979) in the six-product bf16 form —
ltq_ldlq_bcat (right operands of every block, built once per matrix) and ltq_ldlq_inter (W_hat, the fp16 block scale and
the split of err = (w - d G) @ Uinv per block).  The split and W_hat / d are bit-exact against torch's own operations;
err and the whole update are held to the fp32 error bound of a dot product of their length."""
import pytest
import torch

pytestmark = pytest.mark.gpu
U_RND = 2.0 ** -24


def _gamma(n):
    return n * U_RND / (1 - n * U_RND)


def _wide(shape, g, dev):
    return (torch.randn(*shape, generator=g) * torch.exp(torch.randn(*shape, generator=g))).to(dev)


@pytest.mark.parametrize("K", [256, 512, 1280])
def test_ldlq_bcat_is_the_split_of_U(K, cuda_dev):
    from ltq_research_b200 import _lib
    from ltq_research_b200.liqk_v2 import _bcat, _split3
    g = torch.Generator().manual_seed(K)
    U = _wide((K, K), g, cuda_dev)
    n = int(_lib.lib().ltq_ldlq_bcat_elems(K))
    assert n == sum(1536 * (K - 256 * (b + 1)) for b in range(K // 256 - 1))
    out = torch.full((max(n, 1),), -1, dtype=torch.int16, device=cuda_dev)
    st = torch.cuda.current_stream().cuda_stream
    assert _lib.lib().ltq_ldlq_bcat(U.data_ptr(), K, K, out.data_ptr(), st) == 0
    torch.cuda.synchronize()
    off = 0
    for b in range(K // 256 - 1):
        c0, c1 = 256 * b, 256 * (b + 1)
        want = _bcat(_split3(U[c0:c1, c1:].contiguous())).view(torch.int16)
        nb = K - c1
        assert torch.equal(out[off:off + 1536 * nb].view(1536, nb), want), b
        off += 1536 * nb
    assert off == n


def test_ldlq_inter_operands_and_update(cuda_dev):
    from ltq_research_b200 import _lib
    g = torch.Generator().manual_seed(11)
    M, K, ibl = 96, 1024, 1
    c0, c1 = 256 * ibl, 256 * (ibl + 1)
    nblk = K // 256
    W = _wide((M, K), g, cuda_dev)
    G = _wide((M, K), g, cuda_dev)
    d_all = (torch.rand(M, nblk, generator=g) + 0.25).to(cuda_dev)
    d_all[3, ibl] = 0.0    # clamped to 1e-8
    d_all[5, ibl] = 1e-12
    A = torch.randn(256, 256, generator=g) / 16
    Ub = (torch.triu(A) + 2 * torch.eye(256)).to(cuda_dev)
    Uinv = torch.linalg.solve_triangular(Ub, torch.eye(256, device=cuda_dev), upper=True).contiguous()
    U = _wide((K, K), g, cuda_dev)
    what = torch.full((M, K), float("nan"), device=cuda_dev)
    d_full = torch.zeros((M, nblk), dtype=torch.float16, device=cuda_dev)
    acat = torch.zeros((M, 1536), dtype=torch.bfloat16, device=cuda_dev)
    st = torch.cuda.current_stream().cuda_stream
    L = _lib.lib()
    rc = L.ltq_ldlq_inter(W.data_ptr() + 4 * c0, K, d_all.data_ptr() + 4 * ibl, nblk, G.data_ptr() + 4 * c0, K,
                          Uinv.data_ptr(), 256, M, what.data_ptr() + 4 * c0, K, d_full.data_ptr() + 2 * ibl, nblk,
                          acat.data_ptr(), st)
    torch.cuda.synchronize()
    assert rc == 0
    # the reference's operations (src/liqk_v2.py:966-979): d = clamp(d_rb, 1e-8), what = d * G, d_full = fp16(d)
    d = d_all[:, ibl].clamp(min=1e-8)
    want_what = d.unsqueeze(1) * G[:, c0:c1]
    assert torch.equal(what[:, c0:c1], want_what)
    assert torch.isnan(what[:, :c0]).all() and torch.isnan(what[:, c1:]).all()
    assert torch.equal(d_full[:, ibl], d.to(torch.float16))
    assert (d_full[:, :ibl] == 0).all() and (d_full[:, ibl + 1:] == 0).all()
    # acat = [e0 e0 e1 e0 e1 e2]; e0 + e1 + e2 = err within the fp32 dot-product bound of length 256
    parts = acat.view(M, 6, 256)
    assert torch.equal(parts[:, 0], parts[:, 1]) and torch.equal(parts[:, 0], parts[:, 3])
    assert torch.equal(parts[:, 2], parts[:, 4])
    e = (W[:, c0:c1] - want_what).double()
    err64 = e @ Uinv.double()
    err = parts[:, 0].double() + parts[:, 2].double() + parts[:, 5].double()
    bound = _gamma(256) * (e.abs() @ Uinv.double().abs()) + 2 * U_RND * err64.abs()
    assert ((err - err64).abs() <= bound).all()
    # the update as the pipeline issues it: W[:, c1:] -= acat @ bcat_b (one GEMM, fp32 accumulation)
    bcat = torch.empty(int(L.ltq_ldlq_bcat_elems(K)), dtype=torch.bfloat16, device=cuda_dev)
    assert L.ltq_ldlq_bcat(U.data_ptr(), K, K, bcat.data_ptr(), st) == 0
    off = sum(1536 * (K - 256 * (b + 1)) for b in range(ibl))
    nb = K - c1
    W2 = W.clone()
    Wv = W2[:, c1:]
    torch.addmm(Wv, acat, bcat[off:off + 1536 * nb].view(1536, nb), out_dtype=torch.float32, beta=1, alpha=-1, out=Wv)
    torch.cuda.synchronize()
    assert torch.equal(W2[:, :c1], W[:, :c1])
    Ur = U[c0:c1, c1:].double()
    want = W[:, c1:].double() - err64 @ Ur
    # err's own error (above) carried through U, plus the fp32 bound of the length-256 product and the subtraction
    tol = ((bound + _gamma(256) * err64.abs()) @ Ur.abs() + _gamma(256) * (err64.abs() @ Ur.abs())
           + 2 * U_RND * want.abs())
    assert ((W2[:, c1:].double() - want).abs() <= 2 * tol).all()


def test_bf16x6_operands_one_kernel_equal_torch_split(cuda_dev):
    """_left6 / _right6 (ltq_bf16x6_split, one launch) equal _acat(_split3(x)) / _bcat(_split3(x)) bit for bit, for
    row-major operands and transposed views, including values at bf16 rounding ties and subnormal remainders."""
    from ltq_research_b200.liqk_v2 import _acat, _bcat, _left6, _right6, _split3
    g = torch.Generator().manual_seed(4)
    x = _wide((96, 160), g, cuda_dev)
    x[0, :8] = torch.tensor([1 + 2 ** -8, 1 + 3 * 2 ** -8, -(1 + 2 ** -8), 2 ** -130, 1e-38, 0.0, -0.0, 3e38])
    for a in (x, x.T.contiguous().T):
        assert torch.equal(_left6(a).view(torch.int16), _acat(_split3(a.contiguous())).view(torch.int16))
        assert torch.equal(_right6(a).view(torch.int16), _bcat(_split3(a.contiguous())).view(torch.int16))


def test_block_inverses_from_the_cholesky_factor(cuda_dev):
    """The fast mode takes U_blk^-1 from the Cholesky factor (U = P L^-1 P, so U^-1 = P L P and its diagonal blocks are
    the flipped diagonal blocks of L) instead of solving U_blk X = I: the two agree to fp32 rounding, for L in the
    layout the factorization returns."""
    g = torch.Generator(device=cuda_dev).manual_seed(2)
    K = 1024
    nb = K // 256
    X = torch.randn(4096, K, device=cuda_dev, dtype=torch.float64, generator=g)
    H = (X.T @ X / 4096).float()
    H.diagonal().add_(0.05 * H.diagonal().mean())
    L, info = torch.linalg.cholesky_ex(H.flip(0, 1))
    assert int(info) == 0
    U = torch.linalg.solve_triangular(L, torch.eye(K, device=cuda_dev), upper=False).flip(0, 1)
    Ub = torch.stack([U[b * 256:(b + 1) * 256, b * 256:(b + 1) * 256] for b in range(nb)])
    ref = torch.linalg.solve_triangular(Ub, torch.eye(256, device=cuda_dev).expand(nb, -1, -1), upper=True)
    s0, s1 = L.stride()
    got = L.as_strided((nb, 256, 256), (256 * (s0 + s1), s0, s1), L.storage_offset()).flip(0, 1, 2)
    assert ((got - ref).norm() / ref.norm()).item() < 1e-5
    assert (torch.bmm(Ub, got) - torch.eye(256, device=cuda_dev)).abs().max().item() < 1e-4
    assert torch.equal(torch.triu(got), got)


@pytest.mark.parametrize("K", [512, 1024, 1280])
def test_gram_lower_lower_triangle(K, cuda_dev):
    """tcgemm.gram_lower(x) (the refit's Gram matrix on the tcgen05 GEMM, computed on the lower triangle's cover only,
    as the fast mode calls it) against fp64 x^T x: every element on or below the diagonal within the fp32 error bound
    of a dot product of length M, and every 256 x 256 diagonal block computed in full (the blockwise Cholesky reads
    whole diagonal blocks)."""
    from ltq_research_b200 import tcgemm
    g = torch.Generator().manual_seed(K)
    M = 640
    x = _wide((M, K), g, cuda_dev)
    C = tcgemm.gram_lower(x, 256 * (K // 256 // 2) if K >= 4 * 256 else K)
    torch.cuda.synchronize()
    xd = x.double()
    want = xd.T @ xd
    bound = _gamma(M) * (xd.abs().T @ xd.abs()) + 2 * U_RND * want.abs()
    low = torch.tril(torch.ones(K, K, dtype=torch.bool, device=cuda_dev))
    for b in range(K // 256):
        low[256 * b:256 * (b + 1), 256 * b:256 * (b + 1)] = True
    assert ((C.double() - want).abs() <= 2 * bound)[low].all()
