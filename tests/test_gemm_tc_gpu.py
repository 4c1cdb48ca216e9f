"""GPU: the tensor-core GEMMs (ltq_gemm_bf16_tn and the six-product ltq_gemm_bf16x6_tn: tcgen05.mma, TMA, tensor-memory
accumulator) and the compact K-major operands of the LDLQ inter-block update (ltq_ldlq_bcat_t, ltq_ldlq_inter3).

* Small-integer operands make every product and every partial sum exact in fp32, so C must equal the integer reference
  exactly: any error in the shared-memory descriptors, the swizzle, the K stepping, the tensor-memory read-back or the
  edge handling shows up as a mismatch.  Ragged M, N not a multiple of the 256-wide tile, padded row strides, a strided
  C view, beta 0 / 1 / 0.5, alpha -1 / 1.
* Real-valued operands: within the fp32 accumulation bound |C - C64| <= (Kd + 2) u (|alpha| |A||B|^T + |beta C|).
* The six-product kernel from three-part operands equals the concatenated six-slot product exactly on integers.
* ltq_ldlq_bcat_t / ltq_ldlq_inter3 hold the three parts of ltq_ldlq_bcat's / ltq_ldlq_inter's six slots (transposed
  for the right operand), bit for bit; the inter-block update through the six-product tensor-core GEMM agrees with the
  same six-product form through torch (cuBLAS) within the fp32 bound of the 1536-term sum.
"""
import pytest
import torch

pytestmark = pytest.mark.gpu
U32 = 2.0 ** -24


def _gemm(A, B, C, alpha, beta, M=None, N=None, err=None):
    from ltq_research_b200 import _lib
    M = A.shape[0] if M is None else M
    N = B.shape[0] if N is None else N
    Kd = A.shape[1]
    rc = _lib.lib().ltq_gemm_bf16_tn(A.data_ptr(), A.stride(0), B.data_ptr(), B.stride(0), C.data_ptr(), C.stride(0),
                                     M, N, Kd, alpha, beta, None if err is None else err.data_ptr(),
                                     torch.cuda.current_stream().cuda_stream)
    return rc


@pytest.mark.parametrize("M,N,Kd,alpha,beta", [(128, 256, 64, 1.0, 0.0), (16, 16, 64, -1.0, 1.0),
                                               (1040, 272, 1536, -1.0, 1.0), (300, 2816, 1536, 1.0, 0.5),
                                               (4096, 512, 192, -1.0, 1.0)])
def test_gemm_exact_on_small_integers(cuda_dev, M, N, Kd, alpha, beta):
    g = torch.Generator(device=cuda_dev).manual_seed(M + N + Kd)
    A = torch.randint(-3, 4, (M, Kd + 8), generator=g, device=cuda_dev).to(torch.bfloat16)[:, :Kd]
    B = torch.randint(-3, 4, (N, Kd + 16), generator=g, device=cuda_dev).to(torch.bfloat16)[:, :Kd]
    Cw = torch.randint(-1000, 1000, (M, N + 20), generator=g, device=cuda_dev).float()
    C = Cw[:, 4:4 + N]  # strided view, 16-byte aligned
    want = beta * C.double() + alpha * (A.double() @ B.double().T)
    err = torch.zeros(1, dtype=torch.int32, device=cuda_dev)
    guard = Cw.clone()
    assert _gemm(A, B, C, alpha, beta, err=err) == 0
    torch.cuda.synchronize()
    assert int(err) == 0
    assert torch.equal(C.double(), want)
    # the columns outside the view are untouched
    assert torch.equal(Cw[:, :4], guard[:, :4]) and torch.equal(Cw[:, 4 + N:], guard[:, 4 + N:])


def test_gemm_real_values_within_fp32_bound(cuda_dev):
    g = torch.Generator(device=cuda_dev).manual_seed(3)
    M, N, Kd = 777, 1024, 1536
    A = torch.randn(M, Kd, generator=g, device=cuda_dev).to(torch.bfloat16)
    B = torch.randn(N, Kd, generator=g, device=cuda_dev).to(torch.bfloat16)
    C = torch.randn(M, N, generator=g, device=cuda_dev)
    C0 = C.double().clone()
    assert _gemm(A, B, C, -1.0, 1.0) == 0
    torch.cuda.synchronize()
    ref = C0 - A.double() @ B.double().T
    bound = (Kd + 2) * U32 * (A.double().abs() @ B.double().abs().T + C0.abs())
    assert ((C.double() - ref).abs() <= bound).all()


def test_gemm_rejects_bad_arguments(cuda_dev):
    A = torch.zeros(16, 64, dtype=torch.bfloat16, device=cuda_dev)
    C = torch.zeros(16, 16, device=cuda_dev)
    assert _gemm(A, A, C, 1.0, 0.0, N=8) == -1           # N not a multiple of 16
    A2 = torch.zeros(16, 96, dtype=torch.bfloat16, device=cuda_dev)
    assert _gemm(A2, A2, C, 1.0, 0.0) == -1              # Kd not a multiple of 64
    assert _gemm(A, A, C, 1.0, 0.0, M=0) == 0            # empty: nothing launched


def _gemm6(A3, B3, C, alpha, beta, Kp, err=None):
    from ltq_research_b200 import _lib
    return _lib.lib().ltq_gemm_bf16x6_tn(A3.data_ptr(), A3.stride(0), B3.data_ptr(), B3.stride(0), C.data_ptr(),
                                         C.stride(0), A3.shape[0], B3.shape[0], Kp, alpha, beta,
                                         None if err is None else err.data_ptr(), torch.cuda.current_stream().cuda_stream)


def _six(X3, Kp, order):
    """The concatenated six-slot operand of three parts: left [x0 x0 x1 x0 x1 x2], right [x0 x1 x0 x2 x1 x0]."""
    p = [X3[:, i * Kp:(i + 1) * Kp] for i in range(3)]
    idx = (0, 1, 0, 2, 1, 0) if order else (0, 0, 1, 0, 1, 2)
    return torch.cat([p[i] for i in idx], dim=1).contiguous()


# (2600, 4112, 128): 21 x 17 = 357 tiles, more than the SMs, so the beta 0 / 1 products run on the persistent kernel
# (CTAs walking two or three tiles each, a 16-column tail block)
@pytest.mark.parametrize("M,N,Kp", [(16, 16, 64), (1040, 272, 256), (300, 2816, 256), (2048, 512, 128),
                                    (2600, 4112, 128)])
def test_gemm6_exact_on_small_integers(cuda_dev, M, N, Kp):
    g = torch.Generator(device=cuda_dev).manual_seed(M + 3 * N + Kp)
    A3 = torch.randint(-3, 4, (M, 3 * Kp), generator=g, device=cuda_dev).to(torch.bfloat16)
    B3 = torch.randint(-3, 4, (N, 3 * Kp + 8), generator=g, device=cuda_dev).to(torch.bfloat16)[:, :3 * Kp]
    C0 = torch.randint(-1000, 1000, (M, N), generator=g, device=cuda_dev).float()
    a = [A3[:, i * Kp:(i + 1) * Kp].double() for i in range(3)]
    b = [B3[:, i * Kp:(i + 1) * Kp].double() for i in range(3)]
    six = a[0] @ b[0].T + a[0] @ b[1].T + a[1] @ b[0].T + a[0] @ b[2].T + a[1] @ b[1].T + a[2] @ b[0].T
    err = torch.zeros(1, dtype=torch.int32, device=cuda_dev)
    C = C0.clone()
    assert _gemm6(A3, B3, C, -1.0, 1.0, Kp, err) == 0
    C2 = C0.clone()
    assert _gemm(_six(A3, Kp, 0), _six(B3, Kp, 1), C2, -1.0, 1.0) == 0
    torch.cuda.synchronize()
    assert int(err) == 0
    assert torch.equal(C.double(), C0.double() - six) and torch.equal(C, C2)


@pytest.mark.parametrize("K", [512, 1280, 3072])
def test_bcat_t_is_bcat_transposed(cuda_dev, K):
    from ltq_research_b200 import _lib
    L = _lib.lib()
    g = torch.Generator(device=cuda_dev).manual_seed(K)
    U = torch.triu(torch.randn(K, K, generator=g, device=cuda_dev))
    n = int(L.ltq_ldlq_bcat_elems(K))
    a = torch.empty(n, dtype=torch.int16, device=cuda_dev)
    b = torch.empty(n // 2, dtype=torch.int16, device=cuda_dev)
    st = torch.cuda.current_stream().cuda_stream
    assert L.ltq_ldlq_bcat(U.data_ptr(), K, K, a.data_ptr(), st) == 0
    assert L.ltq_ldlq_bcat_t(U.data_ptr(), K, K, b.data_ptr(), st) == 0
    torch.cuda.synchronize()
    off6 = off3 = 0
    for blk in range(K // 256 - 1):
        nb = K - 256 * (blk + 1)
        six = a[off6:off6 + 1536 * nb].view(1536, nb)
        three = b[off3:off3 + 768 * nb].view(nb, 768)
        for part, slot in ((0, 0), (1, 1), (2, 3)):  # the right slots [u0 u1 u0 u2 u1 u0]
            assert torch.equal(six[256 * slot:256 * slot + 256].T, three[:, 256 * part:256 * part + 256]), (blk, part)
        off6 += 1536 * nb
        off3 += 768 * nb


def test_inter3_is_inter_compact(cuda_dev):
    from ltq_research_b200 import _lib
    L = _lib.lib()
    g = torch.Generator(device=cuda_dev).manual_seed(8)
    M = 64
    w = torch.randn(M, 256, generator=g, device=cuda_dev)
    d = torch.rand(M, 1, generator=g, device=cuda_dev) + 0.5
    G = torch.randn(M, 256, generator=g, device=cuda_dev)
    Ui = torch.triu(torch.randn(256, 256, generator=g, device=cuda_dev)) / 8 + torch.eye(256, device=cuda_dev)
    st = torch.cuda.current_stream().cuda_stream
    outs = []
    for fn, width in ((L.ltq_ldlq_inter, 1536), (L.ltq_ldlq_inter3, 768)):
        what = torch.empty(M, 256, device=cuda_dev)
        dh = torch.empty(M, 1, dtype=torch.int16, device=cuda_dev)
        ac = torch.empty(M, width, dtype=torch.int16, device=cuda_dev)
        assert fn(w.data_ptr(), 256, d.data_ptr(), 1, G.data_ptr(), 256, Ui.data_ptr(), 256, M, what.data_ptr(), 256,
                  dh.data_ptr(), 1, ac.data_ptr(), st) == 0
        outs.append((what, dh, ac))
    torch.cuda.synchronize()
    (w6, d6, a6), (w3, d3, a3) = outs
    assert torch.equal(w6, w3) and torch.equal(d6, d3)
    for part, slot in ((0, 0), (1, 2), (2, 5)):  # the left slots [e0 e0 e1 e0 e1 e2]
        assert torch.equal(a6[:, 256 * slot:256 * slot + 256], a3[:, 256 * part:256 * part + 256]), part


def test_inter_block_update_tensor_core_vs_library(cuda_dev):
    """W[:, c1:] -= six-product(acat3, bcat3_b) for one block: the tcgen05 six-product GEMM against torch's GEMM of the
    concatenated six-slot operands, both within the fp32 bound of the 1536-term sum."""
    from ltq_research_b200 import _lib
    L = _lib.lib()
    g = torch.Generator(device=cuda_dev).manual_seed(5)
    M, K = 1024, 1024
    U = torch.triu(torch.randn(K, K, generator=g, device=cuda_dev)) / 16
    n = int(L.ltq_ldlq_bcat_elems(K)) // 2
    bt = torch.empty(n, dtype=torch.bfloat16, device=cuda_dev)
    st = torch.cuda.current_stream().cuda_stream
    assert L.ltq_ldlq_bcat_t(U.data_ptr(), K, K, bt.data_ptr(), st) == 0
    acat3 = torch.randn(M, 768, generator=g, device=cuda_dev).to(torch.bfloat16)
    W = torch.randn(M, K, generator=g, device=cuda_dev)
    nb = K - 256
    B3 = bt[:768 * nb].view(nb, 768)
    W1 = W.clone()
    assert _gemm6(acat3, B3, W1[:, 256:], -1.0, 1.0, 256) == 0
    A6, B6 = _six(acat3, 256, 0), _six(B3, 256, 1)
    W2 = W.clone()
    torch.addmm(W2[:, 256:], A6, B6.T, out_dtype=torch.float32, beta=1, alpha=-1, out=W2[:, 256:])
    torch.cuda.synchronize()
    ref = W[:, 256:].double() - A6.double() @ B6.double().T
    bound = (1536 + 2) * U32 * (A6.double().abs() @ B6.double().abs().T + W[:, 256:].double().abs())
    for got in (W1, W2):
        assert torch.equal(got[:, :256], W[:, :256])
        assert ((got[:, 256:].double() - ref).abs() <= bound).all()


def _parts(x):
    """The three-way bf16 split in torch (each difference exact in fp32)."""
    x0 = x.to(torch.bfloat16)
    r = x - x0.float()
    x1 = r.to(torch.bfloat16)
    x2 = (r - x1.float()).to(torch.bfloat16)
    return x0, x1, x2


@pytest.mark.parametrize("trans,neg", [(False, False), (True, False), (False, True), (True, True)])
def test_split3_layout(cuda_dev, trans, neg):
    from ltq_research_b200.tcgemm import split3
    g = torch.Generator(device=cuda_dev).manual_seed(4)
    big = torch.randn(3, 50, 120, generator=g, device=cuda_dev) * 7
    x = big[:, 3:43, 8:108]  # batch 3 of [40, 100], strided
    Kp = 128
    got = split3(x, trans=trans, neg=neg, Kp=Kp)
    src = -x if neg else x
    src = src.transpose(1, 2) if trans else src
    k = src.shape[2]
    want = torch.zeros(3, src.shape[1], 3 * Kp, dtype=torch.bfloat16, device=cuda_dev)
    for p, part in enumerate(_parts(src.contiguous())):
        want[:, :, p * Kp:p * Kp + k] = part
    assert torch.equal(got.view(torch.int16), want.view(torch.int16))


@pytest.mark.parametrize("nq,batch", [(2, 3), (3, 3), (3, 50)])
def test_gemm3_batched_exact(cuda_dev, nq, batch):
    """Batched part GEMM on small integers into strided C views: beta 0 (TMA store), 1 (TMA reduce-add), 0.5
    (read-modify-write), exactly the integer sum of the nq (nq + 1) / 2 products.  Batch 50 is 200 tiles, more than
    the SMs: its beta 0 / 1 products run on the persistent kernel."""
    from ltq_research_b200.tcgemm import gemm3
    g = torch.Generator(device=cuda_dev).manual_seed(10 + nq + batch)
    M, N, Kp = 200, 272, 128
    A3 = torch.randint(-3, 4, (batch, M, 3 * Kp), generator=g, device=cuda_dev).to(torch.bfloat16)
    B3 = torch.randint(-3, 4, (batch, N, 3 * Kp), generator=g, device=cuda_dev).to(torch.bfloat16)
    a = [A3[:, :, i * Kp:(i + 1) * Kp].double() for i in range(3)]
    b = [B3[:, :, i * Kp:(i + 1) * Kp].double() for i in range(3)]
    prod = sum(a[p] @ b[q].transpose(1, 2) for p in range(3) for q in range(3) if p + q < nq)
    for beta in (0.0, 1.0, 0.5):
        big = torch.randint(-100, 100, (batch, M + 8, N + 32), generator=g, device=cuda_dev).float()
        C = big[:, 4:4 + M, 16:16 + N]
        want = beta * C.double() - prod
        guard = big.clone()
        gemm3(A3, B3, C, Kp, alpha=-1.0, beta=beta, nq=nq)
        torch.cuda.synchronize()
        assert torch.equal(C.double(), want), beta
        mask = torch.ones_like(big, dtype=torch.bool)
        mask[:, 4:4 + M, 16:16 + N] = False
        assert torch.equal(big[mask], guard[mask]), beta


def test_mm_and_gram_within_fp32_bound(cuda_dev):
    from ltq_research_b200.tcgemm import gram_lower, mm
    g = torch.Generator(device=cuda_dev).manual_seed(12)
    a = torch.randn(300, 1000, generator=g, device=cuda_dev)
    b = torch.randn(1000, 512, generator=g, device=cuda_dev) * torch.exp(torch.randn(1, 512, generator=g, device=cuda_dev))
    got = mm(a, b)
    ref = a.double() @ b.double()
    bound = (1000 + 2) * U32 * (a.double().abs() @ b.double().abs())
    torch.cuda.synchronize()
    assert ((got.double() - ref).abs() <= bound).all()
    x = torch.randn(1000, 1024, generator=g, device=cuda_dev)
    C = gram_lower(x, 512)
    ref = x.double().T @ x.double()
    bound = (1000 + 2) * U32 * (x.double().abs().T @ x.double().abs())
    low = torch.tril(torch.ones(1024, 1024, dtype=torch.bool, device=cuda_dev))
    torch.cuda.synchronize()
    assert ((C.double() - ref).abs() <= bound)[low].all()


def test_bounded_wait_times_out_with_error_flag(cuda_dev):
    """The GEMMs' pipeline waits are bounded: a wait on an mbarrier that nothing completes gives up after its poll limit,
    sets the error flag and returns (the kernel ends, the context stays usable); the same wait completes when the
    arrival is made.  No copy and no tensor memory are involved."""
    from ltq_research_b200 import _lib
    L = _lib.lib()
    st = torch.cuda.current_stream(cuda_dev).cuda_stream
    for arrive, want_err, want_done in ((1, 0, 1), (0, 1, 2)):
        err = torch.zeros(1, dtype=torch.int32, device=cuda_dev)
        done = torch.zeros(1, dtype=torch.int32, device=cuda_dev)
        assert L.ltq_gemm_wait_selftest(arrive, 4096, err.data_ptr(), done.data_ptr(), st) == 0
        torch.cuda.synchronize()
        assert int(err) == want_err and int(done) == want_done, (arrive, int(err), int(done))
    assert L.ltq_gemm_wait_selftest(0, 0, err.data_ptr(), done.data_ptr(), st) == -1
    # the device still runs work afterwards
    x = torch.ones(1024, device=cuda_dev)
    assert float(x.sum()) == 1024.0
