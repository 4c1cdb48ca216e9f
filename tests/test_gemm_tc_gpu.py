"""GPU: the tensor-core GEMM (ltq_gemm_bf16_tn: tcgen05.mma, TMA, tensor-memory accumulator) and the K-major operands of
the LDLQ inter-block update (ltq_ldlq_bcat_t).

* Small-integer operands make every product and every partial sum exact in fp32, so C must equal the integer reference
  exactly: any error in the shared-memory descriptors, the swizzle, the K stepping, the tensor-memory read-back or the
  edge handling shows up as a mismatch.  Ragged M, N not a multiple of the 256-wide tile, padded row strides, a strided
  C view, beta 0 / 1 / 0.5, alpha -1 / 1.
* Real-valued operands: within the fp32 accumulation bound |C - C64| <= (Kd + 2) u (|alpha| |A||B|^T + |beta C|).
* ltq_ldlq_bcat_t is ltq_ldlq_bcat's operand transposed, block by block, bit for bit; the inter-block update through
  the tensor-core GEMM agrees with the same six-product form through torch (cuBLAS) within the fp32 bound of the
  six-product sum.
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


@pytest.mark.parametrize("K", [512, 1280, 3072])
def test_bcat_t_is_bcat_transposed(cuda_dev, K):
    from ltq_research_b200 import _lib
    L = _lib.lib()
    g = torch.Generator(device=cuda_dev).manual_seed(K)
    U = torch.triu(torch.randn(K, K, generator=g, device=cuda_dev))
    n = int(L.ltq_ldlq_bcat_elems(K))
    a = torch.empty(n, dtype=torch.int16, device=cuda_dev)
    b = torch.empty(n, dtype=torch.int16, device=cuda_dev)
    st = torch.cuda.current_stream().cuda_stream
    assert L.ltq_ldlq_bcat(U.data_ptr(), K, K, a.data_ptr(), st) == 0
    assert L.ltq_ldlq_bcat_t(U.data_ptr(), K, K, b.data_ptr(), st) == 0
    torch.cuda.synchronize()
    off = 0
    for blk in range(K // 256 - 1):
        nb = K - 256 * (blk + 1)
        assert torch.equal(a[off:off + 1536 * nb].view(1536, nb).T, b[off:off + 1536 * nb].view(nb, 1536)), blk
        off += 1536 * nb


def test_inter_block_update_tensor_core_vs_library(cuda_dev):
    """W[:, c1:] -= acat @ bcat_b for one block: the tcgen05 GEMM against torch's GEMM of the same bf16 operands,
    both within the fp32 bound of the 1536-term sum."""
    from ltq_research_b200 import _lib
    L = _lib.lib()
    g = torch.Generator(device=cuda_dev).manual_seed(5)
    M, K = 1024, 1024
    U = torch.triu(torch.randn(K, K, generator=g, device=cuda_dev)) / 16
    n = int(L.ltq_ldlq_bcat_elems(K))
    bt = torch.empty(n, dtype=torch.bfloat16, device=cuda_dev)
    st = torch.cuda.current_stream().cuda_stream
    assert L.ltq_ldlq_bcat_t(U.data_ptr(), K, K, bt.data_ptr(), st) == 0
    acat = torch.randn(M, 1536, generator=g, device=cuda_dev).to(torch.bfloat16)
    W = torch.randn(M, K, generator=g, device=cuda_dev)
    nb = K - 256
    Bt = bt[:1536 * nb].view(nb, 1536)
    W1 = W.clone()
    assert _gemm(acat, Bt, W1[:, 256:], -1.0, 1.0) == 0
    W2 = W.clone()
    torch.addmm(W2[:, 256:], acat, Bt.T, out_dtype=torch.float32, beta=1, alpha=-1, out=W2[:, 256:])
    torch.cuda.synchronize()
    ref = W[:, 256:].double() - acat.double() @ Bt.double().T
    bound = (1536 + 2) * U32 * (acat.double().abs() @ Bt.double().abs().T + W[:, 256:].double().abs())
    for got in (W1, W2):
        assert torch.equal(got[:, :256], W[:, :256])
        assert ((got[:, 256:].double() - ref).abs() <= bound).all()
