"""Hessian accumulation and factorization on the B200 (lumen-inference/ltq-research src/liqk_v2.py:207-231 and
:1066-1088).

* CovAccumulator — the reference's _CovAccumulator: H = (1/N) sum X^T X over calibration batches, the batch Gram on the
  tensor cores (bf16 / fp16 operands, fp32 output) or as an fp32 product, the batches summed in fp64.  Same API (add,
  get, H, n) and, for the same inputs on the same device, the same bits: the Gram is the same library product and the
  fp64 sum adds the same exactly converted values (one fused fp32 -> fp64 add instead of a conversion and an add).
* tri_inv_lower — X = L^-1 for the lower-triangular Cholesky factor, the K x K triangular inverse behind
  U = flip(L^-1) (:1079-1082).  The reference solves L X = I with a general triangular solve (O(K^3) work that does
  not use the zeros of I); here the 256 x 256 diagonal blocks are inverted by forward substitution in one kernel
  (ltq_trtri256_lower) and adjacent inverted blocks are merged level by level, X21 = -C^-1 (L21 A^-1) for
  L = [[A, 0], [L21, C]], with the two products of every level as one batched tensor-core GEMM each in the six-product
  bf16 form (fp32-accurate, the error bound of an fp32 product).  log2(K / 256) levels, about seven launches each.
* cholesky_lower — the factorization itself (the reference's torch.linalg.cholesky of flip(H_reg), :1078, and the
  refit system's solve, :1163), right-looking in 256-column panels: the diagonal block is factored and its factor
  inverted by one single-CTA kernel (ltq_chol256_diag, which also emits the six-slot operand of the block inverse), the
  panel below it is L21 = A21 L11^-T and the trailing matrix A22 -= L21 L21^T, both tensor-core GEMMs in the six-product
  bf16 form.  The trailing product covers about three quarters of the square instead of all of it (the strictly upper
  part is never read).  With inverse=True the diagonal block inverses seed tri_inv_lower, so the factor and its inverse
  cost one pass of leaf kernels.
"""
from __future__ import annotations

from typing import List, Optional, Tuple

import torch

from . import _lib, tcgemm
from ._lib import ptr

QK = 256


class CovAccumulator:
    """H = (1/N) sum over batches of X^T X (src/liqk_v2.py:207-231), accumulated on the batch's device without
    keeping X: bf16 / fp16 batches by a half-precision tensor-core GEMM with fp32 output, fp32 batches by an fp32
    product; batches summed in fp64."""

    def __init__(self):
        self.H: Optional[torch.Tensor] = None
        self.n = 0

    def add(self, x: torch.Tensor):
        x_2d = x.detach().reshape(-1, x.shape[-1])
        if x_2d.dtype in (torch.bfloat16, torch.float16):
            gram = torch.mm(x_2d.T, x_2d, out_dtype=torch.float32)
        else:
            x_2d = x_2d.float()
            gram = x_2d.T @ x_2d
        if self.H is None:
            self.H = torch.zeros((x_2d.shape[1],) * 2, dtype=torch.float64, device=x_2d.device)
        self.H.add_(gram)  # fp32 -> fp64 is exact: the same sums as converting first
        self.n += x_2d.shape[0]

    def get(self) -> torch.Tensor:
        return (self.H / max(self.n, 1)).to(torch.float32)


def _stream(dev) -> int:
    return torch.cuda.current_stream(dev).cuda_stream


def _check(rc: int, what: str):
    if rc != 0:
        raise RuntimeError(f"{what}: error {rc}")


def _square_fp32_cuda(A: torch.Tensor, what: str):
    if A.dim() != 2 or A.shape[0] != A.shape[1] or A.shape[0] % QK or A.dtype != torch.float32 or not A.is_cuda:
        raise ValueError(f"{what}: a square fp32 CUDA matrix with a multiple of 256 rows is required")


def tri_inv_lower(L: torch.Tensor, X: Optional[torch.Tensor] = None) -> torch.Tensor:
    """L^-1 (row-major fp32 [K, K], upper part exactly 0) of a lower-triangular fp32 L with K a multiple of 256, any
    layout, on the current stream, without host synchronisation.  X: a row-major [K, K] whose 256 x 256 diagonal
    blocks already hold the inverses of L's diagonal blocks and whose other blocks are 0 (cholesky_lower leaves it so);
    the merges then complete it in place."""
    _square_fp32_cuda(L, "tri_inv_lower")
    K = L.shape[0]
    Lr = L if L.stride(1) == 1 and L.stride(0) == K else L.contiguous()
    st = _stream(L.device)
    nb = K // QK
    if X is None:
        X = torch.zeros_like(Lr)
        _check(_lib.lib().ltq_trtri256_lower(ptr(Lr), K, nb, ptr(X), K, st), "ltq_trtri256_lower")
    elif X.shape != Lr.shape or X.stride() != (K, 1) or X.dtype != torch.float32:
        raise ValueError("tri_inv_lower: X must be a row-major fp32 matrix of L's shape")
    blocks: List[Tuple[int, int]] = [(QK * i, QK) for i in range(nb)]  # inverted diagonal blocks (start, size)
    while len(blocks) > 1:
        pairs = [(blocks[2 * i], blocks[2 * i + 1]) for i in range(len(blocks) // 2)]
        carry = [blocks[-1]] if len(blocks) % 2 else []
        # all pairs but possibly the last have equal halves (every block of a level has one size, except a carried
        # smaller last block); equal pairs sit at a constant stride along the diagonal and run as one batch
        eq = [p for p in pairs if p[0][1] == p[1][1] == pairs[0][0][1]]
        rest = pairs[len(eq):]
        if eq:
            _merge(Lr, X, eq[0][0][0], eq[0][0][1], eq[0][1][1], len(eq), 2 * eq[0][0][1])
        for (a0, ba), (c0, bc) in rest:
            _merge(Lr, X, a0, ba, bc, 1, 0)
        blocks = [(a0, ba + bc) for (a0, ba), (_, bc) in pairs] + carry
    return X


def _merge(Lr: torch.Tensor, X: torch.Tensor, a0: int, ba: int, bc: int, batch: int, step: int):
    """For z < batch, with s = a0 + z step: X[s+ba : s+ba+bc, s : s+ba] = -X_C (L21 X_A), X_A = X[s:s+ba, s:s+ba]
    and X_C = X[s+ba : s+ba+bc, s+ba : s+ba+bc] the inverted diagonal blocks, L21 = L[s+ba : s+ba+bc, s : s+ba]."""
    K = X.shape[0]
    bs = step * (K + 1)  # batch stride along the diagonal, in elements
    c0 = a0 + ba
    L21 = Lr.as_strided((batch, bc, ba), (bs, K, 1), Lr.storage_offset() + c0 * K + a0)
    XA = X.as_strided((batch, ba, ba), (bs, K, 1), X.storage_offset() + a0 * K + a0)
    XC = X.as_strided((batch, bc, bc), (bs, K, 1), X.storage_offset() + c0 * K + c0)
    X21 = X.as_strided((batch, bc, ba), (bs, K, 1), X.storage_offset() + c0 * K + a0)
    # T = L21 X_A  [bc, ba], then X21 = (-X_C) T written in place: batched six-product tensor-core GEMMs
    T = torch.empty((batch, bc, ba), dtype=torch.float32, device=X.device)
    tcgemm.gemm3(tcgemm.split3(L21, Kp=ba), tcgemm.split3(XA, trans=True, Kp=ba), T, ba)
    tcgemm.gemm3(tcgemm.split3(XC, neg=True, Kp=bc), tcgemm.split3(T, trans=True, Kp=bc), X21, bc)


def cholesky_lower(A: torch.Tensor, inverse: bool = False, overwrite: bool = False, diag_inv: bool = False
                   ) -> Tuple[torch.Tensor, torch.Tensor, Optional[torch.Tensor]]:
    """(L, info, X): the lower Cholesky factor of the symmetric positive definite fp32 A (lower triangle read; K a
    multiple of 256), row-major with exact zeros above the diagonal; info an int32 device scalar, 0 or the order of the
    first leading minor that is not positive (torch.linalg.cholesky_ex's convention; the factor is then not usable);
    X = L^-1 (as tri_inv_lower) with inverse=True; with diag_inv=True instead the inverses of L's 256 x 256 diagonal
    blocks [K / 256, 256, 256] (lower triangles; what chol_solve needs), as the leaves compute them; else None.
    overwrite=True factors a contiguous A in place.  On the current stream, without host synchronisation."""
    _square_fp32_cuda(A, "cholesky_lower")
    K = A.shape[0]
    dev = A.device
    if not (overwrite and A.is_contiguous()):
        A = A.contiguous().clone() if A.is_contiguous() else A.contiguous()
    if inverse and diag_inv:
        raise ValueError("cholesky_lower: inverse and diag_inv are exclusive")
    info = torch.zeros(1, dtype=torch.int32, device=dev)
    X = torch.zeros_like(A) if inverse else None
    D = torch.zeros((K // QK, QK, QK), dtype=torch.float32, device=dev) if diag_inv else None
    xt3 = torch.empty((QK, 3 * QK), dtype=torch.bfloat16, device=dev)  # the leaf's compact operand of L11^-1
    st = _stream(dev)
    L_ = _lib.lib()
    nb = K // QK
    for p in range(nb):
        c0, c1 = QK * p, QK * (p + 1)
        if D is not None:  # the leaf's inverse into its own compact block (row stride 256)
            _check(L_.ltq_chol256_diag(ptr(A), K, c0, ptr(xt3), ptr(D[p]), QK, ptr(info), st), "ltq_chol256_diag")
        else:
            _check(L_.ltq_chol256_diag(ptr(A), K, c0, ptr(xt3), ptr(X) if X is not None else None, K, ptr(info), st),
                   "ltq_chol256_diag")
        if c1 == K:
            break
        m = K - c1
        A21 = A[c1:, c0:c1]
        # L21 = A21 L11^-T written over A21 (beta = 0: the old values are not read; the operand is split first)
        tcgemm.gemm3(tcgemm.split3(A21, Kp=QK), xt3, A21, QK)
        parts = tcgemm.split3(A21, Kp=QK)  # [m, 768]: L21 = [l0 l1 l2], both operands of L21 L21^T
        A22 = A[c1:, c1:]
        h = QK * (m // QK // 2) if m >= 4 * QK else m
        # A22 -= L21 L21^T on the lower triangle's cover: the leading h x h square, then the rows below it in full
        tcgemm.gemm3(parts[:h], parts[:h], A22[:h, :h], QK, alpha=-1.0, beta=1.0)
        if h < m:
            tcgemm.gemm3(parts[h:], parts, A22[h:], QK, alpha=-1.0, beta=1.0)
        del parts
    A.tril_()
    if inverse:
        tri_inv_lower(A, X)
    return A, info.view(()), (D if diag_inv else X)


def chol_solve(L: torch.Tensor, Dinv: torch.Tensor, b: torch.Tensor) -> torch.Tensor:
    """x with L L^T x = b (src/liqk_v2.py:1163's solve of the refit system, factored by cholesky_lower with
    diag_inv=True): block forward and backward substitution through the inverted diagonal blocks, 2 K / 256 launches
    (ltq_chol_solve), no library kernel.  L [K, K] fp32 lower, Dinv [K / 256, 256, 256], b [K]; on the current stream."""
    K = L.shape[0]
    if L.dtype != torch.float32 or not L.is_cuda or L.stride(1) != 1 or Dinv.shape != (K // QK, QK, QK):
        raise ValueError("chol_solve: an fp32 CUDA factor with unit column stride and its diagonal-block inverses")
    b = b.float().contiguous()
    x = torch.empty(K, dtype=torch.float32, device=L.device)
    work = torch.empty(2 * K, dtype=torch.float32, device=L.device)
    _check(_lib.lib().ltq_chol_solve(ptr(L), L.stride(0), K, ptr(Dinv.contiguous()), ptr(b), ptr(x), ptr(work),
                                     _stream(L.device)), "ltq_chol_solve")
    return x
