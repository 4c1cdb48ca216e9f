"""fp32-accurate products of the fast mode on the B200 tensor cores (libltq_b200.so, tcgen05): every fp32 operand is split
as x = x0 + x1 + x2 in bf16 (24 significand bits together) into a compact part operand [x0 x1 x2] (ltq_bf16x3_split),
and ltq_gemm_bf16x3p_tn accumulates the six leading products a_p b_q^T (p + q <= 2) — or the three with p + q <= 1 —
in fp32 in tensor memory.  The error stays within the bound of an fp32 dot product of the same length,
|C - AB| <= gamma_K |A| |B|, as the library GEMM of the concatenated six-slot form did (tests/test_batch_gpu.py,
tests/test_gemm_tc_gpu.py).

Conventions: C = beta C + alpha A B with A [M, K], B [K, N] fp32; the kernel takes B as its transpose (K contiguous),
which the transposing split provides.  K is padded with zeros to a multiple of 64 (the kernel's K chunk); N must be a
multiple of 16.  Batched forms take 3-D strided views (batch, rows, cols) with unit column stride.
"""
from __future__ import annotations

from typing import Optional

import torch

from . import _lib
from ._lib import ptr

KCHUNK = 64


def _check(rc: int, what: str):
    if rc != 0:
        raise RuntimeError(f"{what}: error code {rc}")


def _pad(k: int) -> int:
    return (k + KCHUNK - 1) // KCHUNK * KCHUNK


def _strides(x: torch.Tensor):
    """(batch, rows, cols, ld, batch stride) of a 2-D or 3-D fp32 view with unit column stride."""
    if x.dim() == 2:
        x = x.unsqueeze(0)
    if x.dtype != torch.float32 or x.stride(2) != 1 or not x.is_cuda:
        raise ValueError("split3: an fp32 CUDA view with unit column stride is required")
    return x.shape[0], x.shape[1], x.shape[2], x.stride(1), x.stride(0) if x.shape[0] > 1 else 0


def split3(x: torch.Tensor, trans: bool = False, neg: bool = False, Kp: Optional[int] = None) -> torch.Tensor:
    """Compact part operand of x ([rows, cols] or [batch, rows, cols]): [rows, 3 Kp] with row r = [x0 x1 x2] of row r
    (Kp >= cols), or with trans [cols, 3 Kp] with row c = the parts of column c (Kp >= rows); zero padding up to Kp
    (default: the next multiple of 64); neg splits -x.  bf16, one kernel."""
    batch, rows, cols, ld, bs = _strides(x)
    k = rows if trans else cols
    Kp = _pad(k) if Kp is None else Kp
    orows = cols if trans else rows
    out = torch.empty((batch, orows, 3 * Kp), dtype=torch.bfloat16, device=x.device)
    _check(_lib.lib().ltq_bf16x3_split(ptr(x), ld, bs, rows, cols, batch, int(trans), int(neg), Kp, ptr(out),
                                       out.stride(1), out.stride(0), _lib.stream_ptr(x.device)), "ltq_bf16x3_split")
    return out if x.dim() == 3 else out[0]


def gemm3(A3: torch.Tensor, B3: torch.Tensor, C: torch.Tensor, Kp: int, alpha: float = 1.0, beta: float = 0.0,
          nq: int = 3, err: Optional[torch.Tensor] = None) -> torch.Tensor:
    """C = beta C + alpha sum_{p + q < nq} a_p b_q^T from part operands A3 [.., M, nq Kp], B3 [.., N, nq Kp] (bf16) into
    the fp32 view C [.., M, N] (unit column stride; batched when 3-D).  Returns C."""
    a3, b3, c3 = (t if t.dim() == 3 else t.unsqueeze(0) for t in (A3, B3, C))
    batch, M, N = c3.shape
    if a3.shape[0] != batch or b3.shape[0] != batch or a3.shape[1] != M or b3.shape[1] != N:
        raise ValueError("gemm3: operand shapes do not match")
    if err is None:
        from .liqk_v2 import gemm_error_flag
        err = gemm_error_flag(C.device)
    _check(_lib.lib().ltq_gemm_bf16x3p_tn(
        ptr(a3), a3.stride(1), a3.stride(0) if batch > 1 else 0, ptr(b3), b3.stride(1), b3.stride(0) if batch > 1 else 0,
        ptr(c3), c3.stride(1), c3.stride(0) if batch > 1 else 0, M, N, Kp, nq, batch, float(alpha), float(beta),
        ptr(err), _lib.stream_ptr(C.device)), "ltq_gemm_bf16x3p_tn")
    return C


def mm(a: torch.Tensor, b: torch.Tensor, out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """a @ b (fp32 [M, K] x [K, N], N a multiple of 16), fp32-accurate on the tensor cores."""
    K = a.shape[1]
    Kp = _pad(K)
    A3 = split3(a, Kp=Kp)
    B3 = split3(b, trans=True, Kp=Kp)
    C = out if out is not None else torch.empty((a.shape[0], b.shape[1]), dtype=torch.float32, device=a.device)
    return gemm3(A3, B3, C, Kp)


def times(a: torch.Tensor, B3: torch.Tensor, Kp: int, out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """a @ B for a prepared right operand B3 = split3(B, trans=True) (shared by several products with B)."""
    C = out if out is not None else torch.empty((a.shape[0], B3.shape[0]), dtype=torch.float32, device=a.device)
    return gemm3(split3(a, Kp=Kp), B3, C, Kp)


def gram_lower(x: torch.Tensor, half: int) -> torch.Tensor:
    """x^T x ([K, K]) of an fp32 [M, K] for a consumer that reads the lower triangle only: the leading half x half square
    and the rows below it are computed, the blocks right of the square in its rows are left uninitialised."""
    K = x.shape[1]
    Kp = _pad(x.shape[0])
    X3 = split3(x, trans=True, Kp=Kp)  # [K, 3 Kp]: row i = the parts of column i of x
    C = torch.empty((K, K), dtype=torch.float32, device=x.device)
    gemm3(X3[:half], X3[:half], C[:half, :half], Kp)
    if half < K:
        gemm3(X3[half:], X3, C[half:], Kp)
    return C
