"""TEST INFRASTRUCTURE ONLY — drives the reference CUDA kernel built from its own source (oracle/_ref, see
oracle/Makefile) the way the reference's Python wrapper does, to pin the oracle and the product against it on a GPU.

``viterbi_ub_cuda_ref`` restates src/tcq_proto.py:567-657 (scratch allocation, tail-biting schedule, code unpacking)
over ``oracle/_ref/libtcq_viterbi_ref.so`` (the unmodified src/cuda/tcq_viterbi.cu compiled for sm_100a).
Only tests/ and the golden-fixture script use it.
"""
from __future__ import annotations

import ctypes
from pathlib import Path

import torch

REF_SO = Path(__file__).resolve().parent / "_ref" / "libtcq_viterbi_ref.so"
_LIB = None


def available() -> bool:
    return REF_SO.exists()


def lib():
    global _LIB
    if _LIB is None:
        L = ctypes.CDLL(str(REF_SO))
        L.tcq_viterbi.restype = ctypes.c_int
        L.tcq_viterbi.argtypes = [ctypes.c_void_p] * 15 + [ctypes.c_int] * 18 + [ctypes.c_void_p, ctypes.c_int,
                                                                                  ctypes.c_void_p]
        _LIB = L
    return _LIB


def _p(t):
    return None if t is None else t.data_ptr()


@torch.no_grad()
def viterbi_ub_cuda_ref(x, small, K, nu, m, gains=None, sub=16, wts=None, init_state=None, return_end_state=False,
                        small_hi=None, gains_hi=None, mix=0, n_cand=0, return_code=False, tail_biting=False,
                        tb_passes=2, tb_cand1=0, tb_window=0, m_extra=(), pair_parity=False, _mid=0, _tail=False,
                        _steps=0, _rot=0):
    if tail_biting:
        N, T = x.shape
        h = T // 2
        kw = dict(sub=sub, small_hi=small_hi, gains_hi=gains_hi, mix=mix, n_cand=n_cand, m_extra=m_extra,
                  pair_parity=pair_parity)
        w_full = None if wts is None else (wts.view(1, T).expand(N, T) if wts.dim() == 1 else wts).float().contiguous()
        x = x.float().contiguous()
        kw1 = dict(kw, n_cand=tb_cand1) if tb_cand1 else kw
        if tb_window:
            _, mid = viterbi_ub_cuda_ref(x, small, K, nu, m, gains, wts=w_full, _mid=tb_window, _steps=2 * tb_window,
                                         _rot=h - tb_window, **kw1)
        else:
            _, mid = viterbi_ub_cuda_ref(x, small, K, nu, m, gains, wts=w_full, _mid=h, **kw1)
        shift = 0
        out = None
        for p in range(1, tb_passes):
            shift = (shift + h) % T
            if p + 1 < tb_passes:
                _, mid = viterbi_ub_cuda_ref(x, small, K, nu, m, gains, wts=w_full, init_state=mid, _tail=True, _mid=h,
                                             _rot=shift, **kw)
            else:
                out = viterbi_ub_cuda_ref(x, small, K, nu, m, gains, wts=w_full, init_state=mid,
                                          return_code=return_code, _tail=True, _rot=shift, **kw)
        return out
    N, ld = x.shape
    T = _steps or ld
    S, U = 1 << nu, 1 << (K - 1)
    dev = x.device
    x = x.float().contiguous()
    w = torch.ones_like(x) if wts is None else (wts.view(1, ld).expand(N, ld) if wts.dim() == 1 else wts).float().contiguous()
    g = (gains if gains is not None else torch.ones(1, device=dev)).float().contiguous()
    tab = small.float().contiguous()
    rec = torch.empty_like(x)
    G_run = n_cand if 0 < n_cand < g.numel() else g.numel()
    bp = torch.empty((N, T, G_run, S // 32), dtype=torch.int32, device=dev)
    gsel = torch.empty((N, max(T // sub, 1), S), dtype=torch.uint8, device=dev)
    tab_hi = small_hi.float().contiguous() if small_hi is not None else tab
    g_hi = gains_hi.float().contiguous() if gains_hi is not None else g
    init = init_state.to(torch.int32).contiguous() if init_state is not None else None
    end = torch.empty(N, dtype=torch.int32, device=dev) if return_end_state else None
    Gfull, cand = g.numel(), None
    best = torch.empty(N, dtype=torch.int32, device=dev)
    code = torch.empty((N, ld), dtype=torch.int32, device=dev) if return_code else None
    mid = torch.empty(N, dtype=torch.int32, device=dev) if _mid else None
    if int(pair_parity) >= 2:
        pbits = torch.empty((N, T // 4, G_run, 9, S // 32), dtype=torch.int32, device=dev)
    else:
        pbits = torch.empty((N, T // 2, G_run, S // 32), dtype=torch.int32, device=dev) if pair_parity else None
    nl = 4 << len(m_extra)
    if 0 < n_cand < Gfull:
        cand = torch.empty((N, T // sub, n_cand), dtype=torch.uint8, device=dev)
    rc = lib().tcq_viterbi(_p(x), _p(w), _p(tab), _p(g), _p(rec), _p(bp), _p(gsel), _p(init), _p(end), _p(tab_hi),
                           _p(g_hi), _p(cand), _p(best), _p(code), _p(mid), _mid, int(_tail), N, T, S, U,
                           n_cand if cand is not None else Gfull, Gfull, m, sub, tab_hi.numel() // nl,
                           mix if small_hi is not None else 0, *(list(m_extra) + [0, 0, 0])[:3], nl, ld, _rot,
                           _p(pbits), int(pair_parity), torch.cuda.current_stream().cuda_stream)
    if rc != 0:
        raise RuntimeError(f"tcq_viterbi: CUDA error code {rc}")
    if _mid:
        return rec, mid
    if return_code:
        return rec, code >> 16, code & 0xffff
    return (rec, end) if return_end_state else rec
