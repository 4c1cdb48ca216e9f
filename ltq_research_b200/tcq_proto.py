"""Viterbi quantizer API of the reference (lumen-inference/ltq-research, src/tcq_proto.py), on the B200 kernels.

``viterbi_ub_cuda`` keeps the reference's signature, argument meaning, return values and error behaviour
(src/tcq_proto.py:567-657), so ``liqk_v2``, ``ltq_format``, ``ple_quant``, ``universal_bench`` and the other callers
work unchanged.  The tail-biting schedule (src/tcq_proto.py:584-609) runs inside the library in one call
(``ltq_viterbi_tb``); non-tail-biting calls go through the reference-compatible C entry ``tcq_viterbi`` with the same
scratch buffers the reference allocates.  Everything runs on CUDA; there is no CPU path.
"""
from __future__ import annotations

import ctypes

import torch

from . import _lib
from ._lib import ptr

__all__ = ["make_gains", "viterbi_ub_cuda", "viterbi_ub", "lut_subs_quant_cuda", "install"]


def make_gains(h: int, step: float, device="cuda") -> torch.Tensor:
    """Gain table 2^((g - (2^h - 1) / 2) * step), g < 2^h (src/tcq_proto.py:247-249).  The values depend on the device
    that evaluates the power, so the format stores them explicitly; this evaluates it the same way the reference does."""
    G = 1 << h
    return 2.0 ** ((torch.arange(G, dtype=torch.float32, device=device) - (G - 1) / 2) * step)


def _raise(rc: int):
    if rc != 0:
        raise RuntimeError(f"tcq_viterbi: CUDA error code {rc}")


@torch.no_grad()
def viterbi_ub_cuda(x: torch.Tensor, small: torch.Tensor, K: int, nu: int, m: int, gains: torch.Tensor | None = None,
                    sub: int = 16, wts: torch.Tensor | None = None, init_state: torch.Tensor | None = None,
                    return_end_state: bool = False, small_hi: torch.Tensor | None = None,
                    gains_hi: torch.Tensor | None = None, mix: int = 0, n_cand: int = 0, return_code: bool = False,
                    tail_biting: bool = False, tb_passes: int = 2, tb_cand1: int = 0, tb_window: int = 0,
                    m_extra: tuple = (), pair_parity: bool = False, _mid: int = 0, _tail: bool = False,
                    _steps: int = 0, _rot: int = 0):
    """TCQ Viterbi over tiles x [N, T] (fp32, CUDA); see src/tcq_proto.py:574-583 for the arguments.

    Returns rec [N, T]; (rec, end_state) with return_end_state; (rec, gain index [N, T], level index label*U+u [N, T])
    with return_code; (rec, middle state [N]) with _mid.  Tail-biting: the tile's path starts and ends in the same state.
    """
    dev = _lib.require_cuda(x)
    L = _lib.lib()
    if tail_biting:
        N, T = x.shape
        x = x.float().contiguous()
        if wts is None:
            w, w_stride = torch.ones(T, dtype=torch.float32, device=dev), 0
        elif wts.dim() == 1 or (wts.dim() == 2 and wts.shape[0] == 1):
            w, w_stride = wts.reshape(T).float().contiguous(), 0
        else:
            w, w_stride = wts.float().contiguous(), T
        g = (gains if gains is not None else torch.ones(1, device=dev)).float().contiguous()
        tab = small.float().contiguous()
        tab_hi = small_hi.float().contiguous() if small_hi is not None else None
        g_hi = gains_hi.float().contiguous() if gains_hi is not None else None
        nl = 4 << len(m_extra)
        U_hi = tab_hi.numel() // nl if tab_hi is not None else (1 << (K - 1))
        me = torch.tensor(list(m_extra) + [0], dtype=torch.int32)  # host array
        rec = torch.empty_like(x)
        code = torch.empty((N, T), dtype=torch.int32, device=dev) if return_code else None
        Gfull = g.numel()
        wsb = L.ltq_viterbi_tb_workspace_bytes(N, T, Gfull, n_cand, sub, int(pair_parity), tb_window, tb_cand1)
        ws = torch.empty(max(int(wsb), 256), dtype=torch.uint8, device=dev)
        rc = L.ltq_viterbi_tb(ptr(x), ptr(w), w_stride, ptr(tab), ptr(g), ptr(tab_hi), ptr(g_hi), ptr(rec), ptr(code),
                              N, T, nu, K, m, ctypes.cast(me.data_ptr(), ctypes.c_void_p), len(m_extra), Gfull,
                              n_cand, sub, U_hi, mix if small_hi is not None else 0, int(pair_parity), tb_passes,
                              tb_cand1, tb_window, ptr(ws), ws.numel(), _lib.stream_ptr(dev))
        _raise(rc)
        if return_code:
            return rec, code >> 16, code & 0xFFFF
        return rec
    N, ld = x.shape
    T = _steps or ld
    S, U = 1 << nu, 1 << (K - 1)
    x = x.float().contiguous()
    if wts is None:
        w = torch.ones_like(x)
    else:
        w = (wts.view(1, ld).expand(N, ld) if wts.dim() == 1 else wts).float().contiguous()
    g = (gains if gains is not None else torch.ones(1, device=dev)).float().contiguous()
    tab = small.float().contiguous()
    rec = torch.empty_like(x)
    G_run = n_cand if 0 < n_cand < g.numel() else g.numel()
    # scratch of the reference wrapper's shapes (src/tcq_proto.py:623-637); the library keeps its survivors there
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
    me = (list(m_extra) + [0, 0, 0])[:3]
    rc = L.tcq_viterbi(ptr(x), ptr(w), ptr(tab), ptr(g), ptr(rec), ptr(bp), ptr(gsel), ptr(init), ptr(end),
                       ptr(tab_hi), ptr(g_hi), ptr(cand), ptr(best), ptr(code), ptr(mid), _mid, int(_tail), N, T, S, U,
                       n_cand if cand is not None else Gfull, Gfull, m, sub, tab_hi.numel() // nl,
                       mix if small_hi is not None else 0, me[0], me[1], me[2], nl, ld, _rot, ptr(pbits),
                       int(pair_parity), _lib.stream_ptr(dev))
    _raise(rc)
    if _mid:
        return rec, mid
    if return_code:
        return rec, code >> 16, code & 0xFFFF
    return (rec, end) if return_end_state else rec


@torch.no_grad()
def viterbi_ub(x: torch.Tensor, small: torch.Tensor, K: int, nu: int, m: int, gains: torch.Tensor | None = None,
               sub: int = 16, wts: torch.Tensor | None = None):
    """Plain Ungerboeck Viterbi with the return values of the reference's torch `viterbi_ub` (src/tcq_proto.py:363-419):
    (rec, labels [N, T], u [N, T], sub-block gain index [N, T // sub]), computed by the CUDA kernel.  The reference's
    torch version rounds g * tab before the subtraction; the kernel fuses it (as the reference CUDA kernel does)."""
    rec, gi, idx = viterbi_ub_cuda(x, small, K, nu, m, gains, sub=sub, wts=wts, return_code=True)
    U = 1 << (K - 1)
    return rec, (idx // U).long(), (idx % U).long(), gi[:, ::sub].long()


@torch.no_grad()
def lut_subs_quant_cuda(x_subs: torch.Tensor, dh: torch.Tensor, lut_val: torch.Tensor, inv_step: float, half_b: float):
    """DP-profile sub-block quantization through the 1-D table (src/tcq_proto.py:538-547, kernel
    src/cuda/tcq_viterbi.cu:768-811): x_subs, dh [S, 16] -> [S, 16], each sub-block's 16 values taken from the table
    column with the smallest weighted error (C-ABI `lut_subs_quant`, one warp per sub-block)."""
    assert lut_val.shape[1] == 64
    dev = _lib.require_cuda(x_subs, dh, lut_val)
    x = x_subs.float().contiguous()
    d = dh.float().reshape(x.shape).contiguous()
    lut = lut_val.float().contiguous()
    out = torch.empty_like(x)
    rc = _lib.lib().lut_subs_quant(ptr(x), ptr(d), ptr(lut), ptr(out), x.shape[0], inv_step, half_b, lut.shape[0],
                                   _lib.stream_ptr(dev))
    if rc != 0:
        raise RuntimeError(f"lut_subs_quant: CUDA error code {rc}")
    return out


def install(module=None):
    """Point a reference `src.tcq_proto` module (or any module binding `viterbi_ub_cuda`) at this implementation, so the
    reference's callers run on the B200 kernels unchanged (they bind `viterbi_ub_cuda` at call time or at import)."""
    import sys
    targets = [module] if module is not None else [m for n, m in list(sys.modules.items())
                                                   if m is not None and n.endswith("tcq_proto")]
    for mod in targets:
        mod.viterbi_ub_cuda = viterbi_ub_cuda
        mod.lut_subs_quant_cuda = lut_subs_quant_cuda
    return targets
