"""Matrix quantizer of the LTQ TCQ formats on B200: the TCQ path of the reference's ``quantize_matrix_liqk_v2``.

Mirrors lumen-inference/ltq-research src/liqk_v2.py (same names, arguments, return values and ``PACK`` side channel):
  * ``compute_optimal_suh`` (:409-441) — column scale suh and the FWHT-256 rotations of W and H (ltq_fwht256 kernel);
  * ``_quantize_rows_tcq_ldlq`` (:872-1021, row-scale branch :956-980) — scale fit (ltq_scale_fit kernel), then per
    256-column block 16 sub-blocks of tail-biting Viterbi with the intra-block error feedback (one fused ltq_ldlq_block
    launch per block) and the inter-block feedback GEMM;
  * ``quantize_matrix_liqk_v2`` (:1029-1198) — damping, Cholesky factorisation, row groups, c_row and suh refits, PACK
    emission.
Two modes for the linear algebra (GEMM_MODES): "fp32" runs the reference's torch operations (cuBLAS fp32, cuSOLVER's
Cholesky and solves) bit for bit; "bf16x6", the batch driver's default, runs the products as fp32-accurate six-product
bf16 GEMMs on the tensor cores and the factorisations through hessian.cholesky_lower / tri_inv_lower.
The TCQ formats of TCQ_CONFIG are handled: the tail-biting row-scale (.ltq) formats on the fused path above, the
earlier non-tail-biting ones (block-scale TCQ2 / 3 / 4, the carry R formats, half-integer TCQ25R / TCQ35R; no .ltq
encoding) through the per-sub-block Viterbi with the reference's torch updates; the reference's other quantizers
(.liqk v2 banks, E8) are out of this path.  Everything runs on CUDA; there is no CPU path.
"""
from __future__ import annotations

import ctypes
import os
from typing import Dict, List, Optional, Tuple

import torch

from . import _lib, tcgemm
from ._lib import ptr
from .hessian import chol_solve, cholesky_lower
from .formats import LIQK_V2_SPECS, QK_K, SUBBLOCK_SIZE, TCQ_CONFIG  # noqa: F401
from .tcq_proto import make_gains

NUM_SUBBLOCKS = QK_K // SUBBLOCK_SIZE
N_LUT_BUCKETS = 8192  # buckets of the DP profile's 1-D table (src/liqk_v2.py:71)
# Packing mode for .ltq: if not None, the quantizer stores each matrix's tile codes, d_row, e and suh in
# PACK["matrix"] (src/liqk_v2.py:72-74)
PACK: Optional[dict] = None


def _check(rc: int, what: str):
    if rc != 0:
        raise RuntimeError(f"{what}: CUDA error code {rc}")


def _stream(dev) -> int:
    return _lib.stream_ptr(dev)


_SIGNS: Dict[tuple, torch.Tensor] = {}


# ------------------------------------------------------------------------------------------------
# fp32 products of the LDLQ update and the refits.  "fp32": torch's fp32 matmul (the reference's operation, bit for
# bit).  "bf16x6": each fp32 operand is split as x = x0 + x1 + x2 in bf16 (x0 = bf16(x), x1 = bf16(x - x0), ...,
# 24 significand bits together) and the six leading products a_i b_j (i + j <= 2) run as ONE bf16 tensor-core GEMM over
# the K-concatenated parts with fp32 accumulation; the dropped terms are ~2^-24 relative, i.e. fp32-level accuracy,
# with the arithmetic on the tensor pipes instead of the FP32 SIMT pipes the Viterbi kernels use.
# ------------------------------------------------------------------------------------------------
GEMM_MODES = ("fp32", "bf16x6")


def _split3(x: torch.Tensor) -> tuple:
    x0 = x.to(torch.bfloat16)
    r = x - x0.float()
    x1 = r.to(torch.bfloat16)
    x2 = (r - x1.float()).to(torch.bfloat16)
    return x0, x1, x2


def _acat(p: tuple) -> torch.Tensor:
    """Left operand [M, 6K]: parts in the order pairing with _bcat's rows (a0 b0, a0 b1, a1 b0, a0 b2, a1 b1, a2 b0)."""
    return torch.cat([p[0], p[0], p[1], p[0], p[1], p[2]], dim=1)


def _bcat(p: tuple) -> torch.Tensor:
    """Right operand [6K, N]."""
    return torch.cat([p[0], p[1], p[0], p[2], p[1], p[0]], dim=0)


def _mm6(acat: torch.Tensor, bcat: torch.Tensor) -> torch.Tensor:
    return torch.mm(acat, bcat, out_dtype=torch.float32)


def _op6(x: torch.Tensor, order: int, side: int) -> Optional[torch.Tensor]:
    """The six-slot bf16 operand of an fp32 matrix with unit column stride in one kernel (ltq_bf16x6_split): order 0
    the left slots (as _acat), 1 the right slots (as _bcat); side 0 slots along the columns, 1 along the rows.  None
    when the layout does not meet the kernel's alignment."""
    rows, cols = x.shape
    if (x.dtype != torch.float32 or not x.is_cuda or x.stride(1) != 1 or cols % 4 or x.stride(0) % 4
            or x.data_ptr() % 16):
        return None
    out = torch.empty((rows, 6 * cols) if side == 0 else (6 * rows, cols), dtype=torch.bfloat16, device=x.device)
    _check(_lib.lib().ltq_bf16x6_split(ptr(x), x.stride(0), rows, cols, order, side, ptr(out), out.stride(0),
                                       _stream(x.device)), "ltq_bf16x6_split")
    return out


def _left6(a: torch.Tensor) -> torch.Tensor:
    """_acat(_split3(a)), bit for bit, with one kernel where the layout allows (a or a.T with unit column stride)."""
    o = _op6(a, 0, 0)
    if o is None and a.stride(0) == 1:
        o = _op6(a.T, 0, 1)
        o = o.T if o is not None else None
    return o if o is not None else _acat(_split3(a))


def _right6(b: torch.Tensor) -> torch.Tensor:
    """_bcat(_split3(b)), bit for bit, with one kernel where the layout allows."""
    o = _op6(b, 1, 1)
    if o is None and b.stride(0) == 1:
        o = _op6(b.T, 1, 0)
        o = o.T if o is not None else None
    return o if o is not None else _bcat(_split3(b))


def _mm(a: torch.Tensor, b: torch.Tensor, gemm: str) -> torch.Tensor:
    """a @ b for fp32 [M, K] x [K, N] in the given mode: torch's fp32 matmul, or the six-product tensor-core GEMM."""
    if gemm == "fp32":
        return a @ b
    if gemm != "bf16x6":
        raise ValueError(f"gemm mode {gemm!r}: expected one of {GEMM_MODES}")
    if b.shape[1] % 16 == 0:
        return tcgemm.mm(a, b)
    return _mm6(_left6(a), _right6(b))


def make_rademacher_signs(dim: int, seed: int, device) -> torch.Tensor:
    """Deterministic +-1 signs from a CPU generator (src/iqk_format.py:173-179).  Device copies are cached, so a
    quantization in flight on a side stream never waits on a pageable host-to-device copy."""
    dev = torch.device(device)
    key = (dim, seed, str(dev))
    t = _SIGNS.get(key)
    if t is None:
        gen = torch.Generator(device="cpu")
        gen.manual_seed(seed)
        bits = torch.randint(0, 2, (dim,), generator=gen, dtype=torch.int64)
        t = (bits * 2 - 1).to(dtype=torch.float32, device=dev)
        if dev.type == "cuda":
            torch.cuda.current_stream(dev).synchronize()
        _SIGNS[key] = t
    return t


def fwht_rows_scaled(x: torch.Tensor, scale: Optional[torch.Tensor] = None, mode: int = 0,
                     out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """FWHT-256 of every 256-block of every row of x [R, C] (fp32 or bf16), after dividing (mode 1) or multiplying
    (mode 2) column c by scale[c]: the normalized transform of src/iqk_format.py:153-170, bit for bit."""
    dev = _lib.require_cuda(x)
    R, C = x.shape
    if x.stride(1) != 1 or x.dtype not in (torch.float32, torch.bfloat16):
        x = x.float().contiguous()
    out = torch.empty((R, C), dtype=torch.float32, device=dev) if out is None else out
    s = scale.float().contiguous() if scale is not None else None
    _check(_lib.lib().ltq_fwht256(ptr(x), int(x.dtype == torch.bfloat16), x.stride(0), ptr(out), out.stride(0), ptr(s),
                                  mode, R, C, _stream(dev)), "ltq_fwht256")
    return out


def fwht_inplace(x: torch.Tensor, block_size: int = 256) -> torch.Tensor:
    """src/iqk_format.py:153-170 for block_size 256 (any leading shape); returns the transformed tensor."""
    assert block_size == QK_K
    shp = x.shape
    return fwht_rows_scaled(x.reshape(-1, shp[-1])).view(shp)


def _fwht_rows(X: torch.Tensor) -> torch.Tensor:
    """Block FWHT-256 over rows (along the first dimension), src/liqk_v2.py:1024-1026."""
    return fwht_rows_scaled(X.T.contiguous()).T.contiguous()


# Trained register banks of the .liqk v2 formats, per (format, device) (src/liqk_v2.py:234, :379-406).  The stored bank
# file of the reference (data/liqk_v2_banks.safetensors) and its trainer belong to the .liqk v2 quantizer, which this
# build does not include: banks are registered here (register_warp_register_bank) and then serve the DP profile.
_WARP_BANK_CACHE: Dict[Tuple[str, str], Dict[str, torch.Tensor]] = {}


def register_warp_register_bank(spec_name: str, grids_all: torch.Tensor, max_grid: float, device=None,
                                ls_all: Optional[torch.Tensor] = None, cb_all: Optional[torch.Tensor] = None) -> dict:
    """Register the bank of `spec_name` (grids_all [C_all, levels] of candidate grids, max_grid their range) on
    `device` and build its 1-D table as the reference does (src/liqk_v2.py:394-396): bucket centres
    z = linspace(-max_g, max_g, N_LUT_BUCKETS), lut_val[b, c] = the point of grid c nearest to z_b (first on ties)."""
    dev = torch.device(device) if device is not None else grids_all.device
    grids_all = grids_all.to(dev, torch.float32)
    z = torch.linspace(-max_grid, max_grid, N_LUT_BUCKETS, device=dev, dtype=torch.float32)
    q_idx = (z[:, None, None] - grids_all[None, :, :]).abs().argmin(dim=-1)
    lut_val = torch.gather(grids_all.unsqueeze(0).expand(N_LUT_BUCKETS, -1, -1), 2,
                           q_idx.unsqueeze(-1)).squeeze(-1).contiguous()
    bank = {"grids_all": grids_all, "ls_all": ls_all, "cb_all": cb_all, "lut_val": lut_val, "max_grid": max_grid}
    _WARP_BANK_CACHE[(spec_name, str(dev))] = bank
    return bank


def get_warp_register_bank(spec_name: str, device) -> Dict[str, torch.Tensor]:
    """The registered bank of `spec_name` on `device` (src/liqk_v2.py:379-406); raises KeyError when none is
    registered (the reference would load data/liqk_v2_banks.safetensors or train one)."""
    key = (spec_name, str(torch.device(device)))
    if key not in _WARP_BANK_CACHE:
        raise KeyError(f"{spec_name}: no register bank on {device}; register one with register_warp_register_bank "
                       "(the trained bank file and trainer of the .liqk v2 formats are not part of this build)")
    return _WARP_BANK_CACHE[key]


LUT_PICK_CHUNK = 32768  # sub-blocks per torch evaluation of the table pick (bounds the [chunk, 16, C] temporaries)


def _lut_pick_torch(xs: torch.Tensor, dh: torch.Tensor, lut_val: torch.Tensor, inv_step: float,
                    half_b: float) -> torch.Tensor:
    """Table pick of one batch of sub-blocks in torch arithmetic: every weight's bucket round(x * inv_step + half_b)
    (product rounded before the add, ties to even, clamped to the table), the weighted squared error of every column
    summed over the sub-block, the first column of least error, and the sub-block's values from that column."""
    nb, C = lut_val.shape
    bucket = torch.clamp((xs * inv_step + half_b).round().long(), 0, nb - 1)          # [s, 16]
    cand = lut_val[bucket]                                                             # [s, 16, C]
    score = ((xs.unsqueeze(-1) - cand).square() * dh.unsqueeze(-1)).sum(dim=1)        # [s, C]
    col = score.argmin(dim=-1)                                                         # [s]
    return cand.gather(2, col.view(-1, 1, 1).expand(-1, xs.shape[1], 1)).squeeze(2)


@torch.no_grad()
def quantize_subs_lut_chunked(x_subs: torch.Tensor, dhs: torch.Tensor, lut_val: torch.Tensor, inv_step: float,
                              half_b: float) -> torch.Tensor:
    """The DP profile's table pick for tables of any width (src/liqk_v2.py:444-466, the reference's path for tables
    other than 64 columns): x_subs [S, 16], dhs [S, 16] or [S, 16, 1] -> [S, 16], evaluated LUT_PICK_CHUNK sub-blocks
    at a time (the reference's batch size, so each batch's reductions see the same shapes)."""
    S = x_subs.shape[0]
    dh = dhs.reshape(S, SUBBLOCK_SIZE)
    parts = [_lut_pick_torch(x_subs[i: i + LUT_PICK_CHUNK], dh[i: i + LUT_PICK_CHUNK], lut_val, inv_step, half_b)
             for i in range(0, S, LUT_PICK_CHUNK)]
    if not parts:
        return torch.empty((0, SUBBLOCK_SIZE), dtype=torch.float32, device=x_subs.device)
    return torch.cat(parts, dim=0)


def _fp16_scale(v: torch.Tensor) -> torch.Tensor:
    """A block scale as stored: rounded to fp16, back in fp32, at least 1e-8."""
    return v.to(torch.float16).float().clamp(min=1e-8)


@torch.no_grad()
def quantize_liqk_v2_diag_rot(W_rot: torch.Tensor, diag_h: torch.Tensor, spec_name: str) -> torch.Tensor:
    """The DP profile's diagonal quantization in the rotated basis (src/liqk_v2.py:469-506), on the device.

    Per 256-column block b of row m: scale d = fp16(max |w| / max_grid); then LIQK_PROFILE_ITERS rounds (default 2)
    of (a) the table pick of every 16-weight sub-block of w / d with the Hessian diagonal as weights — the
    lut_subs_quant kernel for 64-column tables (unless LIQK_PROFILE_CUDA=0), the torch pick otherwise — and (b) the
    weighted least-squares refit d = fp16(sum(h w q) / max(sum(h q q), 1e-12)).  Returns d * q [M, K]."""
    _lib.require_cuda(W_rot, diag_h)
    M, K = W_rot.shape
    nblk = M * (K // QK_K)
    bank = get_warp_register_bank(spec_name, W_rot.device)
    table, max_g = bank["lut_val"], bank["max_grid"]
    inv_step = (N_LUT_BUCKETS - 1) / (2.0 * max_g)
    half_b = (N_LUT_BUCKETS - 1) * 0.5
    use_kernel = table.shape[1] == 64 and os.environ.get("LIQK_PROFILE_CUDA", "1") == "1"
    rounds = int(os.environ.get("LIQK_PROFILE_ITERS", "2"))

    w = W_rot.float().reshape(nblk, QK_K).contiguous()
    # the Hessian diagonal repeated for every row: [nblk, 256] (materialised: the pick reads it per sub-block)
    h = diag_h.float().view(1, K // QK_K, QK_K).expand(M, -1, -1).reshape(nblk, QK_K).contiguous()
    d = _fp16_scale(w.abs().amax(dim=1) / max_g)
    q = None
    for _ in range(rounds):
        x = (w / d[:, None]).reshape(-1, SUBBLOCK_SIZE)
        hs = h.view(-1, SUBBLOCK_SIZE)
        if use_kernel:
            from .tcq_proto import lut_subs_quant_cuda
            q = lut_subs_quant_cuda(x, hs, table, inv_step, half_b)
        else:
            q = quantize_subs_lut_chunked(x, hs, table, inv_step, half_b)
        q = q.view(nblk, QK_K)
        # the reference's products in its order: (h w) q and (h q) q
        d = _fp16_scale((h * w * q).sum(dim=1) / (h * q * q).sum(dim=1).clamp(min=1e-12))
    return (d[:, None] * q).view(M, K)


@torch.no_grad()
def compute_optimal_suh(W: torch.Tensor, H: torch.Tensor, seed: int = 1337,
                        row_weights: Optional[torch.Tensor] = None,
                        row_reduce=None) -> Tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """src/liqk_v2.py:409-441: suh = fp16(sign * clamp(col_rms^0.5 * h_std^-0.25, 0.25, 4));
    W_rot = FWHT(W / suh), H_rot = FWHT(FWHT(H * suh)^T * suh)^T.
    row_reduce: W holds some rows of the matrix and row_reduce(t) sums t in place over the holders of all of them
    (see _quantize_matrix_steps); the column RMS is then taken over every row."""
    device = W.device
    M, K = W.shape
    signs = make_rademacher_signs(K, seed=seed, device=device)
    Wf = W.float()
    if row_reduce is not None:
        if row_weights is not None:
            raise ValueError("row-sharded quantization takes no row weights")
        acc = torch.cat([Wf.square().sum(dim=0), torch.full((1,), float(M), device=device)])
        row_reduce(acc)
        col_rms = (acc[:K] / acc[K]).sqrt().clamp(min=1e-6)
    elif row_weights is not None:
        rw = row_weights.float().clamp(min=float(row_weights.mean().item()) * 0.1)
        rw = (rw / rw.mean().clamp(min=1e-12)).clamp(0.25, 4.0)
        col_rms = ((Wf.square() * rw.unsqueeze(1)).mean(dim=0)).sqrt().clamp(min=1e-6)
    else:
        col_rms = Wf.square().mean(dim=0).sqrt().clamp(min=1e-6)
    col_rms = col_rms / col_rms.mean().clamp(min=1e-6)
    h_std = torch.diagonal(H.float()).clamp(min=1e-8).sqrt()
    h_std = h_std / h_std.mean().clamp(min=1e-6)
    scale = ((col_rms ** 0.5) * (h_std ** -0.25)).clamp(0.25, 4.0)
    suh = (signs * scale).to(torch.float16).to(torch.float32)
    W_rot = fwht_rows_scaled(W if W.dtype in (torch.float32, torch.bfloat16) else Wf, suh, mode=1)
    H_tmp = fwht_rows_scaled(H.float(), suh, mode=2)
    H_rot = fwht_rows_scaled(H_tmp.T.contiguous(), suh, mode=2).T
    return W_rot, H_rot, suh


_TABLES: Dict[tuple, tuple] = {}


def _format_tables(spec: str, device) -> tuple:
    """(lut, gains, m_extra host array) of a format on a device, cached per (format, device, gain function); the
    first use synchronises once so that later uses never wait on a host-to-device copy."""
    dev = torch.device(device)
    key = (spec, str(dev), make_gains)
    t = _TABLES.get(key)
    if t is None:
        cfg = TCQ_CONFIG[spec]
        lut = torch.tensor(cfg["lut"], dtype=torch.float32, device=dev)
        gains = make_gains(cfg["h"], cfg["step"], dev).float().contiguous()
        me = torch.tensor(list(cfg.get("m_extra", ())) + [0], dtype=torch.int32)
        if dev.type == "cuda":
            torch.cuda.current_stream(dev).synchronize()
        t = (lut, gains, me)
        _TABLES[key] = t
    return t


class _FormatArgs:
    """Viterbi parameters of a format: K, sub-block length, parity mode, label masks, gain candidates, TB window."""

    def __init__(self, spec: str, device):
        cfg = TCQ_CONFIG[spec]
        self.cfg = cfg
        self.dev = device
        self.lut, self.gains, self.me = _format_tables(spec, device)
        self.K = cfg["K"]
        self.sub = cfg.get("sub", SUBBLOCK_SIZE)
        self.pp = int(cfg.get("pp", 0))
        self.m_extra = tuple(cfg.get("m_extra", ()))
        self.n_cand = int(os.environ.get("TCQ_NCAND", cfg.get("n_cand", 0) or 0))
        self.tb_window = int(os.environ.get("TCQ_TB_WIN", "32"))

    def me_ptr(self):
        return ctypes.cast(self.me.data_ptr(), ctypes.c_void_p)


class _TcqRunner(_FormatArgs):
    """Sub-block Viterbi calls (ltq_viterbi_tb) over the M/16 tiles of one sub-block: buffers and workspace."""

    def __init__(self, spec: str, M: int, device):
        super().__init__(spec, device)
        self.nt = M // 16
        self.x = torch.empty((self.nt, 256), dtype=torch.float32, device=device)
        self.rec = torch.empty_like(self.x)
        self.code = torch.empty((self.nt, 256), dtype=torch.int32, device=device)
        wsb = _lib.lib().ltq_viterbi_tb_workspace_bytes(self.nt, 256, self.gains.numel(), self.n_cand, self.sub,
                                                        self.pp, self.tb_window, 0)
        self.ws = torch.empty(max(int(wsb), 256), dtype=torch.uint8, device=device)

    def run(self, dw256: torch.Tensor):
        """Tail-biting Viterbi of self.x (tiles of the current sub-block) with per-position weights dw256 [256]."""
        c = self.cfg
        _check(_lib.lib().ltq_viterbi_tb(
            ptr(self.x), ptr(dw256), 0, ptr(self.lut), ptr(self.gains), None, None, ptr(self.rec), ptr(self.code),
            self.nt, 256, c["nu"], self.K, c["m"], self.me_ptr(), len(self.m_extra), self.gains.numel(), self.n_cand,
            self.sub, 1 << (self.K - 1), 0, self.pp, 2, 0, self.tb_window, ptr(self.ws), self.ws.numel(),
            _stream(self.dev)), "tcq_viterbi")


# When a list, every fused block launch appends (start event, end event, add-compare-selects, weights), the events
# recorded on the launch's stream:
# the live roofline of the block kernel in bench.py.
BLOCK_EVENTS: Optional[list] = None


class _BlockRunner(_FormatArgs):
    """Fused block kernel (ltq_ldlq_block) over the M rows of one row group: workspace."""

    def __init__(self, spec: str, M: int, device):
        super().__init__(spec, device)
        self.M = M
        wsb = _lib.lib().ltq_ldlq_block_workspace_bytes(M, self.gains.numel(), self.n_cand, self.sub, self.pp,
                                                        self.tb_window)
        self.ws = torch.empty(max(int(wsb), 256), dtype=torch.uint8, device=device)

    def run(self, W_work, c0: int, d_rb_all, ibl: int, diag_w, Uc, U_blk_inv, G, idx, gi):
        """Block [c0, c0 + 256): G / idx / gi of the block's columns (W_work is read, not written)."""
        K = W_work.shape[1]
        ev = BLOCK_EVENTS
        if ev is not None:
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
        _check(_lib.lib().ltq_ldlq_block(
            ptr(W_work) + 4 * c0, W_work.stride(0), ptr(d_rb_all) + 4 * ibl, d_rb_all.stride(0), ptr(diag_w) + 4 * c0,
            ptr(Uc) + 4 * (c0 * Uc.stride(0) + c0), Uc.stride(0), ptr(U_blk_inv), U_blk_inv.stride(0),
            ptr(G) + 4 * c0, G.stride(0), ptr(idx) + 2 * c0, ptr(gi) + c0, K, self.M, ptr(self.lut), ptr(self.gains),
            self.K, self.cfg["m"], self.me_ptr(), len(self.m_extra), self.gains.numel(), self.n_cand, self.sub,
            self.pp, self.tb_window, ptr(self.ws), self.ws.numel(), _stream(self.dev)), "ltq_ldlq_block")
        if ev is not None:
            e1.record()
            ev.append((e0, e1, self.acs_per_block(), self.M * 256))

    def acs_per_block(self) -> int:
        """Add-compare-selects of one block launch: M x 256 weights x passes (1 + 2 W / 256 for the windowed first
        pass) x 1024 states x gain slots x parity classes."""
        g = self.gains.numel()
        if 0 < self.n_cand < g:
            g = self.n_cand
        passes = 1.0 + (2.0 * self.tb_window / 256.0 if self.tb_window else 1.0)
        return int(self.M * 256 * passes * 1024 * g * (2 if self.pp else 1))


def _drive(gen):
    """Run a step generator to its end and return its value."""
    while True:
        try:
            next(gen)
        except StopIteration as e:
            return e.value


@torch.no_grad()
def _rows_ldlq(W_rot: torch.Tensor, U: torch.Tensor, U_blks_inv: torch.Tensor, diag_w: torch.Tensor, spec_name: str,
               fused: bool = True, gemm: str = "fp32") -> Tuple[torch.Tensor, torch.Tensor, dict]:
    """Block16-LDLQ of one row group (src/liqk_v2.py:872-1021, row-scale branch :956-980) on the current stream,
    without host synchronisation.  Returns (d_full fp16 [M, K/256], W_hat_rot [M, K], group fields).  gemm: the mode of
    the inter-block update products (see GEMM_MODES)."""
    return _drive(_rows_ldlq_steps(W_rot, U, U_blks_inv, diag_w, spec_name, fused, gemm))


_GEMM_ERR: Dict[str, torch.Tensor] = {}


def gemm_error_flag(device) -> torch.Tensor:
    """The device int that the tensor-core GEMM sets when one of its pipeline waits runs out (one per device, shared by
    all streams; cleared by check_gemm_errors)."""
    key = str(torch.device(device))
    t = _GEMM_ERR.get(key)
    if t is None:
        t = torch.zeros(1, dtype=torch.int32, device=device)
        torch.cuda.current_stream(device).synchronize()
        _GEMM_ERR[key] = t
    return t


def check_gemm_errors(device):
    """Raises if a tensor-core GEMM on `device` reported a timed-out pipeline wait since the last check (a host
    synchronisation: call it where the caller synchronises anyway)."""
    t = _GEMM_ERR.get(str(torch.device(device)))
    if t is not None and int(t.item()) != 0:
        t.zero_()
        raise RuntimeError("ltq_gemm_bf16_tn: a pipeline wait ran out; the LDLQ update of this call is not valid")


def _scale_fit_reference(W_rot: torch.Tensor, cfg: dict):
    """The row-scale fit as the reference computes it with torch (src/liqk_v2.py:938-946): block RMS, fp16 geometric
    mean per row, 5-bit exponents; returns (d_row fp32 [M], e int8 [M, K/256], d_rb fp32 [M, K/256])."""
    M, K = W_rot.shape
    rms_rb = W_rot.float().view(M, K // QK_K, QK_K).square().mean(dim=2).sqrt().clamp(min=1e-10) * cfg.get("scale", 1.0)
    d_row = torch.exp(torch.log(rms_rb).mean(dim=1)).to(torch.float16).to(torch.float32).clamp(min=1e-8)
    e_step, e_max = cfg.get("e_step", 0.25), 1 << (cfg.get("e_bits", 5) - 1)
    e_rb = torch.round(torch.log2(rms_rb / d_row.unsqueeze(1)) / e_step).clamp(-e_max, e_max - 1)
    d_rb = d_row.unsqueeze(1) * torch.exp2(e_step * e_rb)
    return d_row, e_rb.to(torch.int8), d_rb.contiguous()


def _legacy_tables(cfg: dict, device) -> tuple:
    """(table, gains, extra Viterbi arguments) of an earlier format (src/liqk_v2.py:885-895): a half-integer format
    runs its "lo" format's table on even tile rows and its "hi" format's table on odd ones, each premultiplied by its
    own scale (its d carries no scale factor)."""
    if "K_hi" not in cfg:
        return (torch.tensor(cfg["lut"], dtype=torch.float32, device=device), make_gains(cfg["h"], cfg["step"], device),
                {})
    lo, hi = TCQ_CONFIG[cfg["lo"]], TCQ_CONFIG[cfg["hi"]]
    tab = torch.tensor(lo["lut"], dtype=torch.float32, device=device) * lo["scale"]
    extra = {"small_hi": torch.tensor(hi["lut"], dtype=torch.float32, device=device) * hi["scale"],
             "gains_hi": make_gains(hi["h"], hi["step"], device), "mix": SUBBLOCK_SIZE}
    return tab, make_gains(lo["h"], lo["step"], device), extra


def _rows_legacy_steps(W_rot, U, U_blks_inv, diag_w, spec_name: str, n_pass: int = 2):
    """The earlier (non-tail-biting) formats through the LDLQ loop of src/liqk_v2.py:948-1021, one Viterbi call per
    16-column sub-block of all rows (tiles of 16 rows x 16 columns, t = 16 r + c), with the reference's torch operations
    for the feedback and block updates (these formats are not on the fast path):
      * R formats (row_scale): d(row, block) from the row-scale fit; the end state of each tile starts the next tile of
        the same rows (carry), across sub-blocks and blocks;
      * TCQ2 / TCQ3 / TCQ4: a scale per (row, block) from the block's rms, refitted over n_pass passes against the
        block's Cholesky-weighted error, the best of (current, refit) kept per row.
    A generator like _rows_ldlq_steps (yields after each block); returns (d_full, W_hat_rot, None): nothing to pack."""
    from .tcq_proto import viterbi_ub_cuda
    cfg = TCQ_CONFIG[spec_name]
    device = W_rot.device
    tab, gains, extra = _legacy_tables(cfg, device)
    M, K = W_rot.shape
    assert M % 16 == 0, "TCQ: number of rows must be divisible by 16"
    nt, nblocks = M // 16, K // QK_K
    n_cand = int(os.environ.get("TCQ_NCAND", cfg.get("n_cand", 0)))
    W_work = W_rot.float().clone()
    W_hat_rot = torch.empty_like(W_work)
    d_full = torch.empty((M, nblocks), dtype=torch.float16, device=device)
    state = [None]  # the tiles' end states, carried to the next sub-block (R formats)

    def tiles_of(xs, dw):  # xs [M, 16] already divided by d, dw [16]: the reconstruction [M, 16]
        t = xs.reshape(nt, 16 * SUBBLOCK_SIZE)
        w = dw.repeat(16)
        if cfg.get("carry"):
            rec, state[0] = viterbi_ub_cuda(t, tab, cfg["K"], cfg["nu"], cfg["m"], gains, sub=SUBBLOCK_SIZE, wts=w,
                                            init_state=state[0], return_end_state=True, n_cand=n_cand, **extra)
        else:
            rec = viterbi_ub_cuda(t, tab, cfg["K"], cfg["nu"], cfg["m"], gains, sub=SUBBLOCK_SIZE, wts=w,
                                  n_cand=n_cand)
        return rec.view(M, SUBBLOCK_SIZE)

    def sweep(w_blk, d, U_blk, U_blk_inv, dw_blk):  # one LDLQ pass over a block's 16 sub-blocks at scale d [M]
        work = w_blk.clone()
        G = torch.empty((M, QK_K), dtype=torch.float32, device=device)
        inv_d = 1.0 / d.unsqueeze(1)
        for ib in range(NUM_SUBBLOCKS):
            s0, s1 = ib * SUBBLOCK_SIZE, (ib + 1) * SUBBLOCK_SIZE
            w_sub = work[:, s0:s1]
            g = tiles_of(w_sub * inv_d, dw_blk[s0:s1])
            G[:, s0:s1] = g
            if s1 < QK_K:
                e = (w_sub - d.unsqueeze(1) * g) @ U_blk_inv[s0:s1, s0:s1]
                work[:, s1:] -= e @ U_blk[s0:s1, s1:]
        return G

    if cfg.get("row_scale"):
        _, _, d_rb_all = _scale_fit_reference(W_work, cfg)
    for ibl in range(nblocks):
        c0, c1 = ibl * QK_K, (ibl + 1) * QK_K
        w_blk = W_work[:, c0:c1].clone()
        U_blk, U_blk_inv, dw_blk = U[c0:c1, c0:c1], U_blks_inv[ibl], diag_w[c0:c1]
        if cfg.get("row_scale"):
            d_best = d_rb_all[:, ibl].clamp(min=1e-8)
            what = d_best.unsqueeze(1) * sweep(w_blk, d_best, U_blk, U_blk_inv, dw_blk)
        else:
            A = w_blk @ U_blk_inv
            d = (w_blk.square().mean(dim=1).sqrt() * cfg.get("scale", 1.0)).to(torch.float16).to(torch.float32)
            d = d.clamp(min=1e-8)
            loss_best = torch.full((M,), float("inf"), device=device)
            d_best, what = d.clone(), torch.zeros((M, QK_K), dtype=torch.float32, device=device)
            for _ in range(n_pass):
                G = sweep(w_blk, d, U_blk, U_blk_inv, dw_blk)
                B = G @ U_blk_inv
                num, den = (A * B).sum(dim=1), (B * B).sum(dim=1).clamp(min=1e-12)
                d_fit = torch.where(den > 0, num / den, d).to(torch.float16).to(torch.float32).clamp(min=1e-8)
                for d_try in (d, d_fit):  # keep the scale with the lower block loss, per row (ties keep the first)
                    loss = (A - d_try.unsqueeze(1) * B).square().sum(dim=1)
                    better = loss < loss_best
                    loss_best = torch.where(better, loss, loss_best)
                    d_best = torch.where(better, d_try, d_best)
                    what = torch.where(better.unsqueeze(1), d_try.unsqueeze(1) * G, what)
                d = d_fit
        W_hat_rot[:, c0:c1] = what
        d_full[:, ibl] = d_best.to(torch.float16)
        if c1 < K:
            W_work[:, c1:] -= ((w_blk - what) @ U_blk_inv) @ U[c0:c1, c1:]
        yield
    return d_full, W_hat_rot, None


def _rows_ldlq_steps(W_rot, U, U_blks_inv, diag_w, spec_name: str, fused: bool = True, gemm: str = "fp32",
                     U_parts: Optional[tuple] = None):
    """_rows_ldlq as a generator that yields after each 256-column block's launches (for interleaved issue).
    U_parts: the bf16 split of U when the caller already has it (bf16x6 mode).  The earlier, non-tail-biting formats
    go through _rows_legacy_steps."""
    cfg = TCQ_CONFIG[spec_name]
    if not cfg.get("tb"):
        return (yield from _rows_legacy_steps(W_rot, U, U_blks_inv, diag_w, spec_name))
    if not cfg.get("row_scale"):
        raise ValueError(f"{spec_name}: the tail-biting TCQ formats are row-scale formats")
    device = W_rot.device
    L = _lib.lib()
    st = _stream(device)
    M, K = W_rot.shape
    assert M % 16 == 0, "TCQ: number of rows must be divisible by 16"
    nblocks = K // QK_K
    W_work = W_rot.float().contiguous().clone()
    W_hat_rot = torch.empty_like(W_work)
    d_full = torch.empty((M, nblocks), dtype=torch.float16, device=device)
    G = torch.empty((M, K), dtype=torch.float32, device=device)
    idx = torch.empty((M, K), dtype=torch.int16, device=device)
    gi = torch.empty((M, K), dtype=torch.uint8, device=device)

    # d(row, block) = d_row * 2^(0.25 e), e 5-bit in [-16, 15]; d_row fp16 = geometric mean of the row's block rms
    e_step, e_bits = cfg.get("e_step", 0.25), cfg.get("e_bits", 5)
    if gemm == "fp32":  # the reference's own expressions (src/liqk_v2.py:938-946): its reduction order, its bits
        d_row, e_rb, d_rb_all = _scale_fit_reference(W_work, cfg)
    else:
        d_row = torch.empty(M, dtype=torch.float32, device=device)
        e_rb = torch.empty((M, nblocks), dtype=torch.int8, device=device)
        d_rb_all = torch.empty((M, nblocks), dtype=torch.float32, device=device)
        _check(L.ltq_scale_fit(ptr(W_work), W_work.stride(0), M, K, float(cfg.get("scale", 1.0)), float(e_step),
                               int(e_bits), None, ptr(d_row), ptr(e_rb), ptr(d_rb_all), st), "ltq_scale_fit")
    group = {"spec": spec_name, "d_row": d_row, "e": e_rb, "idx": idx, "gi": gi, "G": G}

    Uc = U.contiguous()
    if gemm == "bf16x6" and U_parts is None and nblocks > 1 and not fused:
        U_parts = _split3(Uc)

    def inter_block(err_in, c0, c1, U_blk_inv):  # W_work[:, c1:] -= ((w_blk - what) @ U_blk_inv) @ U[c0:c1, c1:]
        if gemm == "fp32":
            err_blk = err_in @ U_blk_inv
            W_work[:, c1:] -= err_blk @ Uc[c0:c1, c1:]
        else:
            err_blk = _mm(err_in, U_blk_inv, gemm)
            W_work[:, c1:] -= _mm6(_acat(_split3(err_blk)), _bcat(tuple(p[c0:c1, c1:] for p in U_parts)))

    if fused and gemm == "bf16x6":
        # per block: the fused block kernel, the inter-block operands (W_hat, d, the split of err @ Uinv) and one
        # tensor-core GEMM W_work[:, c1:] -= acat @ bcat_b
        brun = _BlockRunner(spec_name, M, device)
        dwc = diag_w.float().contiguous()
        # every block's right operand [u0 u1 u2] (K-major), built once per matrix; each block's left operand
        # [e0 e1 e2] of err = (w_blk - what) @ U_blk^-1; the update is the six-product tensor-core GEMM of the two
        bcat = torch.empty(max(int(L.ltq_ldlq_bcat_elems(K)) // 2, 8), dtype=torch.bfloat16, device=device)
        if nblocks > 1:
            _check(L.ltq_ldlq_bcat_t(ptr(Uc), Uc.stride(0), K, ptr(bcat), st), "ltq_ldlq_bcat_t")
        gerr = gemm_error_flag(device)
        acat = torch.empty((M, 3 * QK_K), dtype=torch.bfloat16, device=device)
        U_blks_inv = U_blks_inv.contiguous()  # row-major blocks (a batched triangular solve may return column-major)
        off = 0
        for ibl in range(nblocks):
            c0, c1 = ibl * QK_K, (ibl + 1) * QK_K
            U_blk_inv = U_blks_inv[ibl]
            brun.run(W_work, c0, d_rb_all, ibl, dwc, Uc, U_blk_inv, G, idx, gi)
            last = c1 >= K
            _check(L.ltq_ldlq_inter3(ptr(W_work) + 4 * c0, W_work.stride(0), ptr(d_rb_all) + 4 * ibl, d_rb_all.stride(0),
                                    ptr(G) + 4 * c0, G.stride(0), ptr(U_blk_inv), U_blk_inv.stride(0), M,
                                    ptr(W_hat_rot) + 4 * c0, W_hat_rot.stride(0), ptr(d_full) + 2 * ibl,
                                    d_full.stride(0), None if last else ptr(acat), st), "ltq_ldlq_inter")
            if not last:
                # W_work[:, c1:] -= six-product(acat, bcat_b) on the tensor cores (ltq_gemm_bf16x6_tn, tcgen05)
                nb = K - c1
                _check(L.ltq_gemm_bf16x6_tn(ptr(acat), 3 * QK_K, ptr(bcat) + 2 * off, 3 * QK_K, ptr(W_work) + 4 * c1,
                                            W_work.stride(0), M, nb, QK_K, -1.0, 1.0, ptr(gerr), st),
                       "ltq_gemm_bf16x6_tn")
                off += 3 * QK_K * nb
            yield
        return d_full, W_hat_rot, group

    if fused:
        brun = _BlockRunner(spec_name, M, device)
        dwc = diag_w.float().contiguous()
        for ibl in range(nblocks):
            c0, c1 = ibl * QK_K, (ibl + 1) * QK_K
            U_blk_inv = U_blks_inv[ibl].contiguous()
            brun.run(W_work, c0, d_rb_all, ibl, dwc, Uc, U_blk_inv, G, idx, gi)
            d_rb = d_rb_all[:, ibl].clamp(min=1e-8)
            best_what_row = d_rb.unsqueeze(1) * G[:, c0:c1]
            W_hat_rot[:, c0:c1] = best_what_row
            d_full[:, ibl] = d_rb.to(torch.float16)
            if c1 < K:
                inter_block(W_work[:, c0:c1] - best_what_row, c0, c1, U_blk_inv)
            yield
        return d_full, W_hat_rot, group

    run = _TcqRunner(spec_name, M, device)
    for ibl in range(nblocks):
        c0, c1 = ibl * QK_K, (ibl + 1) * QK_K
        w_blk_start = W_work[:, c0:c1].clone()
        w_sub_work = w_blk_start.clone()
        U_blk_inv = U_blks_inv[ibl].contiguous()
        diag_w_blk = diag_w[c0:c1]
        d_rb = d_rb_all[:, ibl].clamp(min=1e-8).contiguous()
        inv_d = (1.0 / d_rb).contiguous()
        dw_all = diag_w_blk.float().view(NUM_SUBBLOCKS, SUBBLOCK_SIZE).repeat(1, 16).contiguous()  # [16, 256]
        for ib in range(NUM_SUBBLOCKS):
            s0 = ib * SUBBLOCK_SIZE
            _check(L.ltq_ldlq_gather(ptr(w_sub_work) + 4 * s0, w_sub_work.stride(0), ptr(inv_d), M, ptr(run.x), st),
                   "ltq_ldlq_gather")
            run.run(dw_all[ib])
            _check(L.ltq_ldlq_feedback(ptr(w_sub_work), w_sub_work.stride(0), M, s0, ptr(d_rb), ptr(run.rec),
                                       ptr(run.code), ptr(Uc) + 4 * (c0 * K + c0), K, ptr(U_blk_inv), QK_K,
                                       ptr(G) + 4 * c0, K, ptr(idx) + 2 * c0, ptr(gi) + c0, K, st), "ltq_ldlq_feedback")
        best_what_row = d_rb.unsqueeze(1) * G[:, c0:c1]
        W_hat_rot[:, c0:c1] = best_what_row
        d_full[:, ibl] = d_rb.to(torch.float16)
        if c1 < K:
            inter_block(w_blk_start - best_what_row, c0, c1, U_blk_inv)
        yield
    return d_full, W_hat_rot, group


@torch.no_grad()
def _quantize_rows_tcq_ldlq(W_rot: torch.Tensor, U: torch.Tensor, U_blks_inv: torch.Tensor, diag_w: torch.Tensor,
                            spec_name: str, n_pass: int = 2, fused: bool = True) -> Tuple[torch.Tensor, torch.Tensor]:
    """Block16-LDLQ with TCQ tiles, row-scale formats (src/liqk_v2.py:872-1021): returns (d_full fp16 [M, K/256],
    W_hat_rot [M, K]); with PACK set, appends the group's codes to PACK["groups"].  fused: one ltq_ldlq_block launch per
    256-column block; otherwise a gather, a two-pass Viterbi and a feedback launch per 16-column sub-block (same bits)."""
    if PACK is not None and not (TCQ_CONFIG[spec_name].get("tb") and TCQ_CONFIG[spec_name].get("row_scale")):
        raise ValueError(f"{spec_name}: only formats with tail-biting and d_row are written to .ltq")
    d_full, W_hat_rot, group = _rows_ldlq(W_rot, U, U_blks_inv, diag_w, spec_name, fused)
    if PACK is not None:
        PACK["groups"].append(group)
    return d_full, W_hat_rot


@torch.no_grad()
def _quantize_matrix_core(W: torch.Tensor, H: torch.Tensor, spec_or_row_specs, seed: int = 1337, damp: float = 0.02,
                          row_weights: Optional[torch.Tensor] = None, want_pack: bool = False,
                          rows_fn=None, gemm: str = "fp32", row_reduce=None) -> dict:
    """_quantize_matrix_steps run to its end (see there)."""
    return _drive(_quantize_matrix_steps(W, H, spec_or_row_specs, seed, damp, row_weights, want_pack, rows_fn, gemm,
                                         row_reduce))


def _quantize_matrix_steps(W: torch.Tensor, H: torch.Tensor, spec_or_row_specs, seed: int = 1337, damp: float = 0.02,
                           row_weights: Optional[torch.Tensor] = None, want_pack: bool = False, rows_fn=None,
                           gemm: str = "fp32", row_reduce=None):
    """The computation of quantize_matrix_liqk_v2 (src/liqk_v2.py:1029-1198) for the TCQ formats, on the current
    stream and without host synchronisation (with row_weights=None): the reference's data-dependent host branches
    become device-side selections of the same tensors (torch.where), its raising Cholesky / solve their *_ex forms.
    Returns device tensors: qdata, W_hat, num / den of the relative loss, chol_info, and with want_pack the .ltq fields.
    gemm: the mode of the LDLQ inter-block update and refit products ("fp32": the reference's torch operations bit for
    bit; "bf16x6": fp32-accurate split products on the tensor cores, see GEMM_MODES).
    rows_fn: the row-group quantizer called for each format's rows (default: the block-stepped _rows_ldlq).  A
    generator: it yields after the Hessian preparation and after each 256-column block, so that a scheduler can
    interleave the launches of several matrices on several streams; its return value is the result dict.
    row_reduce: for a matrix whose rows are split across ranks (src/liqk_v2.py's quantizer is row-local except for the
    column statistics of suh and the refit's sums over rows), W holds this rank's rows and row_reduce(t) must sum t in
    place over all ranks holding the matrix (e.g. torch.distributed.all_reduce on their group), called in the same
    order on every rank: the column sums of W^2 with the row count, the refit's Gram matrix U^T U and b_in, the two
    refit losses, and num / den.  H is the whole matrix's Hessian on every rank.  No row weights."""
    W_f32 = W.float()
    H_f32 = H.float()
    M, K = W_f32.shape
    nblocks = K // QK_K
    specs_used = [spec_or_row_specs] if isinstance(spec_or_row_specs, str) else [sp for _, _, sp in spec_or_row_specs]
    for sp in specs_used:
        if sp not in TCQ_CONFIG:
            raise ValueError(f"{sp}: not a TCQ format; this path quantizes the TCQ formats only")
        if want_pack and not TCQ_CONFIG[sp].get("tb"):
            raise ValueError(f"{sp}: only formats with tail-biting and d_row are written to .ltq")
    damp *= float(os.environ.get("TCQ_DAMP_MULT", "10"))

    W_rot, H_rot, suh = compute_optimal_suh(W, H_f32, seed=seed, row_weights=row_weights, row_reduce=row_reduce)

    H_reg = H_rot.float().clone()
    diag_mean = H_reg.diagonal().mean().clamp(min=1e-8)
    H_reg.diagonal().add_(damp * diag_mean)
    if gemm == "fp32":  # the reference's factorization and triangular solve L X = I (src/liqk_v2.py:1078-1081)
        L_flip, chol_info = torch.linalg.cholesky_ex(H_reg.flip(0, 1))
        U = torch.linalg.solve_triangular(L_flip, torch.eye(K, dtype=L_flip.dtype, device=L_flip.device), upper=False)
    else:  # blocked factorization whose leaf kernels also invert the diagonal blocks, then the tensor-core merges
        L_flip, chol_info, U = cholesky_lower(H_reg.flip(0, 1), inverse=True, overwrite=True)
    del H_rot, H_reg
    U = U.flip(0, 1)
    diag_w = 1.0 / (torch.diagonal(U) ** 2).clamp(min=1e-12)
    if gemm == "fp32":  # the reference's inverses of U's diagonal blocks (src/liqk_v2.py:1086-1088)
        eye256 = torch.eye(QK_K, dtype=torch.float32, device=W.device).unsqueeze(0).expand(nblocks, -1, -1)
        U_blks = torch.stack([U[b * QK_K:(b + 1) * QK_K, b * QK_K:(b + 1) * QK_K] for b in range(nblocks)], dim=0)
        U_blks_inv = torch.linalg.solve_triangular(U_blks, eye256, upper=True)
    else:
        # U = P L^-1 P (P the reversal), so U^-1 = P L P, and the diagonal blocks of a triangular matrix's inverse are
        # the inverses of its diagonal blocks: U_blk^-1 is the flipped diagonal block of L itself — one strided copy
        # instead of a batched triangular solve (which also blocked the host)
        s0, s1 = L_flip.stride()  # any layout (the factorization may return column-major)
        U_blks_inv = L_flip.as_strided((nblocks, QK_K, QK_K), (QK_K * (s0 + s1), s0, s1),
                                       L_flip.storage_offset()).flip(0, 1, 2).contiguous()
    del L_flip
    U_parts = None  # the fused path builds its own bf16 operands of U (ltq_ldlq_bcat)
    yield

    row_slices = [(0, M, spec_or_row_specs)] if isinstance(spec_or_row_specs, str) else spec_or_row_specs
    by_spec: Dict[str, List[Tuple[int, int]]] = {}
    for r0, r1, sp in row_slices:
        by_spec.setdefault(sp, []).append((r0, r1))

    W_hat_rot = torch.empty_like(W_rot)
    d_full = torch.empty((M, nblocks), dtype=torch.float16, device=W.device)
    pm = None
    if want_pack:
        pm = {"idx": torch.empty((M, K), dtype=torch.int16, device=W.device),
              "gi": torch.empty((M, K), dtype=torch.uint8, device=W.device),
              "G": torch.empty((M, K), dtype=torch.float32, device=W.device), "d_row": torch.empty(M, device=W.device),
              "e": torch.empty((M, nblocks), dtype=torch.int8, device=W.device)}
    for sp, ranges in by_spec.items():
        if len(ranges) == 1 and ranges[0] == (0, M):
            rows_idx = None
            if rows_fn is None:
                d_sub, Wh_sub, g = yield from _rows_ldlq_steps(W_rot, U, U_blks_inv, diag_w, sp, True, gemm, U_parts)
            else:
                d_sub, Wh_sub, g = rows_fn(W_rot, U, U_blks_inv, diag_w, sp)
            W_hat_rot, d_full = Wh_sub, d_sub
            if pm is not None:
                for k in ("idx", "gi", "G", "d_row", "e"):
                    pm[k] = g[k].to(pm[k].dtype)
            continue
        rows_idx = torch.cat([torch.arange(r0, r1, device=W.device) for r0, r1 in ranges], dim=0)
        if rows_fn is None:
            d_sub, Wh_sub, g = yield from _rows_ldlq_steps(W_rot[rows_idx], U, U_blks_inv, diag_w, sp, True, gemm,
                                                           U_parts)
        else:
            d_sub, Wh_sub, g = rows_fn(W_rot[rows_idx], U, U_blks_inv, diag_w, sp)
        W_hat_rot[rows_idx] = Wh_sub
        d_full[rows_idx] = d_sub
        if pm is not None:
            for k in ("idx", "gi", "G", "d_row", "e"):
                pm[k][rows_idx] = g[k].to(pm[k].dtype)
    del U, U_blks_inv, W_rot, U_parts

    if gemm == "fp32":
        def times_h(A):
            return A @ H_f32
    else:
        Kp = tcgemm._pad(K)
        Hb3 = tcgemm.split3(H_f32, trans=True, Kp=Kp)  # the split of H (as the right operand), shared by every product

        def times_h(A):
            return tcgemm.times(A, Hb3, Kp)
    U_base = fwht_inplace(W_hat_rot.clone(), block_size=QK_K)
    W_hat_eff = U_base * suh.unsqueeze(0)
    c_pack = torch.ones((M,), dtype=torch.float32, device=W.device)
    HW = times_h(W_f32)
    HQ = times_h(W_hat_eff)
    c_row = (W_hat_eff * HW).sum(dim=1) / (W_hat_eff * HQ).sum(dim=1).clamp(min=1e-12)
    c_row = torch.where(torch.isfinite(c_row) & (c_row > 0.5) & (c_row < 2.0), c_row, torch.ones_like(c_row))
    d_new = (d_full.float() * c_row.unsqueeze(1)).to(torch.float16)
    c_eff = (d_new.float() / d_full.float().clamp(min=1e-12)).mean(dim=1, keepdim=True)
    U_scaled = U_base * c_eff
    if row_weights is not None:
        rw = row_weights.float().clamp(min=float(row_weights.mean().item()) * 0.1)
        rw = (rw / rw.mean().clamp(min=1e-12)).clamp(0.25, 4.0)
        U_w = U_scaled * rw.unsqueeze(1)
    else:
        rw = torch.ones((M,), dtype=torch.float32, device=W.device)
        U_w = U_scaled
    if gemm == "fp32":
        A_in = U_w.T @ U_scaled
    elif row_weights is None:  # U_w is U_scaled: a Gram matrix, needed on its lower triangle only (Cholesky below)
        A_in = tcgemm.gram_lower(U_scaled, QK_K * (K // QK_K // 2) if K >= 4 * QK_K else K)
    else:
        A_in = _mm(U_w.T, U_scaled, gemm)
    b_in = (U_w * HW).sum(dim=0)
    if row_reduce is not None:  # both are sums over the rows
        row_reduce(A_in)
        row_reduce(b_in)
    A_in = A_in * H_f32
    A_in.diagonal().add_(1e-3 * A_in.diagonal().mean().clamp(min=1e-12))
    # the reference solves, and keeps the refit when the solve succeeds and lowers the loss (src/liqk_v2.py:1161-1180).
    # A_in = (U_w^T U_scaled) o H + eps I is symmetric positive definite by construction (a Schur product of two Gram
    # matrices plus a positive diagonal): the fast mode solves it by Cholesky (no pivot search, no host-blocking LU);
    # a failed factorization skips the refit like the reference's failed solve.  The fp32 mode keeps the reference's LU.
    if gemm == "fp32":
        sol, solve_info = torch.linalg.solve_ex(A_in, b_in)
    else:
        Lc, solve_info, Dinv = cholesky_lower(A_in, overwrite=True, diag_inv=True)
        sol = chol_solve(Lc, Dinv, b_in)
        del Lc, Dinv
    suh_cand = sol.to(torch.float16).to(torch.float32)
    valid_s = torch.isfinite(suh_cand) & (suh_cand.abs() > 0.05) & (suh_cand.abs() < 10.0)
    suh_cand = torch.where(valid_s, suh_cand, suh)
    W_hat_cand = U_scaled * suh_cand.unsqueeze(0)
    HQ_cand = times_h(W_hat_cand)
    diff_base = W_f32 - W_hat_eff
    diff_cand = W_f32 - W_hat_cand
    loss_base = (((HW - HQ) * diff_base).sum(dim=1) * rw).sum()
    loss_cand = (((HW - HQ_cand) * diff_cand).sum(dim=1) * rw).sum()
    if row_reduce is not None:
        losses = torch.stack([loss_base, loss_cand])
        row_reduce(losses)
        loss_base, loss_cand = losses[0], losses[1]
    take = (solve_info == 0) & (loss_cand < loss_base)
    W_hat_eff = torch.where(take, W_hat_cand, W_hat_eff)
    d_full = torch.where(take, d_new, d_full)
    suh = torch.where(take, suh_cand, suh)
    HQ = torch.where(take, HQ_cand, HQ)
    c_pack = torch.where(take, c_eff.squeeze(1), c_pack)
    del W_hat_cand, HQ_cand, diff_base, diff_cand, U_scaled, U_w, A_in
    pack = None
    if pm is not None:
        d_row_p = (pm["d_row"] * c_pack).to(torch.float16)
        suh_p = suh.to(torch.float16)
        scale = d_row_p.float().unsqueeze(1) * torch.exp2(0.25 * pm["e"].float())
        Wq_rot = (scale.unsqueeze(2) * pm["G"].view(M, nblocks, QK_K)).view(M, K)
        W_pk = fwht_inplace(Wq_rot, block_size=QK_K) * suh_p.float().unsqueeze(0)
        if gemm == "fp32":
            HQ = times_h(W_pk)
        else:
            # the packed reconstruction differs from W_hat_eff only by the fp16 roundings of the row scale and suh:
            # HQ takes the product of that small change, in the three-product bf16 form (a0 b0 + a1 b0 + a0 b1:
            # relative error ~2^-16 of the change, far below fp32 rounding of HQ itself)
            HQ = tcgemm.gemm3(tcgemm.split3(W_pk - W_hat_eff, Kp=Kp), Hb3, HQ, Kp, beta=1.0, nq=2)
        W_hat_eff = W_pk
        pack = {"row_slices": row_slices, "idx": pm["idx"], "gi": pm["gi"], "G": pm["G"], "d_row": d_row_p,
                "e": pm["e"], "suh": suh_p}
    del times_h
    diff = W_f32 - W_hat_eff
    num = ((HW - HQ) * diff).sum()
    den = (HW * W_f32).sum()
    if row_reduce is not None:
        nd = torch.stack([num, den])
        row_reduce(nd)
        num, den = nd[0], nd[1]
    den = den.clamp(min=1e-12)
    qdata = {"d": d_full, "suh": suh.to(torch.float16), "row_slices": row_slices}
    return {"qdata": qdata, "W_hat": W_hat_eff, "num": num, "den": den, "chol_info": chol_info, "pack": pack}


@torch.no_grad()
def quantize_matrix_liqk_v2(W: torch.Tensor, H: torch.Tensor, spec_or_row_specs, seed: int = 1337, damp: float = 0.02,
                            row_weights: Optional[torch.Tensor] = None, cd_sweeps: int = 2, out_rot: bool = False):
    """src/liqk_v2.py:1029-1198 for the TCQ formats: returns (qdata, W_hat [M, K] fp32, rel_loss); with PACK set,
    PACK["matrix"] holds the .ltq fields (row_slices, idx, gi, G, d_row fp16, e int8, suh fp16).  Raises like
    torch.linalg.cholesky when the damped Hessian is not positive definite."""
    _lib.require_cuda(W, H)
    if out_rot:
        s_out = make_rademacher_signs(W.shape[0], seed=seed + 7919, device=W.device)
        rw = None
        if row_weights is not None:
            rw = row_weights.float().view(-1, QK_K).mean(dim=1, keepdim=True).expand(-1, QK_K).reshape(-1)
        q_res, w_hat_r, rel = quantize_matrix_liqk_v2(_fwht_rows(W.float() * s_out.unsqueeze(1)), H, spec_or_row_specs,
                                                      seed=seed, damp=damp, row_weights=rw, cd_sweeps=cd_sweeps)
        q_res["s_out"] = s_out.to(torch.int8)
        return q_res, _fwht_rows(w_hat_r) * s_out.unsqueeze(1), rel

    want_pack = PACK is not None
    if want_pack:
        PACK["groups"] = []

    def rows_fn(W_rot, U, U_blks_inv, diag_w, sp):  # the row groups also pass through PACK["groups"], as in the reference
        d_sub, Wh_sub = _quantize_rows_tcq_ldlq(W_rot, U, U_blks_inv, diag_w, sp)
        return d_sub, Wh_sub, (PACK["groups"].pop() if want_pack else {})

    r = _quantize_matrix_core(W, H, spec_or_row_specs, seed, damp, row_weights, want_pack,
                              rows_fn=rows_fn if want_pack else None)
    if int(r["chol_info"].item()) != 0:
        raise torch.linalg.LinAlgError("linalg.cholesky: the damped Hessian is not positive-definite "
                                       f"(leading minor of order {int(r['chol_info'].item())})")
    if want_pack:
        PACK["matrix"] = r["pack"]
    rel_loss = float(r["num"].item()) / float(r["den"].item())
    return r["qdata"], r["W_hat"], rel_loss
