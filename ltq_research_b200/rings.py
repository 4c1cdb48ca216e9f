"""Row tables quantized as LTQ rings (lumen-inference/ltq-research src/ple_quant.py:29-80): a table [rows, n * 256] is cut
into rings of 256 values, each ring one tail-biting trellis of a .ltq format (the same Viterbi as the matrices, no
Hessian: plain MSE) with an fp16 scale per ring, optionally after a Hadamard-256 rotation with fixed random signs.

Organisation on the device: per chunk of rings, the rotation is one kernel (ltq_fwht256 with the signs as column
scale), the candidate ring scales s x rms x the format's multiplier are evaluated together — all tries of the chunk go
to ONE tail-biting Viterbi call over (tries x rings) tiles, since rings are independent tiles — and the choice among
the tries is a first-index argmin over their squared errors, which is the reference's sequential rule (a later try
replaces the kept one only with a strictly smaller error; an error that is NaN is never taken, except by the first
try, which is then kept).  The int8 comparison format is one kernel (ltq_int8_rings).
"""
from __future__ import annotations

from typing import Sequence, Tuple

import torch

from . import _lib
from ._lib import ptr
from .formats import TCQ_CONFIG, load_formats
from .liqk_v2 import fwht_inplace, fwht_rows_scaled
from .tcq_proto import viterbi_ub_cuda

RING = 256
SIGN_SEED = 4242  # seed of the rotation's sign vector (part of the ring format: src/ple_quant.py:31-34)


def hadamard_signs(seed: int = SIGN_SEED) -> torch.Tensor:
    """The ring rotation's +-1 signs: 256 fair bits from torch's CPU generator seeded with `seed`, as 2 b - 1."""
    bits = torch.randint(0, 2, (RING,), generator=torch.Generator().manual_seed(seed))
    return (2 * bits - 1).float()


def _target_device(W: torch.Tensor, device) -> torch.device:
    dev = torch.device(device) if device is not None else (W.device if W.is_cuda else torch.device("cuda"))
    if dev.type != "cuda":
        raise RuntimeError("ring quantization needs a CUDA device; there is no CPU path")
    return dev


def _first_best(errs: torch.Tensor) -> torch.Tensor:
    """Index of the kept try per ring, errs [tries, rings]: the first try of least error; a NaN error is never taken
    (and a NaN first try is kept)."""
    e = errs.clone()
    e[1:] = torch.nan_to_num(e[1:], nan=float("inf"))
    first_nan = torch.isnan(e[0])
    e[0] = torch.where(first_nan, torch.full_like(e[0], -float("inf")), e[0])
    return e.argmin(dim=0)


@torch.no_grad()
def quantize_rings(W: torch.Tensor, spec: str, rot: bool, chunk: int = 1 << 17, scales: Sequence[float] = (0.9, 1.0, 1.12),
                   device=None) -> Tuple[torch.Tensor, float]:
    """W [rows, n * 256] -> (reconstructed table with W's device and dtype, bits per value = tile bits + fp16 scale).
    Each ring's scale is the fp16 value of s * rms * (format multiplier) for the s in `scales` whose reconstruction
    has the least squared error (src/ple_quant.py:37-65)."""
    dev = _target_device(W, device)
    fmt = load_formats([spec], dev)[spec]
    mult = TCQ_CONFIG[spec].get("scale", 1.0)
    n_cand = TCQ_CONFIG[spec].get("n_cand", 0)
    lut = torch.tensor(fmt.lut, device=dev)
    gains = torch.tensor(fmt.gain_tab, device=dev)
    signs = hadamard_signs().to(dev)
    rings = W.reshape(-1, RING)
    out = torch.empty_like(rings)
    for r0 in range(0, rings.shape[0], chunk):
        x = rings[r0: r0 + chunk].to(dev).float().contiguous()
        n = x.shape[0]
        if rot:  # H256(x * signs): the sign flip is exact, so the scaled-column transform is the same bits
            x = fwht_rows_scaled(x, signs, mode=2)
        rms = x.square().mean(dim=1, keepdim=True).sqrt().clamp(min=1e-8) * mult
        d = [(rms * s).half().float() for s in scales]                      # per try: [n, 1]
        tiles = torch.cat([x / dk for dk in d], dim=0)                      # [tries * n, 256]
        q = viterbi_ub_cuda(tiles, lut, fmt.K, 10, fmt.masks[0], gains, sub=fmt.sub, tail_biting=True,
                            m_extra=fmt.masks[1:], pair_parity=fmt.frac, n_cand=n_cand)
        recs = [q[k * n: (k + 1) * n] * dk for k, dk in enumerate(d)]       # per try: [n, 256]
        errs = torch.stack([(rk - x).square().sum(dim=1) for rk in recs])   # [tries, n]
        keep = _first_best(errs)
        best = torch.stack(recs).gather(0, keep.view(1, n, 1).expand(1, n, RING)).squeeze(0)
        if rot:
            best = fwht_inplace(best.contiguous(), block_size=RING) * signs
        out[r0: r0 + n] = best.to(out.dtype).to(out.device)
    return out.view_as(W), fmt.tile_bytes() * 8 / RING + 16 / RING


@torch.no_grad()
def int8_rows(W: torch.Tensor, chunk: int = 1 << 17, device=None) -> Tuple[torch.Tensor, float]:
    """The comparison format of the ring tables (src/ple_quant.py:68-77): per ring of 256 values the fp16 scale
    d = max(fp16(max |x| / 127), 1e-10) and the values round(x / d) clamped to [-127, 127], times d.  One kernel per
    chunk (ltq_int8_rings), reading and writing the table's own dtype (fp32 or bf16).  Returns (table, 8 + 16/256)."""
    dev = _target_device(W, device)
    if W.dtype not in (torch.float32, torch.bfloat16):
        raise TypeError("int8_rows: the table must be fp32 or bf16")
    rings = W.reshape(-1, RING)
    out = torch.empty_like(rings)
    bf16 = 1 if W.dtype == torch.bfloat16 else 0
    for r0 in range(0, rings.shape[0], chunk):
        x = rings[r0: r0 + chunk].to(dev).contiguous()
        y = torch.empty_like(x)
        rc = _lib.lib().ltq_int8_rings(ptr(x), ptr(y), x.shape[0], bf16, _lib.stream_ptr(dev))
        if rc != 0:
            raise RuntimeError(f"ltq_int8_rings: error code {rc}")
        out[r0: r0 + x.shape[0]] = y.to(out.device)
    return out.view_as(W), 8 + 16 / RING
