"""Row tables quantized as LTQ rings (lumen-inference/ltq-research src/ple_quant.py:29-80): a table [rows, n * 256] is cut
into rings of 256 values, each ring one tail-biting trellis of a .ltq format (the same Viterbi as the matrices, no
Hessian: plain MSE) with an fp16 scale per ring, optionally after a Hadamard-256 rotation with fixed random signs.

The reference tries three ring scales one Viterbi call at a time; here the three tries of a chunk are one call over
3 x the rings (the rings are independent tiles, so the codes are the same), and the selection keeps the reference's
order (a later scale replaces an earlier one only with a strictly smaller error).  Everything runs on the device; the
result returns to the table's device and dtype.
"""
from __future__ import annotations

from typing import Tuple

import torch

from . import _lib
from .formats import TCQ_CONFIG, load_formats
from .liqk_v2 import fwht_inplace
from .tcq_proto import viterbi_ub_cuda

RING = 256


def hadamard_signs(seed: int = 4242) -> torch.Tensor:
    """The ring rotation's ±1 signs (src/ple_quant.py:31-34), from the CPU generator."""
    g = torch.Generator().manual_seed(seed)
    return (torch.randint(0, 2, (RING,), generator=g) * 2 - 1).float()


@torch.no_grad()
def quantize_rings(W: torch.Tensor, spec: str, rot: bool, chunk: int = 1 << 17, scales=(0.9, 1.0, 1.12),
                   device=None) -> Tuple[torch.Tensor, float]:
    """W [rows, n * 256] -> (reconstructed table, same device and dtype as W; bits per value).  The ring scale is fp16,
    the MSE-best of `scales` x rms x the format's scale multiplier (src/ple_quant.py:37-65)."""
    dev = torch.device(device) if device is not None else (W.device if W.is_cuda else torch.device("cuda"))
    if dev.type != "cuda":
        raise RuntimeError("quantize_rings: a CUDA device is required; there is no CPU path")
    _lib.lib()
    fmt = load_formats([spec], dev)[spec]
    cfg = TCQ_CONFIG[spec]
    lut = torch.tensor(fmt.lut, device=dev)
    gains = torch.tensor(fmt.gain_tab, device=dev)
    signs = hadamard_signs().to(dev)
    rings = W.view(-1, RING)
    out = torch.empty_like(rings)
    for i in range(0, rings.shape[0], chunk):
        x = rings[i: i + chunk].to(dev).float()
        n = x.shape[0]
        if rot:
            x = fwht_inplace((x * signs).contiguous(), block_size=RING)
        rms = x.square().mean(dim=1, keepdim=True).sqrt().clamp(min=1e-8) * cfg.get("scale", 1.0)
        ds = [(rms * sc).half().float() for sc in scales]
        recs = viterbi_ub_cuda(torch.cat([x / d for d in ds], dim=0), lut, fmt.K, 10, fmt.masks[0], gains, sub=fmt.sub,
                               tail_biting=True, m_extra=fmt.masks[1:], pair_parity=fmt.frac,
                               n_cand=cfg.get("n_cand", 0))
        best, best_err = None, None
        for k, d in enumerate(ds):
            rec = recs[k * n: (k + 1) * n] * d
            err = (rec - x).square().sum(dim=1)
            if best is None:
                best, best_err = rec, err
            else:
                better = err < best_err
                best = torch.where(better.unsqueeze(1), rec, best)
                best_err = torch.where(better, err, best_err)
        if rot:
            best = fwht_inplace(best.contiguous(), block_size=RING) * signs
        out[i: i + chunk] = best.to(out.dtype).to(out.device)
    return out.view_as(W), fmt.tile_bytes() * 8 / RING + 16 / RING


@torch.no_grad()
def int8_rows(W: torch.Tensor, chunk: int = 1 << 17, device=None) -> Tuple[torch.Tensor, float]:
    """int8 with an fp16 absmax scale per ring of 256 values (src/ple_quant.py:68-77), the comparison baseline."""
    dev = torch.device(device) if device is not None else (W.device if W.is_cuda else torch.device("cuda"))
    rings = W.view(-1, RING)
    out = torch.empty_like(rings)
    for i in range(0, rings.shape[0], chunk):
        x = rings[i: i + chunk].to(dev).float()
        d = (x.abs().amax(dim=1, keepdim=True) / 127).half().float().clamp(min=1e-10)
        out[i: i + chunk] = ((x / d).round().clamp(-127, 127) * d).to(out.dtype).to(out.device)
    return out.view_as(W), 8 + 16 / RING
