"""GPU: row tables quantized as LTQ rings (src/ple_quant.py:29-80, config 5's path).

quantize_rings runs the three scale tries of a chunk as one Viterbi call; it must equal (bit for bit) the reference's
structure of one call per try, and the same function with the Viterbi replaced by the pinned CPU oracle.  int8_rows
equals its restatement.  Inputs: a seeded bf16 table with the config's value distribution (N(0, 0.03) x a log-normal
row scale), small enough for the oracle."""
import numpy as np
import pytest
import torch

from oracle import oracle as O

pytestmark = pytest.mark.gpu


def _table(rows, cols, seed):
    g = torch.Generator().manual_seed(seed)
    return (torch.randn(rows, cols, generator=g) * 0.03 * torch.exp(0.5 * torch.randn(rows, 1, generator=g))
            ).to(torch.bfloat16)


def _per_try_reference(W, spec, rot, scales=(0.9, 1.0, 1.12)):
    """src/ple_quant.py:37-65 as written: one Viterbi call per scale try."""
    from ltq_research_b200.formats import TCQ_CONFIG, load_formats
    from ltq_research_b200.liqk_v2 import fwht_inplace
    from ltq_research_b200.rings import RING, hadamard_signs
    from ltq_research_b200.tcq_proto import viterbi_ub_cuda
    fmt = load_formats([spec], "cuda")[spec]
    cfg = TCQ_CONFIG[spec]
    lut = torch.tensor(fmt.lut, device="cuda")
    gains = torch.tensor(fmt.gain_tab, device="cuda")
    signs = hadamard_signs().cuda()
    x = W.view(-1, RING).cuda().float()
    if rot:
        x = fwht_inplace((x * signs).contiguous(), block_size=RING)
    rms = x.square().mean(dim=1, keepdim=True).sqrt().clamp(min=1e-8) * cfg.get("scale", 1.0)
    best, best_err = None, None
    for sc in scales:
        d = (rms * sc).half().float()
        rec = viterbi_ub_cuda(x / d, lut, fmt.K, 10, fmt.masks[0], gains, sub=fmt.sub, tail_biting=True,
                              m_extra=fmt.masks[1:], pair_parity=fmt.frac, n_cand=cfg.get("n_cand", 0)) * d
        err = (rec - x).square().sum(dim=1)
        if best is None:
            best, best_err = rec, err
        else:
            better = err < best_err
            best = torch.where(better.unsqueeze(1), rec, best)
            best_err = torch.where(better, err, best_err)
    if rot:
        best = fwht_inplace(best.contiguous(), block_size=RING) * signs
    return best.to(W.dtype).cpu().view_as(W)


@pytest.mark.parametrize("spec,rot", [("TCQ4X", True), ("TCQ3X", False), ("TCQ25X", True)])
def test_quantize_rings_batched_tries_equal_per_try(spec, rot, cuda_dev):
    from ltq_research_b200.rings import quantize_rings
    W = _table(96, 1024, 7)
    got, bpv = quantize_rings(W, spec, rot, chunk=200)
    assert got.dtype == W.dtype and got.device == W.device and got.shape == W.shape
    assert torch.equal(got, _per_try_reference(W, spec, rot))
    rel = ((got.float() - W.float()).square().sum() / W.float().square().sum()).item()
    assert rel < 0.1, rel
    from ltq_research_b200.formats import load_formats
    assert bpv == load_formats([spec], cuda_dev)[spec].tile_bytes() * 8 / 256 + 16 / 256


def test_quantize_rings_on_oracle_viterbi(cuda_dev, monkeypatch):
    """The same function with the Viterbi replaced by the CPU oracle gives the same table."""
    import ltq_research_b200.rings as R
    W = _table(16, 512, 9)
    got, _ = R.quantize_rings(W, "TCQ4X", True)

    def oracle_viterbi(x, small, K, nu, m, gains=None, **kw):
        rec = O.viterbi(x.cpu().numpy(), small.cpu().numpy(), K, nu, m, gains.cpu().numpy(), **kw)
        return torch.from_numpy(np.asarray(rec)).to(x.device)
    monkeypatch.setattr(R, "viterbi_ub_cuda", oracle_viterbi)
    want, _ = R.quantize_rings(W, "TCQ4X", True)
    assert torch.equal(got, want)


def _int8_reference(W):
    """src/ple_quant.py:68-77 restated: fp16 absmax scale per ring, round half to even, clamp, rescale (torch, CPU)."""
    x = W.reshape(-1, 256).float()
    d = (x.abs().amax(dim=1, keepdim=True) / 127).half().float().clamp(min=1e-10)
    return ((x / d).round().clamp(-127, 127) * d).to(W.dtype).view_as(W)


def _same(a, b):
    """Equal values, NaN where NaN (bit patterns of NaN aside)."""
    an, bn = torch.isnan(a.float()), torch.isnan(b.float())
    return torch.equal(an, bn) and torch.equal(a[~an], b[~bn])


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_int8_rows(cuda_dev, dtype):
    """ltq_int8_rings (one warp per ring) against the reference's torch expression: a seeded table, plus rings of
    zeros, exact half-steps (ties to even), a NaN, an infinity and values beyond fp16's range."""
    from ltq_research_b200.rings import int8_rows
    W = _table(32, 512, 11).to(dtype)
    got, bpv = int8_rows(W)
    assert got.dtype == W.dtype and got.device == W.device and bpv == 8 + 16 / 256
    assert torch.equal(got, _int8_reference(W))
    S = torch.zeros(6, 256, dtype=torch.float32)
    S[1] = (torch.arange(256) % 200 - 100) + 0.5  # max |x| = 127 below gives d = 1: x / d = k + 0.5, ties to even
    S[1, 0] = 127.0
    S[2] = torch.randn(256, generator=torch.Generator().manual_seed(3))
    S[2, 5] = float("nan")
    S[3] = torch.randn(256, generator=torch.Generator().manual_seed(4))
    S[3, 9] = float("inf")
    S[4] = torch.randn(256, generator=torch.Generator().manual_seed(5)) * 1e7   # max / 127 above fp16's range
    S[5] = torch.randn(256, generator=torch.Generator().manual_seed(6)) * 1e-12  # scale clamped to 1e-10
    S = S.to(dtype)
    got, _ = int8_rows(S.to(cuda_dev))
    assert _same(got.cpu(), _int8_reference(S))
