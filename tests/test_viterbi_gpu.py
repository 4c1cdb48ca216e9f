"""GPU parity of the B200 Viterbi (through the C ABI via ltq_research_b200.viterbi_ub_cuda) against the CPU oracle
and, when built, against the reference CUDA kernel compiled from its own source for sm_100a (oracle/_ref).
Bit-exact: reconstruction bits, gain indices, level indices, start / end / middle states."""
import numpy as np
import pytest
import torch

from oracle import oracle as O
from oracle import ref_kernel as R
from tests import vit_cases as VC

pytestmark = pytest.mark.gpu

ALL_CASES = (VC.menu_tb_cases(N=24, L=256, seed=1) + VC.menu_tb_cases(N=16, L=160, seed=2)
             + VC.menu_tb_cases(N=16, L=256, seed=4, window=32, weighted=True) + VC.special_cases()
             + VC.direct_cases() + VC.nl32_cases() + VC.s256_cases())


def _to_dev(kw, dev):
    out = dict(kw)
    for k in ("small", "gains", "small_hi", "gains_hi"):
        if k in out and out[k] is not None:
            out[k] = torch.from_numpy(np.ascontiguousarray(out[k])).to(dev)
    if out.get("init_state") is not None:
        out["init_state"] = torch.from_numpy(out["init_state"]).to(dev)
    return out


def _run_dev(fn, kw, x, wts, dev):
    kw = _to_dev(kw, dev)
    small = kw.pop("small")
    xd = torch.from_numpy(x).to(dev)
    wd = None if wts is None else torch.from_numpy(np.ascontiguousarray(wts)).to(dev)
    out = fn(xd, small, wts=wd, **kw)
    torch.cuda.synchronize()
    return tuple(o.cpu().numpy() for o in out) if isinstance(out, tuple) else (out.cpu().numpy(),)


def _run_oracle(kw, x, wts):
    kw = dict(kw)
    small = kw.pop("small")
    out = O.viterbi(x, small, wts=wts, **kw)
    return out if isinstance(out, tuple) else (out,)


def _same(a, b, kw, name):
    if kw.get("_mid"):
        assert np.array_equal(a[1], b[1]), f"{name}: middle state"
        return
    assert np.array_equal(np.ascontiguousarray(a[0]).view(np.uint32), np.ascontiguousarray(b[0]).view(np.uint32)), \
        f"{name}: reconstruction differs in {(a[0] != b[0]).sum()} of {a[0].size}"
    for i in range(1, len(a)):
        assert np.array_equal(a[i], b[i]), f"{name}: output {i} differs in {(a[i] != b[i]).sum()}"


@pytest.mark.parametrize("case", ALL_CASES, ids=[c[0] for c in ALL_CASES])
def test_kernel_matches_oracle(case, cuda_dev):
    from ltq_research_b200.tcq_proto import viterbi_ub_cuda
    name, kw, x, wts = case
    got = _run_dev(viterbi_ub_cuda, kw, x, wts, cuda_dev)
    want = _run_oracle(kw, x, wts)
    _same(got, want, kw, name)


@pytest.mark.skipif(not R.available(), reason="reference kernel not built (make -C oracle ref)")
@pytest.mark.parametrize("case", ALL_CASES, ids=[c[0] for c in ALL_CASES])
def test_kernel_matches_reference_kernel(case, cuda_dev):
    from ltq_research_b200.tcq_proto import viterbi_ub_cuda
    name, kw, x, wts = case
    got = _run_dev(viterbi_ub_cuda, kw, x, wts, cuda_dev)
    ref = _run_dev(R.viterbi_ub_cuda_ref, kw, x, wts, cuda_dev)
    _same(got, ref, kw, name)


def test_config1_full_size_properties(cuda_dev):
    """Config 1 at full size (65,536 tiles of a seeded 4096 x 4096 N(0,1) matrix): every tile closes (tail-biting
    labels recomputed from the code bits), packs and decodes to its reconstruction, and a sample of tiles matches the
    oracle bit for bit."""
    from ltq_research_b200.tcq_proto import viterbi_ub_cuda
    c = VC.F["_config1_tcq_K2_h2"]
    g = torch.Generator(device="cpu").manual_seed(0)
    W = torch.randn(4096, 4096, generator=g)
    tiles = W.reshape(256, 16, 256, 16).permute(0, 2, 1, 3).reshape(-1, 256).contiguous()
    d = tiles.square().mean(dim=1, keepdim=True).sqrt().half().float()
    x = (tiles / d).to(cuda_dev)
    small = torch.tensor(c["lut"], device=cuda_dev)
    gains = torch.tensor(c["gains_cpu"], device=cuda_dev)
    rec, gi, idx = viterbi_ub_cuda(x, small, 2, 10, 359, gains, sub=16, tail_biting=True, return_code=True)
    torch.cuda.synchronize()
    assert rec.shape == (65536, 256)
    # closure of every tile on the GPU: state from the code bits, label recomputed, equal to the chosen label
    lab = (idx // 2).long()
    cb = lab & 1
    s = sum(torch.roll(cb, j, dims=1) << j for j in range(10))
    par = torch.zeros_like(s)
    v = (s >> 1) & 359
    for _ in range(9):
        par ^= v & 1
        v >>= 1
    assert torch.equal((s & 1) | (par << 1), lab)
    # reconstruction = gain * lut[label * U + u]
    assert torch.equal(rec, gains[gi.long()] * small[idx.long()])
    sel = torch.arange(0, 65536, 4099)
    want = O.viterbi(x[sel].cpu().numpy(), c["lut"], 2, 10, 359, np.asarray(c["gains_cpu"], np.float32),
                     tail_biting=True, return_code=True)
    assert np.array_equal(rec[sel].cpu().numpy().view(np.uint32), want[0].view(np.uint32))
    assert np.array_equal(idx[sel].cpu().numpy(), want[2])
    mse = float(((x - rec) * d.to(cuda_dev)).square().mean())
    assert 0.05 < mse < 0.08, mse
