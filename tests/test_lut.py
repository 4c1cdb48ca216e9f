"""DP-profile sub-block quantization through the 1-D table (src/cuda/tcq_viterbi.cu:768-811, src/liqk_v2.py:444-506).

Pins: the oracle (oracle.lut_subs) against the reference's own kernel run on a B200 (tests/golden/lut_subs.npz from
tests/golden/make_golden_lut.py, inputs rebuilt by tests/golden/lut_inputs.py: bucket-boundary ties, clamping,
duplicate columns, zero weights, NaN / inf); the product kernel (lut_subs_quant, one warp per sub-block) bit for bit
against both, and at the reference's 8192-bucket size; quantize_liqk_v2_diag_rot on the kernel equals the same
function with the kernel replaced by the oracle."""
from pathlib import Path

import numpy as np
import pytest
import torch

from oracle import oracle as O
from tests.golden.lut_inputs import case, table

GOLDEN = Path(__file__).resolve().parent / "golden" / "lut_subs.npz"


def test_oracle_matches_reference_kernel():
    xs, dh, lut, inv_step, half_b = case()
    want = np.load(GOLDEN)["out"]
    got = O.lut_subs(xs, dh, lut, inv_step, half_b)
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))


@pytest.mark.gpu
def test_kernel_matches_reference_kernel(cuda_dev):
    from ltq_research_b200.tcq_proto import lut_subs_quant_cuda
    xs, dh, lut, inv_step, half_b = case()
    got = lut_subs_quant_cuda(torch.from_numpy(xs).to(cuda_dev), torch.from_numpy(dh).to(cuda_dev),
                              torch.from_numpy(lut).to(cuda_dev), inv_step, half_b).cpu().numpy()
    want = np.load(GOLDEN)["out"]
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))


@pytest.mark.gpu
def test_kernel_matches_oracle_full_table(cuda_dev):
    """The reference's table size (8192 buckets x 64) and a profile-sized batch of sub-blocks."""
    from ltq_research_b200.tcq_proto import lut_subs_quant_cuda
    g = np.random.default_rng(8)
    max_g = 3.7
    lut = table(8192, max_g)
    S = 40000
    xs = (g.standard_normal((S, 16)) * 1.3).astype(np.float32)
    dh = g.uniform(0.01, 3.0, (S, 16)).astype(np.float32)
    inv_step, half_b = 8191 / (2 * max_g), 8191 * 0.5
    got = lut_subs_quant_cuda(torch.from_numpy(xs).to(cuda_dev), torch.from_numpy(dh).to(cuda_dev),
                              torch.from_numpy(lut).to(cuda_dev), inv_step, half_b).cpu().numpy()
    want = O.lut_subs(xs, dh, lut, inv_step, half_b)
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))


@pytest.mark.gpu
def test_lut_subs_rejects_bad_arguments(cuda_dev):
    from ltq_research_b200 import _lib
    L = _lib.lib()
    st = torch.cuda.current_stream().cuda_stream
    x = torch.zeros(16, device=cuda_dev)
    assert L.lut_subs_quant(x.data_ptr(), x.data_ptr(), None, x.data_ptr(), 1, 1.0, 0.0, 1, st) == -1
    assert L.lut_subs_quant(x.data_ptr(), x.data_ptr(), x.data_ptr(), x.data_ptr(), 1, 1.0, 0.0, 0, st) == -1
    assert L.lut_subs_quant(x.data_ptr(), x.data_ptr(), x.data_ptr(), x.data_ptr(), 0, 1.0, 0.0, 1, st) == 0


@pytest.mark.gpu
def test_diag_rot_profile_on_kernel_equals_oracle(cuda_dev, monkeypatch):
    """quantize_liqk_v2_diag_rot (src/liqk_v2.py:469-506) with a registered bank: the kernel path and the same
    function with lut_subs_quant_cuda replaced by the oracle give the same bits; the torch path (other table widths)
    runs on the same bank."""
    import ltq_research_b200.liqk_v2 as L
    import ltq_research_b200.tcq_proto as T
    g = torch.Generator().manual_seed(5)
    levels = torch.stack([torch.linspace(-1, 1, 15) * (1.5 + 0.04 * c) for c in range(64)])
    L.register_warp_register_bank("TEST_BANK", levels, 2.0, cuda_dev)
    W = (torch.randn(64, 512, generator=g) * torch.exp(torch.randn(64, 1, generator=g))).to(cuda_dev)
    dh = (torch.rand(512, generator=g) + 0.1).to(cuda_dev)
    got = L.quantize_liqk_v2_diag_rot(W, dh, "TEST_BANK")

    def via_oracle(x_subs, d, lut_val, inv_step, half_b):
        out = O.lut_subs(x_subs.cpu().numpy(), d.cpu().numpy(), lut_val.cpu().numpy(), inv_step, half_b)
        return torch.from_numpy(out).to(x_subs.device)
    monkeypatch.setattr(T, "lut_subs_quant_cuda", via_oracle)
    want = L.quantize_liqk_v2_diag_rot(W, dh, "TEST_BANK")
    assert torch.equal(got, want)
    monkeypatch.setenv("LIQK_PROFILE_CUDA", "0")
    torch_path = L.quantize_liqk_v2_diag_rot(W, dh, "TEST_BANK")
    assert torch_path.shape == got.shape and torch.isfinite(torch_path).all()
    # the two bucket roundings (fused vs separate multiply-add) rarely differ; the profiles agree closely
    assert (torch_path == got).float().mean().item() > 0.99
    with pytest.raises(KeyError):
        L.get_warp_register_bank("NO_SUCH_BANK", cuda_dev)
