"""GPU: the concurrent multi-matrix driver (ltq_research_b200.batch.quantize_matrices) gives, for every matrix, the
same bits as quantize_matrix_liqk_v2 run alone (PACK fields, scales, W_hat) and the same relative loss."""
import pytest
import torch

from tests.golden.matrix_inputs import synth

pytestmark = pytest.mark.gpu

JOBS = [(64, 512, "TCQ3X", 21), (128, 768, "TCQ25X", 22), (32, 512, "TCQ275X2", 23), (96, 256, "TCQ4X", 24),
        (64, 512, [(0, 32, "TCQ3X"), (32, 64, "TCQ45X")], 25), (48, 1024, "TCQ2X", 26)]


def test_quantize_matrices_equals_one_at_a_time(cuda_dev):
    import ltq_research_b200.liqk_v2 as L
    from ltq_research_b200.batch import quantize_matrices
    inputs = []
    for M, K, spec, seed in JOBS:
        W, H = synth(M, K, seed)
        inputs.append((W.to(cuda_dev), H.to(cuda_dev), spec))
    ref = []
    for W, H, spec in inputs:
        L.PACK = {}
        try:
            q, w_hat, rel = L.quantize_matrix_liqk_v2(W, H, spec, seed=1337, damp=0.02)
            ref.append((q, w_hat, rel, dict(L.PACK["matrix"])))
        finally:
            L.PACK = None
    got = quantize_matrices(inputs, seed=1337, damp=0.02, n_streams=4, pack=True, keep_w_hat=True)
    # host inputs (copied to the device on the matrices' streams) give the same results
    got_h = quantize_matrices([(W.cpu().pin_memory(), H.cpu().pin_memory(), sp) for W, H, sp in inputs], n_streams=3)
    for i, ((q, w_hat, rel, pm), g, gh) in enumerate(zip(ref, got, got_h)):
        assert g["rel_loss"] == rel and gh["rel_loss"] == rel, i
        assert torch.equal(g["W_hat"], w_hat), i
        assert torch.equal(g["qdata"]["d"], q["d"]) and torch.equal(g["qdata"]["suh"], q["suh"]), i
        for k in ("idx", "gi", "G", "d_row", "e", "suh"):
            assert torch.equal(g["pack"][k], pm[k]), (i, k)
            assert torch.equal(gh["pack"][k], pm[k]), (i, k)


def test_quantize_matrices_rejects_non_positive_hessian(cuda_dev):
    from ltq_research_b200.batch import quantize_matrices
    W, H = synth(32, 256, 3)
    H = -torch.eye(256) * 1e3  # negative definite even after damping
    with pytest.raises(torch.linalg.LinAlgError):
        quantize_matrices([(W.to(cuda_dev), H.to(cuda_dev), "TCQ3X")])
