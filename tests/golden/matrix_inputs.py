"""Seeded synthetic inputs of the matrix-quantizer fixtures (shared by tests/golden/make_golden_matrix.py and the GPU
parity tests): bf16 Student-t(5) * 0.02 weights with 0.5 % of input channels x 20, and H = X^T X / n of n = 4K Gaussian
activation rows with log-normal(0, 1) per-channel scales (the BASELINE config-2 distributions at small sizes)."""
import torch

CASES = [
    # name, M, K, spec (or row slices), seed
    ("m64k512_TCQ3X", 64, 512, "TCQ3X", 1),
    ("m64k512_TCQ25X", 64, 512, "TCQ25X", 2),
    ("m32k512_TCQ275X2", 32, 512, "TCQ275X2", 3),
    ("m32k512_TCQ4X", 32, 512, "TCQ4X", 4),
    ("m32k768_TCQ2X", 32, 768, "TCQ2X", 5),
    ("m32k512_TCQ4W2", 32, 512, "TCQ4W2", 6),
    ("m64k512_slices", 64, 512, [(0, 32, "TCQ3X"), (32, 64, "TCQ45X")], 7),
]


# the earlier, non-tail-biting formats (no .ltq encoding): carry R formats, half-integer rows, gain candidates, the
# block-scale refit, and two of them in one matrix
LEGACY_CASES = [
    ("m32k512_TCQ3R", 32, 512, "TCQ3R", 11),
    ("m32k512_TCQ25R", 32, 512, "TCQ25R", 12),
    ("m32k512_TCQ4RH3", 32, 512, "TCQ4RH3", 13),
    ("m32k512_TCQ3", 32, 512, "TCQ3", 14),
    ("m64k512_TCQ2R_TCQ4", 64, 512, [(0, 32, "TCQ2R"), (32, 64, "TCQ4")], 15),
]


def synth(M: int, K: int, seed: int, device="cpu"):
    """(W bf16 [M, K], H fp32 [K, K]) from a generator on `device` (the values depend on the device's generator)."""
    g = torch.Generator(device=device).manual_seed(seed)
    z = torch.randn(M, K, generator=g, device=device)
    chi2 = torch.randn(M, K, 5, generator=g, device=device).square().sum(-1)   # Student-t(5) = N(0,1) / sqrt(chi2_5 / 5)
    W = z / (chi2 / 5).sqrt() * 0.02
    n_out = max(1, int(round(0.005 * K)))
    cols = torch.randperm(K, generator=g, device=device)[:n_out]
    W[:, cols] *= 20
    W = W.to(torch.bfloat16)
    X = torch.randn(4 * K, K, generator=g, device=device) * torch.exp(torch.randn(1, K, generator=g, device=device))
    H = (X.T @ X) / X.shape[0]
    return W, H
