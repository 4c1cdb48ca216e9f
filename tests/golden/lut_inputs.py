"""Seeded inputs of the DP-profile table quantizer (lut_subs_quant, src/cuda/tcq_viterbi.cu:768-811), rebuilt
identically from numpy wherever the tests run, so only the reference kernel's outputs are stored
(tests/golden/lut_subs.npz, made by tests/golden/make_golden_lut.py).

The table imitates a trained bank's (src/liqk_v2.py:394-396): bucket centres z_b = linspace(-max_g, max_g, nb), each of
the 64 columns the nearest point of a uniform grid of its own spacing; columns 10 and 11 are equal (ties between
candidates).  max_g = 1023 / 256 with nb = 1024 makes inv_step = 128 a power of two, so x = (k - 511) / 128 lands exactly
on bucket boundaries k + 0.5 (round-half-even cases).  The inputs also cover clamping at both ends, zero weights, and
sub-blocks holding a NaN or an infinity."""
import numpy as np

NB = 1024
MAX_G = 1023.0 / 256.0
INV_STEP = np.float32((NB - 1) / (2.0 * MAX_G))
HALF_B = np.float32((NB - 1) * 0.5)


def table(nb: int = NB, max_g: float = MAX_G) -> np.ndarray:
    z = np.linspace(-max_g, max_g, nb, dtype=np.float32)
    lut = np.empty((nb, 64), dtype=np.float32)
    for c in range(64):
        s = np.float32(0.05 + 0.013 * c)
        lut[:, c] = np.clip(np.round(z / s) * s, -max_g, max_g).astype(np.float32)
    lut[:, 11] = lut[:, 10]
    return lut


def case(S: int = 2048, seed: int = 3):
    g = np.random.default_rng(seed)
    xs = (g.standard_normal((S, 16)) * 1.6).astype(np.float32)
    dh = g.uniform(0.05, 2.0, (S, 16)).astype(np.float32)
    # exact bucket boundaries (round half to even) and exact centres
    k = g.integers(0, NB - 1, (64, 16))
    xs[:64] = ((k - 511) / 128.0).astype(np.float32)
    xs[64:96] = ((g.integers(0, NB, (32, 16)) - 511.5) / 128.0).astype(np.float32)
    # far outside the table on both sides (clamped buckets)
    xs[96:104] = (g.standard_normal((8, 16)) * 50).astype(np.float32)
    dh[104:112] = 0.0                       # all errors 0: candidate 0
    dh[112:120, ::2] = 0.0
    xs[120, 3] = np.nan
    xs[121, 0] = np.inf
    xs[122, 15] = -np.inf
    dh[123, 5] = np.nan
    return xs, dh, table(), float(INV_STEP), float(HALF_B)
