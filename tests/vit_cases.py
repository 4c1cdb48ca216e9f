"""Seeded Viterbi parity cases shared by the CPU oracle tests and the GPU parity tests.

Each case is (name, kwargs, x, wts) where kwargs are the keyword arguments of `viterbi_ub_cuda`
(src/tcq_proto.py:567-573) except x / wts / small / gains, which are numpy arrays in the case ("small", "gains",
"small_hi", "gains_hi").  Gains come from the format table's float32 values (fixture), the same numbers on both sides.
"""
from __future__ import annotations

import json
from pathlib import Path

import numpy as np

GOLDEN = Path(__file__).resolve().parent / "golden"
FORMATS = json.loads((GOLDEN / "formats.json").read_text())
MENU = FORMATS["menu_TCQPQ"]
F = FORMATS["formats"]


def fmt_kwargs(name: str) -> dict:
    c = F[name]
    return dict(K=c["K"], nu=10, m=c["m"], sub=c["sub"], n_cand=c["n_cand"], m_extra=tuple(c["m_extra"]),
                pair_parity=c["pp"], small=np.asarray(c["lut"], np.float32),
                gains=np.asarray(c["gains_cpu"], np.float32))


def _x(rng, N, T, scale=1.0):
    return (rng.standard_normal((N, T)) * scale).astype(np.float32)


def menu_tb_cases(N=24, L=256, seed=0, window=0, weighted=False):
    """The reference self-test shape: every TCQPQ format, tail-biting, candidates as configured (src/ltq_format.py:150-181)."""
    out = []
    for i, name in enumerate(MENU):
        c = F[name]
        if L != 256 and c["sub"] != 16:
            continue
        rng = np.random.default_rng(seed * 1000 + i)
        kw = fmt_kwargs(name)
        kw.update(tail_biting=True, return_code=True, tb_window=window)
        x = _x(rng, N, L)
        wts = (rng.uniform(0.2, 3.0, L).astype(np.float32) if weighted else None)
        out.append((f"{name}_L{L}_w{window}{'_wt' if weighted else ''}", kw, x, wts))
    return out


def special_cases(N=16, seed=7):
    rng = np.random.default_rng(seed)
    out = []
    g1 = F["_config1_tcq_K2_h2"]
    kw = dict(K=2, nu=10, m=359, sub=16, small=np.asarray(g1["lut"], np.float32),
              gains=np.asarray(g1["gains_cpu"], np.float32), tail_biting=True, return_code=True)
    out.append(("config1_gauss_k2h2", kw, _x(rng, N, 256), None))
    # LDLQ-style calls: per-position weights repeated per row, tail-biting with the 32-sample first-pass window
    for name in ("TCQ3X", "TCQ25X", "TCQ275X2", "TCQ5X", "TCQ2X", "TCQ4W3"):
        kw = fmt_kwargs(name)
        kw.update(tail_biting=True, tb_window=32, return_code=True)
        dw = rng.uniform(0.05, 4.0, 16).astype(np.float32)
        out.append((f"ldlq_{name}", kw, _x(rng, N, 256, 1.3), np.tile(dw, 16)))
    # per-tile weights [N, T]
    kw = fmt_kwargs("TCQ35X")
    kw.update(tail_biting=True, return_code=True)
    out.append(("tileweights_TCQ35X", kw, _x(rng, N, 256), rng.uniform(0.0, 2.0, (N, 256)).astype(np.float32)))
    # carried start state, end state returned (reference "carry" mode); plain, D2 and D4
    for name in ("TCQ3X", "TCQ35X", "TCQ375X", "TCQ2X0"):
        kw = fmt_kwargs(name)
        kw.update(return_end_state=True)
        kw["init_state"] = rng.integers(-1, 1024, N).astype(np.int32)
        out.append((f"carry_{name}", kw, _x(rng, N, 256), None))
    # tail-biting extras: three passes, cheap first pass over fewer candidates
    kw = fmt_kwargs("TCQ4X")
    kw.update(tail_biting=True, tb_passes=3, return_code=True)
    out.append(("tb3_TCQ4X", kw, _x(rng, N, 256), None))
    kw = fmt_kwargs("TCQ5X")
    kw.update(tail_biting=True, tb_cand1=2, return_code=True)
    out.append(("tbcand1_TCQ5X", kw, _x(rng, N, 256), None))
    # masks that have no compiled-in instantiation (run-time masks), 4 / 8 / 16 subsets
    for me, K in (((), 3), ((123,), 3), ((77, 301), 2)):
        nl = 4 << len(me)
        U = 1 << (K - 1)
        q = np.sort(rng.standard_normal(nl * U)).astype(np.float32)
        small = q.reshape(U, nl).T.copy().reshape(-1)
        kw = dict(K=K, nu=10, m=299 if not me else 359, sub=16, small=small,
                  gains=np.asarray(F["TCQ3X"]["gains_cpu"], np.float32), m_extra=me, tail_biting=True,
                  return_code=True)
        out.append((f"rtmask_nl{nl}", kw, _x(rng, N, 256), None))
    # run-time masks with D2 / D4 / EQ
    for pp in (1, 2, 3):
        c = F["TCQ275X"]
        kw = dict(K=3, nu=10, m=359, sub=16, small=np.asarray(c["lut"], np.float32),
                  gains=np.asarray(c["gains_cpu"], np.float32), m_extra=(99,), pair_parity=pp, tail_biting=True,
                  return_code=True)
        out.append((f"rtmask_pp{pp}", kw, _x(rng, N, 256), None))
    # EQ formats (K + 0.25 menu, src/equal_bpw.py:71-72)
    for name in ("TCQ225X", "TCQ325X"):
        kw = fmt_kwargs(name)
        kw.update(tail_biting=True, return_code=True)
        out.append((f"eq_{name}", kw, _x(rng, N, 256), None))
    # half-integer rate: positions with (t // mix) odd use a K + 1 table and their own gains
    c2, c3 = F["TCQ3X1"], F["TCQ4X1"]
    kw = dict(K=3, nu=10, m=359, sub=16, small=np.asarray(c2["lut"], np.float32)[:16],
              gains=np.asarray(c2["gains_cpu"], np.float32), small_hi=np.asarray(c3["lut"], np.float32),
              gains_hi=np.asarray(c3["gains_cpu"], np.float32), mix=16, tail_biting=True, return_code=True)
    out.append(("halfint_mix16", kw, _x(rng, N, 256), None))
    # all 8 gains without candidates (G = 8), and G = 3 via candidates
    c = F["TCQ4X"]
    kw = dict(K=4, nu=10, m=359, sub=16, small=np.asarray(c["lut"], np.float32),
              gains=np.asarray(c["gains_cpu"], np.float32), tail_biting=True, return_code=True)
    out.append(("g8_nocand", kw, _x(rng, N, 256), None))
    kw = dict(kw, n_cand=3)
    out.append(("g3_cand", kw, _x(rng, N, 256), None))
    # sub-blocks of 6 (not a multiple of 4): plain and D2, T = 96
    c = F["TCQ3X1"]
    kw = dict(K=3, nu=10, m=359, sub=6, small=np.asarray(c["lut"], np.float32), m_extra=(241,),
              gains=np.asarray(c["gains_cpu"], np.float32), tail_biting=True, return_code=True)
    out.append(("sub6_plain", kw, _x(rng, N, 96), None))
    kw = dict(kw, pair_parity=1)
    out.append(("sub6_d2", kw, _x(rng, N, 96), None))
    # no gains (h = 0, one slot), rings of 160
    kw = fmt_kwargs("TCQ2X0")
    kw.update(tail_biting=True, return_code=True)
    out.append(("h0_ring160", kw, _x(rng, N, 160), None))
    return out


def direct_cases(N=16, seed=11):
    """Single passes with the private schedule arguments (_mid / _steps / _rot / _tail) of viterbi_ub_cuda."""
    rng = np.random.default_rng(seed)
    out = []
    for name in ("TCQ3X", "TCQ35X", "TCQ375X"):
        kw = fmt_kwargs(name)
        x = _x(rng, N, 256)
        out.append((f"mid_window_{name}", dict(kw, _mid=32, _steps=64, _rot=96), x, None))
        out.append((f"mid_full_{name}", dict(kw, _mid=128), x, None))
        init = rng.integers(0, 1024, N).astype(np.int32)
        out.append((f"tail_rot_{name}", dict(kw, init_state=init, _tail=True, _rot=128, return_code=True), x, None))
    return out


def nl32_cases(N=12, seed=31):
    """32 label subsets (three extra masks; no format of the tables uses them, the reference kernel accepts them): the
    run-time-mask kernel in the plain, D2 and D4 modes, with gain candidates, and a single carried pass."""
    rng = np.random.default_rng(seed)
    me = (77, 301, 123)
    out = []

    def table(K):
        U = 1 << (K - 1)
        q = np.sort(rng.standard_normal(32 * U)).astype(np.float32)
        return q.reshape(U, 32).T.copy().reshape(-1)
    g4 = np.asarray(F["TCQ3X"]["gains_cpu"], np.float32)
    g8 = np.asarray(F["TCQ4X"]["gains_cpu"], np.float32)
    base = dict(nu=10, m=359, sub=16, m_extra=me, tail_biting=True, return_code=True)
    out.append(("nl32_plain", dict(base, K=2, small=table(2), gains=g4), _x(rng, N, 256), None))
    for pp in (1, 2):
        out.append((f"nl32_pp{pp}", dict(base, K=3, small=table(3), gains=g4, pair_parity=pp), _x(rng, N, 256), None))
    out.append(("nl32_cand2of8", dict(base, K=3, small=table(3), gains=g8, n_cand=2, tb_window=32),
                _x(rng, N, 256), rng.uniform(0.2, 3.0, 256).astype(np.float32)))
    init = rng.integers(0, 1024, N).astype(np.int32)
    out.append(("nl32_carry", dict(K=2, nu=10, m=359, sub=16, m_extra=me, small=table(2), gains=g4, init_state=init,
                                   return_end_state=True), _x(rng, N, 256), None))
    return out


def s256_cases(N=12, seed=41):
    """The 256-state trellis (nu = 8; 4 subsets, plain mode, as the reference's table allows): tail-biting with and
    without the first-pass window, gain candidates, all 8 gains, half-integer tables, a carried pass and a middle-state
    pass."""
    rng = np.random.default_rng(seed)

    def table(K):
        U = 1 << (K - 1)
        q = np.sort(rng.standard_normal(4 * U)).astype(np.float32)
        return q.reshape(U, 4).T.copy().reshape(-1)
    g4 = np.asarray(F["TCQ3X"]["gains_cpu"], np.float32)
    g8 = np.asarray(F["TCQ4X"]["gains_cpu"], np.float32)
    base = dict(nu=8, m=91, sub=16, tail_biting=True, return_code=True)
    out = [("s256_k2", dict(base, K=2, small=table(2), gains=g4), _x(rng, N, 256), None),
           ("s256_k3_window", dict(base, K=3, small=table(3), gains=g4, tb_window=32), _x(rng, N, 256),
            rng.uniform(0.2, 3.0, 256).astype(np.float32)),
           ("s256_g8", dict(base, K=3, small=table(3), gains=g8), _x(rng, N, 256), None),
           ("s256_cand3of8", dict(base, K=3, small=table(3), gains=g8, n_cand=3), _x(rng, N, 256), None)]
    c2, c3 = F["TCQ3X1"], F["TCQ4X1"]
    out.append(("s256_mix16", dict(base, K=3, m=45, small=np.asarray(c2["lut"], np.float32)[:16],
                                   gains=np.asarray(c2["gains_cpu"], np.float32),
                                   small_hi=np.asarray(c3["lut"], np.float32)[:32],
                                   gains_hi=np.asarray(c3["gains_cpu"], np.float32), mix=16), _x(rng, N, 256), None))
    init = rng.integers(0, 256, N).astype(np.int32)
    out.append(("s256_carry", dict(K=2, nu=8, m=91, sub=16, small=table(2), gains=g4, init_state=init,
                                   return_end_state=True), _x(rng, N, 256), None))
    out.append(("s256_mid", dict(K=3, nu=8, m=91, sub=16, small=table(3), gains=g4, _mid=128), _x(rng, N, 256), None))
    return out
