"""The reference's own Python driven through the B200 library, and this package's matrix quantizer at config-2 sizes
against the reference's quantize_matrix_liqk_v2 run on the same GPU.

Needs the reference's install in baseline/_ref (`make -C oracle refpy LTQ_REF_ROOT=...`) and the reference kernel built
from its own source (oracle/_ref, `make -C oracle ref`); skipped without them.  The reference is never modified: its
ctypes binding `_TCQ_LIB` (src/tcq_proto.py:514-533) is pointed at one library or the other, exactly as a maintainer
would rebind it.

* The reference's self-test (src/ltq_format.py:148-181) through libltq_b200.so: 0 label / fractional-mode / decode
  mismatches for all 19 tile formats (L = 256) and 17 ring formats (L = 160), as recorded in
  results/ltq_format_selftest.json.
* The reference's viterbi_ub_cuda (its scratch allocation, tail-biting schedule and code unpacking,
  src/tcq_proto.py:567-657) on the same inputs through the reference kernel and through libltq_b200.so: identical
  reconstructions and codes for every format of the menu, full and windowed first passes, with position weights.
* The reference's quantize_matrix_liqk_v2 (src/liqk_v2.py:1029-1198) at config-2 shapes (3072 x 3072 TCQ3X,
  1024 x 3072 TCQ25X, seeded inputs with the config's distributions) with the reference kernel and with
  libltq_b200.so as its Viterbi: identical .ltq fields (codes, gain indices, tile values, d_row, e, suh), W_hat and loss.
* This package's own pipeline against that reference run, same inputs, same GPU: gemm "fp32" (quantize_matrix_liqk_v2)
  bit for bit; the benched fast mode (batch.quantize_matrices, bf16x6 tensor-core products) within the bounds written
  in its test.  The statistics (code agreement, per-tile-group H-weighted error relative differences, rel_loss) go to
  $LTQ_REPORT_DIR/parity_<case>.json when that variable is set.
"""
from __future__ import annotations

import ctypes
import json
import os
from pathlib import Path

import numpy as np
import pytest
import torch

from oracle import ref_kernel
from oracle.refroot import import_reference, reference_root
from tests.golden.matrix_inputs import synth

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(reference_root() is None or not ref_kernel.available(),
                                 reason="reference install (baseline/_ref) or reference kernel (oracle/_ref) missing")]

# the four distinct matrix shapes of the config-2 layer (q / o, k / v, gate / up, down), both formats of the bench
CONFIG2 = [("q3072x3072_TCQ3X", 3072, 3072, "TCQ3X", 11), ("k1024x3072_TCQ25X", 1024, 3072, "TCQ25X", 12),
           ("gate8192x3072_TCQ25X", 8192, 3072, "TCQ25X", 13), ("down3072x8192_TCQ3X", 3072, 8192, "TCQ3X", 14)]


@pytest.fixture(scope="module")
def ref(cuda_dev):
    import_reference()
    import src.liqk_v2 as lv2
    import src.ltq_format as lf
    import src.tcq_proto as tp
    return tp, lf, lv2


def _bind(tp, so: Path):
    """The reference's ctypes binding (src/tcq_proto.py:527-532) over library `so`."""
    L = ctypes.CDLL(str(so))
    L.tcq_viterbi.restype = ctypes.c_int
    L.tcq_viterbi.argtypes = [ctypes.c_void_p] * 15 + [ctypes.c_int] * 18 + [ctypes.c_void_p, ctypes.c_int,
                                                                              ctypes.c_void_p]
    L.lut_subs_quant.restype = ctypes.c_int
    L.lut_subs_quant.argtypes = [ctypes.c_void_p] * 4 + [ctypes.c_int, ctypes.c_float, ctypes.c_float, ctypes.c_int,
                                                         ctypes.c_void_p]
    tp._TCQ_LIB = L
    return L


def _ours():
    from ltq_research_b200 import _lib
    return _lib.LIB_PATH


def _report(name: str, stats: dict):
    d = os.environ.get("LTQ_REPORT_DIR")
    if d:
        Path(d).mkdir(parents=True, exist_ok=True)
        Path(d, f"parity_{name}.json").write_text(json.dumps(stats, indent=1))


def test_reference_self_test_through_b200_library(ref, monkeypatch):
    tp, lf, _ = ref
    monkeypatch.setattr(tp, "_TCQ_LIB", None)
    _bind(tp, _ours())
    tiles = lf.self_test()
    rings = lf.self_test(n_tiles=256, L=160)
    assert len(tiles) == 19 and len(rings) == 17
    for res in (tiles, rings):
        for name, r in res.items():
            assert (r["label_mismatch"], r["frac_violations"], r["decode_mismatch"]) == (0, 0, 0), (name, r)


@pytest.mark.parametrize("window", [0, 32])
def test_reference_wrapper_same_bits_on_both_libraries(ref, monkeypatch, cuda_dev, window):
    tp, lf, lv2 = ref
    from src.equal_bpw import SETS
    fmts = lf.load_formats(SETS["TCQPQ"])
    g = torch.Generator(device=cuda_dev).manual_seed(100 + window)
    monkeypatch.setattr(tp, "_TCQ_LIB", None)
    for name, f in fmts.items():
        x = torch.randn(96, 256, device=cuda_dev, generator=g) * 1.3
        w = torch.rand(256, device=cuda_dev, generator=g) + 0.25
        kw = dict(sub=f.sub, wts=w, return_code=True, tail_biting=True, tb_window=window, m_extra=f.masks[1:],
                  pair_parity=f.frac, n_cand=lv2.TCQ_CONFIG[name].get("n_cand", 0))
        lut, gains = torch.tensor(f.lut, device=cuda_dev), torch.tensor(f.gain_tab, device=cuda_dev)
        outs = []
        for so in (ref_kernel.REF_SO, _ours()):
            _bind(tp, so)
            outs.append([t.cpu() for t in tp.viterbi_ub_cuda(x, lut, f.K, 10, f.masks[0], gains, **kw)])
        for a, b in zip(*outs):
            assert torch.equal(a.view(torch.int32) if a.dtype == torch.float32 else a,
                               b.view(torch.int32) if b.dtype == torch.float32 else b), name


def _ref_quantize(ref, so: Path, W, H, spec):
    """The reference's quantize_matrix_liqk_v2 with PACK on, its Viterbi bound to library `so`."""
    tp, _, lv2 = ref
    _bind(tp, so)
    lv2.PACK = {"groups": []}
    try:
        _, w_hat, rel = lv2.quantize_matrix_liqk_v2(W, H, spec, seed=1337, damp=0.02)
        pm = dict(lv2.PACK["matrix"])
    finally:
        lv2.PACK = None
    torch.cuda.synchronize()
    return pm, w_hat, rel


@pytest.fixture(scope="module")
def ref_runs(ref, cuda_dev):
    """Per config-2 case: inputs and the reference run with the reference kernel (computed once)."""
    tp = ref[0]
    keep = tp._TCQ_LIB
    out = {}
    try:
        for name, M, K, spec, seed in CONFIG2:
            W, H = synth(M, K, seed, device=cuda_dev)
            out[name] = (W, H, spec, _ref_quantize(ref, ref_kernel.REF_SO, W, H, spec))
    finally:
        tp._TCQ_LIB = keep
    return out


@pytest.mark.parametrize("case", [c[0] for c in CONFIG2])
def test_reference_pipeline_same_bits_on_both_libraries(ref, ref_runs, case):
    tp = ref[0]
    keep = tp._TCQ_LIB
    W, H, spec, (pm0, wh0, rel0) = ref_runs[case]
    try:
        pm1, wh1, rel1 = _ref_quantize(ref, _ours(), W, H, spec)
    finally:
        tp._TCQ_LIB = keep
    for k in ("idx", "gi", "G", "d_row", "e", "suh"):
        a, b = pm0[k], pm1[k]
        assert torch.equal(a.view(torch.int32) if a.dtype == torch.float32 else a,
                           b.view(torch.int32) if b.dtype == torch.float32 else b), (case, k)
    assert torch.equal(wh0.view(torch.int32), wh1.view(torch.int32)) and rel0 == rel1, case


def _group_losses(W, w_hat, H):
    """Per 16-row tile group: sum over its rows of (w - w_hat) H (w - w_hat)^T, in fp64."""
    D = W.double() - w_hat.double()
    per_row = ((D @ H.double()) * D).sum(dim=1)
    return per_row.view(-1, 16).sum(dim=1)


def _compare(name, mode, W, H, ref_pm, ref_wh, ref_rel, pm, w_hat, rel) -> dict:
    lr = _group_losses(W, ref_wh, H)
    lo = _group_losses(W, w_hat, H)
    rd = ((lo - lr).abs() / lr.clamp(min=1e-300)).cpu().numpy()
    s = {"case": name, "mode": mode,
         "codes_equal": float((pm["idx"] == ref_pm["idx"]).float().mean()),
         "gain_index_equal": float((pm["gi"] == ref_pm["gi"]).float().mean()),
         "tile_values_equal": float((pm["G"] == ref_pm["G"]).float().mean()),
         "d_row_equal": float((pm["d_row"] == ref_pm["d_row"]).float().mean()),
         "e_equal": float((pm["e"] == ref_pm["e"]).float().mean()),
         "suh_equal": float((pm["suh"] == ref_pm["suh"]).float().mean()),
         "rel_loss": rel, "rel_loss_ref": ref_rel, "rel_loss_rel_diff": abs(rel - ref_rel) / ref_rel,
         "tile_group_wmse_rel_diff": {"median": float(np.median(rd)), "p99": float(np.quantile(rd, 0.99)),
                                      "max": float(rd.max()), "frac_within_1e-6": float((rd <= 1e-6).mean())},
         "tile_group_wmse_mean_rel_diff": float((lo.sum() - lr.sum()).abs() / lr.sum())}
    _report(f"{name}_{mode}", s)
    return s


@pytest.mark.parametrize("case", [c[0] for c in CONFIG2])
def test_fp32_pipeline_against_reference_run(ref_runs, case):
    """gemm "fp32" — the reference's torch operations for the rotation statistics, factorisation, scale fit, inter-block
    update and refits; this package's kernels for the FWHT, the Viterbi and the fused LDLQ block (intra-block feedback
    as sequential fma chains): bit for bit the reference run on the same GPU — every .ltq field, W_hat, the loss, so
    every tile group's H-weighted error is equal (relative difference 0, within north_star's 1e-6)."""
    import ltq_research_b200.liqk_v2 as L
    W, H, spec, (pm0, wh0, rel0) = ref_runs[case]
    L.PACK = {}
    try:
        _, w_hat, rel = L.quantize_matrix_liqk_v2(W, H, spec, seed=1337, damp=0.02)
        pm = dict(L.PACK["matrix"])
    finally:
        L.PACK = None
    s = _compare(case, "fp32", W, H, pm0, wh0, rel0, pm, w_hat, rel)
    for k in ("idx", "gi", "G", "d_row", "e", "suh"):
        a, b = pm0[k], pm[k]
        assert torch.equal(a.view(torch.int32) if a.dtype == torch.float32 else a,
                           b.view(torch.int32) if b.dtype == torch.float32 else b), (k, s)
    assert torch.equal(w_hat.view(torch.int32), wh0.view(torch.int32)) and rel == rel0, s
    assert s["tile_group_wmse_rel_diff"]["max"] == 0.0, s


@pytest.mark.parametrize("case", [c[0] for c in CONFIG2])
def test_fast_pipeline_against_reference_run(ref_runs, case):
    """The benched mode (batch.quantize_matrices: bf16x6 tensor-core products accurate to fp32's error bound, blocked
    tensor-core Cholesky, scale-fit kernel) against the reference run.  Its products round differently from cuBLAS's
    fp32 GEMMs in the last bits; where that moves a Viterbi decision near a tie, the LDLQ feedback carries the change
    along the row (the longer the row, the more: K = 8192 diverges most), so this mode is compared statistically:
    codes >= 97 % equal, rel_loss within 1e-3 relative, the summed H-weighted error of the tile groups within 1e-3,
    >= 90 % of tile groups' H-weighted error within 1e-6 of the reference's (measured on a B200 at the four shapes:
    codes 98.1-100 % equal, rel_loss within 1.1e-4, tile groups within 1e-6: 92.7-100 %)."""
    from ltq_research_b200.batch import quantize_matrices
    W, H, spec, (pm0, wh0, rel0) = ref_runs[case]
    r = quantize_matrices([(W, H, spec)], keep_w_hat=True, gemm="bf16x6")[0]
    s = _compare(case, "bf16x6", W, H, pm0, wh0, rel0, r["pack"], r["W_hat"], r["rel_loss"])
    assert s["codes_equal"] >= 0.97, s
    assert s["rel_loss_rel_diff"] < 1e-3, s
    assert s["tile_group_wmse_mean_rel_diff"] < 1e-3, s
    assert s["tile_group_wmse_rel_diff"]["frac_within_1e-6"] >= 0.90, s
