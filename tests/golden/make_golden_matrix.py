"""Golden fixtures of the matrix quantizer: the reference's quantize_matrix_liqk_v2 (src/liqk_v2.py:1029-1198, TCQ
formats, PACK mode) run from the reference tree on CPU, with its CUDA-only viterbi_ub_cuda replaced by the CPU oracle
(oracle/oracle.py, pinned bit for bit against the reference kernel).  Synthetic seeded inputs shaped like the BASELINE
configs (bf16 Student-t(5) * 0.02 weights with 0.5 % outlier input channels x 20, H = X^T X of log-normal-scaled
Gaussian activations).

    PYTHONDONTWRITEBYTECODE=1 TCQ_NO_COMPILE=1 python tests/golden/make_golden_matrix.py [--legacy]

--legacy: the earlier non-tail-biting formats (LEGACY_CASES) -> matrix_quant_legacy.npz.
"""
from __future__ import annotations

import json
import sys
from pathlib import Path

import numpy as np

OUT = Path(__file__).resolve().parent
ROOT = OUT.parent.parent
sys.path.insert(0, str(ROOT))
from oracle.refroot import import_reference  # noqa: E402

REF = import_reference()  # the tree named by LTQ_REF_ROOT, else the install in baseline/_ref

import torch  # noqa: E402

import src.liqk_v2 as lv2  # noqa: E402
import src.tcq_proto as tp  # noqa: E402
from oracle import oracle as O  # noqa: E402
from tests.golden.matrix_inputs import CASES, LEGACY_CASES, synth  # noqa: E402


def oracle_viterbi_ub_cuda(x, small, K, nu, m, gains=None, **kw):
    """viterbi_ub_cuda's contract on torch CPU tensors, computed by the oracle."""
    def np_(t):
        return None if t is None else (t.detach().cpu().numpy() if torch.is_tensor(t) else t)
    for k in ("wts", "init_state", "small_hi", "gains_hi"):
        if k in kw:
            kw[k] = np_(kw[k])
    out = O.viterbi(np_(x), np_(small), K, nu, m, np_(gains), **kw)
    if isinstance(out, tuple):
        return tuple(torch.from_numpy(np.ascontiguousarray(o)) for o in out)
    return torch.from_numpy(out)


captured = []


def main():
    tp.viterbi_ub_cuda = oracle_viterbi_ub_cuda
    orig_rows = lv2._quantize_rows_tcq_ldlq

    def rows_hook(W_rot, *a, **k):  # records each row group's pre-refit d_row (fp16-rounded, as fp32)
        out = orig_rows(W_rot, *a, **k)
        captured.append(lv2.PACK["groups"][-1]["d_row"].clone())
        return out
    lv2._quantize_rows_tcq_ldlq = rows_hook
    arrays, meta = {}, []
    for name, M, K, spec, seed in CASES:
        W, H = synth(M, K, seed)
        captured.clear()
        specs = [(0, M, spec)] if isinstance(spec, str) else spec
        by = {}
        for r0, r1, sp in specs:
            by.setdefault(sp, []).append(torch.arange(r0, r1))
        group_rows = [torch.cat(v) for v in by.values()]  # the order quantize_matrix_liqk_v2 visits the groups
        lv2.PACK = {}
        q, w_hat, rel = lv2.quantize_matrix_liqk_v2(W, H, spec, seed=1337, damp=0.02)
        pm = lv2.PACK["matrix"]
        arrays[f"{name}/w_hat_norm"] = np.array([float(w_hat.norm())])
        # before the refits: the rotation's suh (compute_optimal_suh) and the rows' scale fit (PACK groups)
        _, _, suh0 = lv2.compute_optimal_suh(W.float(), H.float(), seed=1337)
        arrays[f"{name}/suh0"] = suh0.to(torch.float16).view(torch.int16).numpy()
        d0 = torch.zeros(M)
        for rows, dr in zip(group_rows, captured):
            d0[rows] = dr
        arrays[f"{name}/d_row0"] = d0.numpy()
        for k in ("idx", "gi", "e"):
            arrays[f"{name}/{k}"] = pm[k].numpy()
        arrays[f"{name}/d_row"] = pm["d_row"].view(torch.int16).numpy()
        arrays[f"{name}/suh"] = pm["suh"].view(torch.int16).numpy()
        meta.append({"name": name, "M": M, "K": K, "spec": spec, "rel_loss": rel})
        print(name, "rel_loss", rel, flush=True)
    lv2.PACK = None
    arrays["meta"] = np.frombuffer(json.dumps(meta).encode(), dtype=np.uint8)
    np.savez_compressed(OUT / "matrix_quant.npz", **arrays)
    print((OUT / "matrix_quant.npz").stat().st_size, "bytes")


def legacy_main():
    """The earlier formats (no PACK mode in the reference for them): per case the row groups' d_full and W_hat_rot
    before the refits (recorded at _quantize_rows_tcq_ldlq), and the returned d, suh and rel_loss ->
    matrix_quant_legacy.npz."""
    tp.viterbi_ub_cuda = oracle_viterbi_ub_cuda
    orig_rows = lv2._quantize_rows_tcq_ldlq
    rec = []

    def rows_hook(W_rot, *a, **k):
        d_sub, wh = orig_rows(W_rot, *a, **k)
        rec.append((d_sub.clone(), wh.clone()))
        return d_sub, wh
    lv2._quantize_rows_tcq_ldlq = rows_hook
    arrays, meta = {}, []
    for name, M, K, spec, seed in LEGACY_CASES:
        W, H = synth(M, K, seed)
        rec.clear()
        specs = [(0, M, spec)] if isinstance(spec, str) else spec
        by = {}
        for r0, r1, sp in specs:
            by.setdefault(sp, []).append(torch.arange(r0, r1))
        d0 = torch.zeros((M, K // 256), dtype=torch.float16)
        wh0 = torch.zeros((M, K))
        q, w_hat, rel = lv2.quantize_matrix_liqk_v2(W, H, spec, seed=1337, damp=0.02)
        for rows, (d_sub, wh) in zip([torch.cat(v) for v in by.values()], rec):
            d0[rows], wh0[rows] = d_sub, wh
        arrays[f"{name}/d0"] = d0.view(torch.int16).numpy()
        arrays[f"{name}/w_hat_rot0"] = wh0.numpy()
        arrays[f"{name}/d"] = q["d"].view(torch.int16).numpy()
        arrays[f"{name}/suh"] = q["suh"].view(torch.int16).numpy()
        meta.append({"name": name, "M": M, "K": K, "spec": spec, "rel_loss": rel})
        print(name, "rel_loss", rel, flush=True)
    lv2._quantize_rows_tcq_ldlq = orig_rows
    arrays["meta"] = np.frombuffer(json.dumps(meta).encode(), dtype=np.uint8)
    np.savez_compressed(OUT / "matrix_quant_legacy.npz", **arrays)
    print((OUT / "matrix_quant_legacy.npz").stat().st_size, "bytes")


if __name__ == "__main__":
    if "--legacy" in sys.argv:
        legacy_main()
    else:
        main()
