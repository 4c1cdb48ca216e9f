"""Record the reference CUDA kernel's outputs on every Viterbi parity case (tests/vit_cases.py) as fixtures.

Runs on a GPU box: the reference kernel is oracle/_ref/libtcq_viterbi_ref.so, built here from the reference's own
src/cuda/tcq_viterbi.cu (make -C oracle ref) and driven like the reference's Python wrapper (oracle/ref_kernel.py).
The CPU test suite then pins the oracle against these fixtures (tests/test_oracle_golden.py::test_ref_kernel_fixtures).

    python tests/golden/make_ref_kernel_golden.py  [out_dir]
"""
from __future__ import annotations

import json
import sys
from pathlib import Path

import numpy as np
import torch

ROOT = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(ROOT))

from oracle import ref_kernel as R  # noqa: E402
from tests import vit_cases as VC  # noqa: E402


def record(cases, path: Path):
    dev = torch.device("cuda:0")
    arrays, meta = {}, []
    for name, kw, x, wts in cases:
        kwd = dict(kw)
        arrs = {"x": x}
        if wts is not None:
            arrs["wts"] = np.ascontiguousarray(wts)
        for k in ("small", "gains", "small_hi", "gains_hi", "init_state"):
            if kwd.get(k) is not None:
                arrs[k] = np.ascontiguousarray(kwd.pop(k))
        tkw = {k: torch.from_numpy(v).to(dev) for k, v in arrs.items() if k not in ("x", "wts")}
        out = R.viterbi_ub_cuda_ref(torch.from_numpy(x).to(dev), tkw.pop("small"),
                                    wts=None if wts is None else torch.from_numpy(arrs["wts"]).to(dev), **tkw, **kwd)
        torch.cuda.synchronize()
        out = out if isinstance(out, tuple) else (out,)
        out = [o.cpu().numpy() for o in out]
        if kwd.get("_mid"):
            arrs["mid"] = out[1]
        elif kwd.get("return_code"):
            arrs["rec"], arrs["gi"], arrs["idx"] = out
        elif kwd.get("return_end_state"):
            arrs["rec"], arrs["end"] = out
        else:
            arrs["rec"] = out[0]
        for k, v in arrs.items():
            arrays[f"{name}/{k}"] = v
        meta.append({"name": name, "kw": {k: (list(v) if isinstance(v, tuple) else v) for k, v in kwd.items()}})
    arrays["meta"] = np.frombuffer(json.dumps(meta).encode(), dtype=np.uint8)
    np.savez_compressed(path, **arrays)
    print(path, path.stat().st_size, "bytes,", len(meta), "cases")


if __name__ == "__main__":
    out = Path(sys.argv[1]) if len(sys.argv) > 1 else Path(__file__).resolve().parent
    out.mkdir(parents=True, exist_ok=True)
    if not R.available():
        raise SystemExit("oracle/_ref/libtcq_viterbi_ref.so is missing (make -C oracle ref)")
    record(VC.menu_tb_cases(N=8, L=256, seed=21), out / "ref_kernel_menu_tiles.npz")
    record(VC.menu_tb_cases(N=6, L=160, seed=22), out / "ref_kernel_menu_rings.npz")
    record(VC.menu_tb_cases(N=6, L=256, seed=23, window=32, weighted=True), out / "ref_kernel_menu_ldlq.npz")
    record(VC.special_cases(N=6, seed=24) + VC.direct_cases(N=6, seed=25), out / "ref_kernel_special.npz")
    record(VC.nl32_cases(N=6, seed=26), out / "ref_kernel_nl32.npz")
    record(VC.s256_cases(N=6, seed=27), out / "ref_kernel_s256.npz")
