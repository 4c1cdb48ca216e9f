"""Generate golden fixtures from the reference Python implementation (lumen-inference/ltq-research).

Runs only where the reference tree is importable (LTQ_REF_ROOT names its root); the GPU box and the product never
run it.  Fixtures written next to this file:

* torch_viterbi_ub.npz  — the reference torch Viterbi `viterbi_ub` (src/tcq_proto.py:363-419) on seeded inputs, CPU.
* ltq_format_tiles.npz  — `pack_tile` / `decode_tile` / `states_from_codes` / `labels_from_states`
                          (src/ltq_format.py:76-147) for every format of the TCQPQ menu, tiles and rings of 160.
* ltq_file_slices.npz   — `pack_slice` / `decode_slice` (src/ltq_file.py:79-148) for a few formats.
* fwht.npz              — `fwht_inplace` (src/iqk_format.py:153-170) and `make_rademacher_signs` (:173-179).
* formats.json          — the TCQPQ menu parameters as the reference's TCQ_CONFIG builds them (src/liqk_v2.py:834-840)
                          with the gain tables evaluated by torch on CPU (the format stores its gain table explicitly),
                          and the earlier non-tail-biting formats (src/liqk_v2.py:786-821) under "legacy".

    PYTHONDONTWRITEBYTECODE=1 TCQ_NO_COMPILE=1 python tests/golden/make_golden.py [--formats-only]
"""
from __future__ import annotations

import json
import sys
from pathlib import Path

import numpy as np

OUT = Path(__file__).resolve().parent
sys.path.insert(0, str(OUT.parent.parent))
from oracle.refroot import import_reference  # noqa: E402

REF = import_reference()  # the tree named by LTQ_REF_ROOT, else the install in baseline/_ref

import torch  # noqa: E402

from src import ltq_file, ltq_format  # noqa: E402
import src.liqk_v2 as lv2  # noqa: E402
from src.equal_bpw import SETS  # noqa: E402
from src.iqk_format import fwht_inplace, make_rademacher_signs  # noqa: E402
from src.tcq_proto import make_gains, viterbi_ub  # noqa: E402


def fmt_of(name: str) -> ltq_format.LtqFormat:
    c = lv2.TCQ_CONFIG[name]
    return ltq_format.LtqFormat(name, c["K"], int(c.get("pp", 0)), (c["m"],) + tuple(c.get("m_extra", ())), c["h"],
                                float(c["step"]), c.get("sub", 16), np.asarray(c["lut"], dtype=np.float32),
                                make_gains(c["h"], c["step"], "cpu").numpy())


def formats_json():
    """Format constants of every tail-biting (.ltq) format of the reference's TCQ_CONFIG.  Written twice: as a fixture
    and as the package's format table (ltq_research_b200/data/tcq_formats.json) — the LUT values, masks, gain steps and
    scales define the format, so they must be identical to the reference's for files to be compatible."""
    menu = SETS["TCQPQ"]
    out = {}
    tb_names = [n for n, c in lv2.TCQ_CONFIG.items() if c.get("tb")]
    for name in tb_names:
        c = lv2.TCQ_CONFIG[name]
        out[name] = {"K": c["K"], "nu": c["nu"], "m": c["m"], "m_extra": list(c.get("m_extra", ())), "h": c["h"],
                     "step": float(c["step"]), "sub": c.get("sub", 16), "pp": int(c.get("pp", 0)),
                     "scale": float(c.get("scale", 1.0)), "n_cand": int(c.get("n_cand", 0)),
                     "lut": [float(v) for v in np.asarray(c["lut"], np.float32)],
                     "gains_cpu": [float(v) for v in make_gains(c["h"], c["step"], "cpu").numpy()],
                     "in_tcqpq": name in menu, "bits": float(lv2.LIQK_V2_SPECS[name].block_bytes * 8)}
    u = json.loads((REF / "results" / "universal_gaussian.json").read_text())["tcq_K2_h2"]
    out["_config1_tcq_K2_h2"] = {"K": 2, "nu": 10, "m": 359, "m_extra": [], "h": 2, "step": float(u["step"]), "sub": 16,
                                 "pp": 0, "scale": 1.0, "n_cand": 0,
                                 "lut": [float(v) for v in np.asarray(u["tab"], np.float32)],
                                 "gains_cpu": [float(v) for v in make_gains(2, u["step"], "cpu").numpy()],
                                 "in_tcqpq": False, "gap": float(u["gap"])}
    # the earlier (non-tail-biting) formats: per-block scale with a refit (TCQ2 / TCQ3 / TCQ4), one scale per row with
    # the trellis state carried from tile to tile (the R formats), half-integer rows (TCQ25R / TCQ35R: tables of the
    # "lo" / "hi" formats premultiplied by their scales).  Quantized by the driver; not written to .ltq files.
    legacy = {}
    for name, c in lv2.TCQ_CONFIG.items():
        if c.get("tb"):
            continue
        e = {"K": c["K"], "nu": c["nu"], "m": c["m"], "h": c["h"], "scale": float(c.get("scale", 1.0)),
             "row_scale": bool(c.get("row_scale", False)), "carry": bool(c.get("carry", False)),
             "n_cand": int(c.get("n_cand", 0)), "bits": float(lv2.LIQK_V2_SPECS[name].block_bytes * 8)}
        if "K_hi" in c:
            e.update({"K_hi": c["K_hi"], "lo": c["lo"], "hi": c["hi"]})
        else:
            e.update({"step": float(c["step"]), "lut": [float(v) for v in np.asarray(c["lut"], np.float32)]})
        legacy[name] = e
    doc = {"menu_TCQPQ": menu, "sets": {k: v for k, v in SETS.items() if v is not None and k.startswith("TCQ")},
           "formats": out, "legacy": legacy}
    (OUT / "formats.json").write_text(json.dumps(doc, indent=1))
    pkg = OUT.parent.parent / "ltq_research_b200" / "data"
    pkg.mkdir(exist_ok=True)
    (pkg / "tcq_formats.json").write_text(json.dumps(doc, indent=1))
    return out


def torch_viterbi_cases():
    """viterbi_ub covers the plain mode only: 4 subsets, no tail-biting, no candidates, no init / end state."""
    cases = [
        # name, K, h, step, sub, weighted, N, T, seed
        ("k2_h0", 2, 0, 0.0, 16, False, 6, 256, 1),
        ("k2_h2", 2, 2, 0.3, 16, False, 6, 256, 2),
        ("k3_h1_w", 3, 1, 0.4, 16, True, 6, 256, 3),
        ("k4_h2_w", 4, 2, 0.25, 16, True, 4, 256, 4),
        ("k3_h2_sub32", 3, 2, 0.3, 32, True, 4, 256, 5),
        ("k2_h1_T160", 2, 1, 0.4, 16, False, 5, 160, 6),
    ]
    arrays = {}
    meta = []
    for name, K, h, step, sub, weighted, N, T, seed in cases:
        g = torch.Generator().manual_seed(seed)
        U = 1 << (K - 1)
        n = 4 * U
        lev = torch.special.ndtri((torch.arange(n, dtype=torch.float64) + 0.5) / n).float()
        small = lev.view(U, 4).T.contiguous().flatten()
        x = torch.randn(N, T, generator=g) * 1.1
        gains = make_gains(h, step, "cpu") if h > 0 else None
        wts = (torch.rand(T, generator=g) * 2 + 0.2) if weighted else None
        rec, labels, u, gidx = viterbi_ub(x, small, K, 10, 359, gains, sub=sub, wts=wts)
        arrays[f"{name}/x"] = x.numpy()
        arrays[f"{name}/small"] = small.numpy()
        arrays[f"{name}/gains"] = (gains if gains is not None else torch.ones(1)).numpy()
        arrays[f"{name}/wts"] = (wts if wts is not None else torch.ones(T)).numpy()
        arrays[f"{name}/rec"] = rec.numpy()
        arrays[f"{name}/labels"] = labels.numpy().astype(np.int32)
        arrays[f"{name}/u"] = u.numpy().astype(np.int32)
        arrays[f"{name}/gidx"] = gidx.numpy().astype(np.int32)
        meta.append({"name": name, "K": K, "h": h, "sub": sub, "weighted": weighted, "N": N, "T": T})
    arrays["meta"] = np.frombuffer(json.dumps(meta).encode(), dtype=np.uint8)
    np.savez_compressed(OUT / "torch_viterbi_ub.npz", **arrays)


def _random_codes(fmt, L, rng):
    """Random valid tile content: code bits, levels obeying the fractional-mode parity, gain index per sub-block."""
    c = rng.integers(0, 2, L).astype(np.uint32)
    lab = ltq_format.labels_from_states(ltq_format.states_from_codes(c), fmt)
    u = rng.integers(0, fmt.U, L).astype(np.uint32)
    if fmt.frac == 1:
        u[1::2] = (u[1::2] & ~np.uint32(1)) | (u[0::2] & 1)
    elif fmt.frac == 2:
        q = u.reshape(-1, 4)
        q[:, 3] = (q[:, 3] & ~np.uint32(1)) | (q[:, :3].sum(axis=1).astype(np.uint32) & 1)
        u = q.reshape(-1)
    gsub = rng.integers(0, 1 << fmt.h, L // fmt.sub).astype(np.uint32) if fmt.h else np.zeros(L // fmt.sub, np.uint32)
    gidx = np.repeat(gsub, fmt.sub)
    return c, lab, u, gidx


def ltq_format_cases():
    rng = np.random.default_rng(1234)
    arrays = {}
    for name in SETS["TCQPQ"]:
        fmt = fmt_of(name)
        for L in (256, 160):
            if L != 256 and fmt.sub != 16:
                continue
            for k in range(3):
                c, lab, u, gidx = _random_codes(fmt, L, rng)
                f = ltq_format.pack_tile(lab, u, gidx, fmt)
                dec = ltq_format.decode_tile(f, fmt)
                key = f"{name}/L{L}/{k}"
                arrays[key + "/codebits"] = c.astype(np.uint8)
                arrays[key + "/states"] = ltq_format.states_from_codes(c).astype(np.int32)
                arrays[key + "/labels"] = lab.astype(np.int32)
                arrays[key + "/u"] = u.astype(np.int32)
                arrays[key + "/gidx"] = gidx.astype(np.int32)
                arrays[key + "/words"] = np.concatenate([f["codes"], f["planes"].reshape(-1), f["lsb"],
                                                         f["gains"]]).astype(np.uint16)
                arrays[key + "/decoded"] = dec
                arrays[key + "/tile_bytes"] = np.array([fmt.tile_bytes(L)], np.int32)
    np.savez_compressed(OUT / "ltq_format_tiles.npz", **arrays)


def ltq_file_cases():
    rng = np.random.default_rng(99)
    arrays = {}
    for name in ("TCQ2X", "TCQ3X", "TCQ4W3", "TCQ35X", "TCQ275X2", "TCQ5X"):
        fmt = fmt_of(name)
        R, K = 32, 512
        idx = np.zeros((R, K), np.int64)
        gi = np.zeros((R, K), np.int64)
        tl = np.zeros(((R // 16) * (K // 16), 256), np.int64)
        tg = np.zeros_like(tl)
        for t in range(tl.shape[0]):
            c, lab, u, gidx = _random_codes(fmt, 256, rng)
            tl[t] = lab.astype(np.int64) * fmt.U + u
            tg[t] = gidx
        idx = ltq_file._untiles(torch.from_numpy(tl), R, K).numpy()
        gi = ltq_file._untiles(torch.from_numpy(tg), R, K).numpy()
        raw = ltq_file.pack_slice(torch.from_numpy(idx).to(torch.int16), torch.from_numpy(gi).to(torch.uint8), fmt)
        dec = ltq_file.decode_slice(raw, R, K, fmt, "cpu").numpy()
        arrays[f"{name}/idx"] = idx.astype(np.int16)
        arrays[f"{name}/gi"] = gi.astype(np.uint8)
        arrays[f"{name}/bytes"] = np.frombuffer(raw, dtype=np.uint8)
        arrays[f"{name}/decoded"] = dec
    np.savez_compressed(OUT / "ltq_file_slices.npz", **arrays)


def fwht_cases():
    g = torch.Generator().manual_seed(7)
    x = torch.randn(24, 512, generator=g) * torch.exp(torch.randn(24, 1, generator=g))
    y = fwht_inplace(x.clone(), block_size=256)
    signs = make_rademacher_signs(1024, seed=1337, device="cpu")
    np.savez_compressed(OUT / "fwht.npz", x=x.numpy(), y=y.numpy(), signs_1337_1024=signs.numpy())


if __name__ == "__main__":
    formats_json()
    if "--formats-only" in sys.argv:
        raise SystemExit(0)
    torch_viterbi_cases()
    ltq_format_cases()
    ltq_file_cases()
    fwht_cases()
    for p in sorted(OUT.glob("*.npz")) + [OUT / "formats.json"]:
        print(p.name, p.stat().st_size)
