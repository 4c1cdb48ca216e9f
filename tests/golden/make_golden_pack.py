"""Golden fixtures of the .ltq tile packing: the reference's own pack_slice / decode_slice (src/ltq_file.py:79-148)
run from the reference tree on CPU, on seeded random codes (idx = label * U + u, gi) of every .ltq tile format of
TCQ_CONFIG (fractional modes none / D2 / D4) and slice shapes with several row groups and column blocks.

    PYTHONDONTWRITEBYTECODE=1 python tests/golden/make_golden_pack.py
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

import src.ltq_file as lf  # noqa: E402
from src.ltq_format import LtqFormat as RefFormat  # noqa: E402
from ltq_research_b200.formats import TCQ_CONFIG  # noqa: E402
from ltq_research_b200.tcq_proto import make_gains  # noqa: E402

SHAPES = [(32, 256), (16, 256), (16, 512)]


def main():
    arrays, meta = {}, []
    rng = np.random.default_rng(20261201)
    for i, (name, c) in enumerate(sorted((n, c) for n, c in TCQ_CONFIG.items() if c.get("tb"))):
        if int(c.get("pp", 0)) > 2:
            continue
        masks = (c["m"],) + tuple(c.get("m_extra", ()))
        gains = make_gains(c["h"], c["step"], "cpu").numpy().astype(np.float32)
        f = RefFormat(name, c["K"], int(c.get("pp", 0)), masks, c["h"], float(c["step"]), c.get("sub", 16),
                      np.asarray(c["lut"], np.float32), gains)
        R, K = SHAPES[i % len(SHAPES)]
        nl = 2 ** len(masks) * 2
        idx = rng.integers(0, nl * f.U, size=(R, K)).astype(np.int16)
        gi = rng.integers(0, 1 << c["h"], size=(R, K)).astype(np.uint8) if c["h"] else np.zeros((R, K), np.uint8)
        raw = lf.pack_slice(torch.from_numpy(idx), torch.from_numpy(gi), f)
        vals = lf.decode_slice(raw, R, K, f, "cpu").numpy()
        arrays[f"{name}/idx"] = idx
        arrays[f"{name}/gi"] = gi
        arrays[f"{name}/bytes"] = np.frombuffer(raw, dtype=np.uint8)
        arrays[f"{name}/vals"] = vals.astype(np.float32)
        arrays[f"{name}/gains"] = gains
        meta.append({"name": name, "R": R, "K": K, "bytes": len(raw)})
        print(name, R, K, len(raw), flush=True)
    arrays["meta"] = np.frombuffer(json.dumps(meta).encode(), dtype=np.uint8)
    np.savez_compressed(OUT / "pack_slices.npz", **arrays)
    print((OUT / "pack_slices.npz").stat().st_size, "bytes")


if __name__ == "__main__":
    main()
