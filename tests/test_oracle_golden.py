"""Pin the CPU oracle against the reference's own outputs (fixtures made by tests/golden/make_golden.py from the
reference tree, and — when present — tests/golden/ref_kernel_*.npz made on a B200 from the reference CUDA kernel
compiled from its own source).  No GPU needed."""
import json
from pathlib import Path

import numpy as np
import pytest

from oracle import oracle as O
from tests import vit_cases as VC

GOLDEN = Path(__file__).resolve().parent / "golden"


def _fmt(name, gains=None):
    c = VC.F[name]
    return O.LtqFormat(name, c["K"], c["pp"], (c["m"],) + tuple(c["m_extra"]), c["h"], c["step"], c["sub"],
                       np.asarray(c["lut"], np.float32),
                       np.asarray(c["gains_cpu"] if gains is None else gains, np.float32))


def test_torch_viterbi_ub_bit_exact():
    """oracle (products rounded first, as torch on CPU) == reference torch viterbi_ub (src/tcq_proto.py:363-419)."""
    z = np.load(GOLDEN / "torch_viterbi_ub.npz")
    meta = json.loads(bytes(z["meta"]).decode())
    assert len(meta) >= 6
    for m in meta:
        n = m["name"]
        K, U = m["K"], 1 << (m["K"] - 1)
        g = z[f"{n}/gains"] if m["h"] > 0 else None
        w = z[f"{n}/wts"] if m["weighted"] else None
        rec, gi, idx = O.viterbi(z[f"{n}/x"], z[f"{n}/small"], K, 10, 359, g, sub=m["sub"], wts=w, return_code=True,
                                 round_mode=O.ROUND_TORCH)
        assert np.array_equal(rec.view(np.uint32), z[f"{n}/rec"].view(np.uint32)), n
        assert np.array_equal(idx // U, z[f"{n}/labels"]), n
        assert np.array_equal(idx % U, z[f"{n}/u"]), n
        assert np.array_equal(gi[:, :: m["sub"]] if m["h"] > 0 else np.zeros_like(z[f"{n}/gidx"]), z[f"{n}/gidx"]), n


def test_format_tiles_match_reference():
    """states_from_codes / labels_from_states / pack_tile / decode_tile == src/ltq_format.py on random valid tiles."""
    z = np.load(GOLDEN / "ltq_format_tiles.npz")
    keys = sorted({k.rsplit("/", 1)[0] for k in z.files})
    assert len(keys) == 19 * 3 + 17 * 3
    for key in keys:
        name, L, _ = key.split("/")
        fmt = _fmt(name)
        c = z[key + "/codebits"].astype(np.uint32)
        st = O.states_from_codes(c)
        assert np.array_equal(st.astype(np.int32), z[key + "/states"]), key
        lab = O.labels_from_states(st, fmt)
        assert np.array_equal(lab.astype(np.int32), z[key + "/labels"]), key
        f = O.pack_tile(lab, z[key + "/u"], z[key + "/gidx"], fmt)
        assert np.array_equal(O.tile_words(f), z[key + "/words"]), key
        assert 2 * len(O.tile_words(f)) == int(z[key + "/tile_bytes"][0]) == fmt.tile_bytes(int(L[1:])), key
        assert np.array_equal(O.decode_tile(f, fmt).view(np.uint32), z[key + "/decoded"].view(np.uint32)), key


def test_tile_bytes_match_selftest_record():
    """Tile sizes of the 19 formats as recorded by the reference self-test (results/ltq_format_selftest.json)."""
    expect = {"TCQ2X0": 64, "TCQ2X": 66, "TCQ3X1": 98, "TCQ3X": 100, "TCQ4X1": 130, "TCQ4X2": 132, "TCQ4X": 134,
              "TCQ5X3": 166, "TCQ5X": 168, "TCQ4W2": 130, "TCQ4W3": 132, "TCQ25X": 82, "TCQ35X1": 114, "TCQ35X": 116,
              "TCQ45X": 148, "TCQ275X": 90, "TCQ275X2": 92, "TCQ375X": 124, "TCQ475X": 156}
    assert sorted(expect) == sorted(VC.MENU)
    for name, b in expect.items():
        assert _fmt(name).tile_bytes() == b, name


def test_slices_match_reference():
    """pack_slice / decode_slice == src/ltq_file.py:79-148 (SoA regions on 64-byte boundaries)."""
    z = np.load(GOLDEN / "ltq_file_slices.npz")
    names = sorted({k.split("/")[0] for k in z.files})
    assert len(names) == 6
    for name in names:
        fmt = _fmt(name)
        idx, gi = z[f"{name}/idx"].astype(np.int64), z[f"{name}/gi"].astype(np.int64)
        raw = O.pack_slice(idx, gi, fmt)
        assert np.array_equal(np.frombuffer(raw, np.uint8), z[f"{name}/bytes"]), name
        dec = O.decode_slice(raw, idx.shape[0], idx.shape[1], fmt)
        assert np.array_equal(dec.view(np.uint32), z[f"{name}/decoded"].view(np.uint32)), name


def test_fwht_matches_reference():
    z = np.load(GOLDEN / "fwht.npz")
    y = O.fwht(z["x"], 256)
    assert np.array_equal(y.view(np.uint32), z["y"].view(np.uint32))


@pytest.mark.parametrize("L", [256, 160])
def test_oracle_tail_biting_self_test(L):
    """The reference self-test criteria (src/ltq_format.py:150-181) on oracle outputs: labels recomputed from the code
    bits equal the quantizer's labels (tail-biting closure), the fractional-mode parity holds, and the packed tile
    decodes to the reconstruction bit for bit.  Recorded result: 0 / 0 / 0 for every format."""
    cases = VC.menu_tb_cases(N=6, L=L, seed=3)
    assert len(cases) == (19 if L == 256 else 17)
    for name, kw, x, wts in cases:
        kw = dict(kw)
        small, gains = kw.pop("small"), kw.pop("gains")
        rec, gi, idx = O.viterbi(x, small, wts=wts, gains=gains, **kw)
        fmt = _fmt(name.split("_")[0], gains)
        for n in range(x.shape[0]):
            lab, u = idx[n] // fmt.U, idx[n] % fmt.U
            assert np.array_equal(O.labels_from_states(O.states_from_codes(lab & 1), fmt), lab), name
            if fmt.frac == 1:
                assert np.all((u[0::2] & 1) == (u[1::2] & 1)), name
            if fmt.frac == 2:
                assert not np.any((u.reshape(-1, 4) & 1).sum(axis=1) & 1), name
            dec = O.decode_tile(O.pack_tile(lab, u, gi[n], fmt), fmt)
            assert np.array_equal(dec.view(np.uint32), rec[n].view(np.uint32)), name


def test_oracle_mse_close_to_recorded_gap():
    """Quality pin: the config-1 format (K = 2, h = 2) on the Gaussian rig reaches the recorded R(D) gap within
    sampling noise (results/universal_gaussian.json tcq_K2_h2: 0.1756 bits on 8192 tiles, seed 123, 9 scales)."""
    c = VC.F["_config1_tcq_K2_h2"]
    rng = np.random.default_rng(123)
    w = rng.standard_normal((96, 256)).astype(np.float32)
    d = np.sqrt((w * w).mean(axis=1, keepdims=True)).astype(np.float16).astype(np.float32)
    best = None
    for sc in (0.9, 0.95, 1.0, 1.05):
        rec = O.viterbi(w / (d * np.float32(sc)), np.asarray(c["lut"], np.float32), 2, 10, 359,
                        np.asarray(c["gains_cpu"], np.float32), tail_biting=True)
        D = float(((w - rec * d * np.float32(sc)) ** 2).mean())
        best = D if best is None else min(best, D)
    gap = 2 + 2 / 16 + 7 / 256 - 0.5 * np.log2(1.0 / best)
    assert abs(gap - c["gap"]) < 0.02, gap


def test_ref_kernel_fixtures():
    """oracle == the reference CUDA kernel (compiled for sm_100a from src/cuda/tcq_viterbi.cu, run on a B200) on every
    case of tests/vit_cases.py (fixtures from tests/golden/make_ref_kernel_golden.py)."""
    files = sorted(GOLDEN.glob("ref_kernel_*.npz"))
    if not files:
        pytest.skip("no reference-kernel fixtures recorded yet")
    n = 0
    for f in files:
        z = np.load(f, allow_pickle=False)
        meta = json.loads(bytes(z["meta"]).decode())
        for case in meta:
            name = case["name"]
            kw = dict(case["kw"])
            for k in ("m_extra",):
                if k in kw:
                    kw[k] = tuple(kw[k])
            arrs = {k.split("/", 1)[1]: z[k] for k in z.files if k.startswith(name + "/")}
            x = arrs.pop("x")
            wts = arrs.pop("wts", None)
            for k in ("small", "gains", "small_hi", "gains_hi", "init_state"):
                if k in arrs:
                    kw[k] = arrs.pop(k)
            out = O.viterbi(x, wts=wts, **kw)
            if kw.get("_mid"):
                assert np.array_equal(out[1], arrs["mid"]), name
            elif kw.get("return_code"):
                rec, gi, idx = out
                assert np.array_equal(rec.view(np.uint32), arrs["rec"].view(np.uint32)), name
                assert np.array_equal(gi, arrs["gi"]) and np.array_equal(idx, arrs["idx"]), name
            elif kw.get("return_end_state"):
                assert np.array_equal(out[0].view(np.uint32), arrs["rec"].view(np.uint32)), name
                assert np.array_equal(out[1], arrs["end"]), name
            n += 1
    assert n > 0


def _ltq_fmt(name, gains):
    from ltq_research_b200.formats import TCQ_CONFIG
    c = TCQ_CONFIG[name]
    return O.LtqFormat(name, c["K"], int(c.get("pp", 0)), (c["m"],) + tuple(c.get("m_extra", ())), c["h"],
                       float(c["step"]), c.get("sub", 16), np.asarray(c["lut"], np.float32), np.asarray(gains, np.float32))


def test_pack_slices_all_formats_match_reference():
    """The oracle's pack_slice / decode_slice == the reference's (src/ltq_file.py:79-148) for every .ltq tile format
    of TCQ_CONFIG (tests/golden/pack_slices.npz, made by tests/golden/make_golden_pack.py)."""
    z = np.load(GOLDEN / "pack_slices.npz")
    meta = json.loads(bytes(z["meta"]).decode())
    assert len(meta) == 35  # every tail-biting format but the three EQ ones, which have no .ltq encoding
    for m in meta:
        n = m["name"]
        fmt = _ltq_fmt(n, z[f"{n}/gains"])
        raw = O.pack_slice(z[f"{n}/idx"].astype(np.int64), z[f"{n}/gi"].astype(np.int64), fmt)
        assert np.array_equal(np.frombuffer(raw, np.uint8), z[f"{n}/bytes"]), n
        dec = O.decode_slice(raw, m["R"], m["K"], fmt)
        assert np.array_equal(dec.view(np.uint32), z[f"{n}/vals"].view(np.uint32)), n


def test_legacy_formats_table():
    """The earlier, non-tail-biting formats (src/liqk_v2.py:786-821) load with the reference's constants and bit counts
    (tests/golden/formats.json "legacy", written from the reference's TCQ_CONFIG / LIQK_V2_SPECS), and stay out of the
    .ltq format list."""
    import json
    from pathlib import Path
    from ltq_research_b200.formats import LEGACY_FORMATS, LIQK_V2_SPECS, LTQ_FORMATS, TCQ_CONFIG
    doc = json.loads((Path(__file__).resolve().parent / "golden" / "formats.json").read_text())
    assert sorted(LEGACY_FORMATS) == sorted(doc["legacy"]) == sorted(
        ["TCQ2", "TCQ3", "TCQ4", "TCQ2R", "TCQ3R", "TCQ4R", "TCQ3RH", "TCQ4RH", "TCQ4RH3", "TCQ25R", "TCQ35R"])
    assert not set(LEGACY_FORMATS) & set(LTQ_FORMATS) and len(LTQ_FORMATS) == 38
    for name, t in doc["legacy"].items():
        c = TCQ_CONFIG[name]
        assert not c.get("tb") and bool(c.get("row_scale")) == t["row_scale"] and bool(c.get("carry")) == t["carry"]
        assert LIQK_V2_SPECS[name].block_bytes * 8 == t["bits"], name
        if "K_hi" in t:
            assert (c["lo"], c["hi"], c["K_hi"]) == (t["lo"], t["hi"], t["K_hi"])
        else:
            assert c["lut"] == t["lut"] and c["step"] == t["step"]
    assert TCQ_CONFIG["TCQ4RH3"]["n_cand"] == 4 and TCQ_CONFIG["TCQ3R"]["carry"] and "row_scale" not in TCQ_CONFIG["TCQ3"]
