"""GPU: .ltq packing and spec decode kernels (ltq_pack_slice / ltq_decode_slice) against the reference's own
pack_slice / decode_slice outputs (tests/golden/pack_slices.npz), the on-device verify of LtqWriter.add_matrix, and a
write / read round trip of a .ltq file."""
import json
from pathlib import Path

import numpy as np
import pytest
import torch

from tests.golden.matrix_inputs import synth

pytestmark = pytest.mark.gpu
GOLDEN = Path(__file__).resolve().parent / "golden"


def _fmt(name, gains):
    from ltq_research_b200.formats import TCQ_CONFIG, LtqFormat
    c = TCQ_CONFIG[name]
    return LtqFormat(name, c["K"], int(c.get("pp", 0)), (c["m"],) + tuple(c.get("m_extra", ())), c["h"],
                     float(c["step"]), c.get("sub", 16), np.asarray(c["lut"], np.float32), np.asarray(gains, np.float32))


def test_pack_and_decode_match_reference_all_formats(cuda_dev):
    from ltq_research_b200.ltq_file import decode_slice, pack_slice, pack_slice_device, slice_bytes
    z = np.load(GOLDEN / "pack_slices.npz")
    meta = json.loads(bytes(z["meta"]).decode())
    for m in meta:
        n, R, K = m["name"], m["R"], m["K"]
        f = _fmt(n, z[f"{n}/gains"])
        idx = torch.from_numpy(z[f"{n}/idx"]).to(cuda_dev)
        gi = torch.from_numpy(z[f"{n}/gi"]).to(cuda_dev)
        assert slice_bytes(R, K, f) == m["bytes"], n
        raw = pack_slice(idx, gi, f)
        assert raw == z[f"{n}/bytes"].tobytes(), n
        # strided row slice of a wider matrix (as LtqWriter packs row slices of PACK["matrix"])
        wide_i = torch.zeros((R + 32, K), dtype=torch.int16, device=cuda_dev)
        wide_g = torch.zeros((R + 32, K), dtype=torch.uint8, device=cuda_dev)
        wide_i[16:16 + R], wide_g[16:16 + R] = idx, gi
        assert pack_slice_device(wide_i[16:16 + R], wide_g[16:16 + R], f).cpu().numpy().tobytes() == raw, n
        # every byte of the slice is written (padding included): an output buffer full of 0xAB gives the same bytes
        dirty = torch.full((len(raw) + 128,), 0xAB, dtype=torch.uint8, device=cuda_dev)
        assert pack_slice_device(idx, gi, f, out=dirty).cpu().numpy().tobytes() == raw, n
        assert bool((dirty[len(raw):] == 0xAB).all()), n
        vals = decode_slice(raw, R, K, f, cuda_dev).cpu().numpy()
        assert np.array_equal(vals.view(np.uint32), z[f"{n}/vals"].view(np.uint32)), n
        # rows that are not 16-byte aligned (scalar stores / loads) decode and verify the same values
        from ltq_research_b200.ltq_file import decode_slice_device
        buf = dirty[: len(raw)]
        wide = torch.zeros((R, K + 1), dtype=torch.float32, device=cuda_dev)
        decode_slice_device(buf, R, K, f, out=wide[:, 1:])
        assert np.array_equal(wide[:, 1:].cpu().numpy().view(np.uint32), z[f"{n}/vals"].view(np.uint32)), n
        bad = torch.zeros(1, dtype=torch.int64, device=cuda_dev)
        decode_slice_device(buf, R, K, f, ref=wide[:, 1:], mismatches=bad)
        assert int(bad) == 0, n


def test_pack_kernel_validation(cuda_dev):
    from ltq_research_b200 import _lib
    L = _lib.lib()
    st = torch.cuda.current_stream().cuda_stream
    idx = torch.zeros((16, 256), dtype=torch.int16, device=cuda_dev)
    gi = torch.zeros((16, 256), dtype=torch.uint8, device=cuda_dev)
    out = torch.zeros(4096, dtype=torch.uint8, device=cuda_dev)
    assert L.ltq_slice_bytes(15, 256, 3, 0, 2, 16) == 0                       # rows not a multiple of 16
    assert L.ltq_slice_bytes(16, 256, 3, 3, 2, 16) == 0                       # EQ has no .ltq encoding
    assert L.ltq_pack_slice(idx.data_ptr(), gi.data_ptr(), 256, 16, 256, 3, 0, 2, 16, out.data_ptr(), 8, st) == -1
    assert L.ltq_pack_slice(idx.data_ptr() + 2, gi.data_ptr(), 256, 16, 256, 3, 0, 2, 16, out.data_ptr(), 4096,
                            st) == -1                                       # misaligned idx
    assert L.ltq_pack_slice(idx.data_ptr(), gi.data_ptr(), 256, 16, 256, 3, 0, 2, 16, out.data_ptr(), 4096, st) == 0


@pytest.mark.parametrize("spec", ["TCQ3X", "TCQ25X", "TCQ275X2", "TCQ2X0", "TCQ4W2"])
def test_verify_on_device_with_quantizer_output(spec, cuda_dev):
    """The packed codes of a quantized matrix decode to the quantizer's tile values in every weight; a tile value that
    disagrees with its codes (changed in the reference tensor, on the host side of the check) is counted."""
    import ltq_research_b200.liqk_v2 as Lq
    from ltq_research_b200.formats import load_formats
    from ltq_research_b200.ltq_file import pack_matrix_device
    W, H = synth(64, 512, 31)
    Lq.PACK = {}
    try:
        Lq.quantize_matrix_liqk_v2(W.to(cuda_dev), H.to(cuda_dev), spec, damp=0.02)
        m = dict(Lq.PACK["matrix"])
    finally:
        Lq.PACK = None
    fmts = load_formats([spec], cuda_dev)
    data, rows, bad = pack_matrix_device(m, fmts, verify=True)
    assert int(bad.item()) == 0
    assert rows == [[0, 64, 0, 0]]
    G2 = m["G"].clone()
    G2[5, 300] = G2[5, 300] + 1.0
    G2[40, 7] = -G2[40, 7] - 0.5
    m2 = dict(m, G=G2)
    _, _, bad2 = pack_matrix_device(m2, fmts, verify=True)
    assert int(bad2.item()) == 2


def test_ltq_file_round_trip(cuda_dev, tmp_path):
    """LtqWriter (device pack + verify) -> LtqFile.decode_matrix reproduces the quantizer's W_hat bit for bit, for a
    single-format matrix and a matrix with two row slices of different formats."""
    import ltq_research_b200.liqk_v2 as Lq
    from ltq_research_b200.formats import load_formats
    from ltq_research_b200.ltq_file import LtqFile, LtqWriter, format_json
    fm = load_formats(["TCQ3X", "TCQ45X", "TCQ25X"], cuda_dev)
    jobs = {"blk.0.q": (synth(64, 512, 41), "TCQ3X"),
            "blk.0.o": (synth(64, 256, 42), [(0, 32, "TCQ25X"), (32, 64, "TCQ45X")])}
    path = tmp_path / "t.ltq"
    w = LtqWriter(path, list(fm.values()), reserve=(1 << 20) - 16)
    want = {}
    for name, ((W, H), spec) in jobs.items():
        Lq.PACK = {}
        try:
            _, w_hat, _ = Lq.quantize_matrix_liqk_v2(W.to(cuda_dev), H.to(cuda_dev), spec, damp=0.02)
            w.add_matrix(name, Lq.PACK["matrix"])
        finally:
            Lq.PACK = None
        want[name] = w_hat
    w.finalize({"quantization": {"formats": [format_json(f) for f in fm.values()]}})
    lf = LtqFile(path)
    for name, w_hat in want.items():
        got = lf.decode_matrix(name, device=cuda_dev)
        assert torch.equal(got, w_hat), name
