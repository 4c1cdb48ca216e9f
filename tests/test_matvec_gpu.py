"""GPU: the batch-1 product straight from packed .ltq slices (ltq_matvec_slice; the reference prototypes it in
src/cuda/ltq_matvec_bench.cu:77-150).  With unit scales and one-hot inputs it returns the spec-decoded tile values
bit for bit on the reference's own packed slices of all 35 .ltq formats (tests/golden/pack_slices.npz); on quantized
matrices (one format, and two row slices of different formats) it equals assemble(...) @ x within the fp32 bound of
its length-K sum; LtqFile.matvec gives the same from a written file."""
import json
from pathlib import Path

import numpy as np
import pytest
import torch

from tests.golden.matrix_inputs import synth
from tests.test_pack_gpu import _fmt

pytestmark = pytest.mark.gpu
GOLDEN = Path(__file__).resolve().parent / "golden"


def test_matvec_one_hot_returns_decoded_values_all_formats(cuda_dev):
    from ltq_research_b200.ltq_file import decode_slice_device, matvec_slice_device
    z = np.load(GOLDEN / "pack_slices.npz")
    meta = json.loads(bytes(z["meta"]).decode())
    g = np.random.default_rng(2)
    for m in meta:
        n, R, K = m["name"], m["R"], m["K"]
        f = _fmt(n, z[f"{n}/gains"])
        raw = z[f"{n}/bytes"]
        data = torch.zeros(((raw.size + 63) // 64) * 64, dtype=torch.uint8, device=cuda_dev)
        data[: raw.size] = torch.from_numpy(raw).to(cuda_dev)
        val = decode_slice_device(data, R, K, f)
        d_row = torch.ones(R, dtype=torch.float16, device=cuda_dev)
        e = torch.zeros((R, K // 256), dtype=torch.int8, device=cuda_dev)
        for k in g.choice(K, 4, replace=False):
            x = torch.zeros(K, device=cuda_dev)
            x[int(k)] = 1.0
            y = matvec_slice_device(data, R, K, f, d_row, e, x)
            assert torch.equal(y, val[:, int(k)]), (n, int(k))


def _bound(W, x):
    K = W.shape[1]
    u = 2.0 ** -24
    return (2 * K * u) * (W.double().abs() @ x.double().abs()) + 1e-30


def test_matvec_quantized_matrices(cuda_dev):
    """Quantized matrices through the batch driver (single format; two row slices in two formats, one of them D2):
    matvec from the packed tensors vs the assembled matrix times x in float64."""
    from ltq_research_b200.batch import quantize_matrices
    from ltq_research_b200.formats import load_formats
    from ltq_research_b200.ltq_file import assemble, decode_slice_device, matvec
    fm = load_formats(["TCQ3X", "TCQ45X", "TCQ25X"], cuda_dev)
    names = list(fm)
    jobs = [(*synth(96, 768, 51), "TCQ3X"), (*synth(64, 512, 52), [(0, 32, "TCQ25X"), (32, 64, "TCQ45X")])]
    res = quantize_matrices([(W.to(cuda_dev), H.to(cuda_dev), sp) for W, H, sp in jobs], ltq_formats=fm, pack=True)
    g = torch.Generator(device=cuda_dev).manual_seed(3)
    for r in res:
        lt = r["ltq"]
        M, K = lt["d_row"].shape[0], lt["suh"].shape[0]
        data = torch.zeros(((lt["data"].numel() + 63) // 64) * 64, dtype=torch.uint8, device=cuda_dev)
        data[: lt["data"].numel()] = lt["data"]
        G = torch.empty((M, K), device=cuda_dev)
        for r0, r1, fi, off in lt["slices"]:
            decode_slice_device(data[off:], r1 - r0, K, fm[names[fi]], out=G[r0:r1])
        W = assemble(G, lt["d_row"], lt["e"], lt["suh"])
        for _ in range(3):
            x = torch.randn(K, device=cuda_dev, generator=g)
            y = matvec(data, lt["slices"], list(fm.values()), lt["d_row"], lt["e"], lt["suh"], x)
            want = W.double() @ x.double()
            assert ((y.double() - want).abs() <= _bound(W, x)).all()
        # deterministic
        assert torch.equal(matvec(data, lt["slices"], list(fm.values()), lt["d_row"], lt["e"], lt["suh"], x), y)


def test_ltq_file_matvec(cuda_dev, tmp_path):
    import ltq_research_b200.liqk_v2 as Lq
    from ltq_research_b200.formats import load_formats
    from ltq_research_b200.ltq_file import LtqFile, LtqWriter, format_json
    fm = load_formats(["TCQ3X", "TCQ25X"], cuda_dev)
    W, H = synth(64, 512, 61)
    path = tmp_path / "m.ltq"
    w = LtqWriter(path, list(fm.values()), reserve=(1 << 20) - 16)
    Lq.PACK = {}
    try:
        _, w_hat, _ = Lq.quantize_matrix_liqk_v2(W.to(cuda_dev), H.to(cuda_dev), "TCQ25X", damp=0.02)
        w.add_matrix("blk.0.v", Lq.PACK["matrix"])
    finally:
        Lq.PACK = None
    w.finalize({"quantization": {"formats": [format_json(f) for f in fm.values()]}})
    lf = LtqFile(path)
    x = torch.randn(512, device=cuda_dev)
    y = lf.matvec("blk.0.v", x, device=cuda_dev)
    want = w_hat.double() @ x.double()
    assert ((y.double() - want).abs() <= _bound(w_hat, x)).all()
