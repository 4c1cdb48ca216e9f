"""GPU: a matrix quantized in row shards (the quantizer core with row_reduce, the path of shard.row_ranges /
nccl_row_reduce for matrices split across ranks) against the same matrix quantized whole.

The shards run as threads of one process on one GPU, each on its own stream, with a row_reduce that adds the shards'
tensors in shard order (the place of an NCCL all-reduce between processes).  Every shard must reach the same suh bit
for bit (the row sums are the only coupling); against the whole-matrix run, the sums only change order, so suh, the
codes and the relative loss agree within rounding.  Through the batch driver, the shards' packed fields merged by
shard.merge_row_shards give the same y = W x as the shards' own."""
import threading

import pytest
import torch

from tests.golden.matrix_inputs import synth

pytestmark = pytest.mark.gpu


class _ThreadSum:
    """row_reduce for n shards run as threads: each call waits for all shards and leaves the sum, in shard order, in
    every shard's tensor."""

    def __init__(self, n: int):
        self.n, self.slots = n, [None] * n
        self.bar = threading.Barrier(n, timeout=120)

    def fn(self, k: int):
        def reduce(t: torch.Tensor):
            self.slots[k] = t.clone()
            torch.cuda.current_stream().synchronize()
            self.bar.wait()
            total = self.slots[0].clone()
            for j in range(1, self.n):
                total += self.slots[j]
            torch.cuda.current_stream().synchronize()
            self.bar.wait()
            t.copy_(total)
        return reduce


def _run_shards(fn, n):
    """fn(k, reduce) in n threads, each on its own CUDA stream; results in shard order, errors re-raised."""
    red = _ThreadSum(n)
    out, err = [None] * n, []
    torch.cuda.synchronize()  # inputs made on the default stream are complete before the shards' streams read them

    def body(k):
        try:
            with torch.cuda.stream(torch.cuda.Stream()):
                out[k] = fn(k, red.fn(k))
                torch.cuda.current_stream().synchronize()
        except BaseException as e:  # noqa: BLE001
            err.append(e)
            red.bar.abort()
    ts = [threading.Thread(target=body, args=(k,)) for k in range(n)]
    for t in ts:
        t.start()
    for t in ts:
        t.join(timeout=300)
    if err:
        raise err[0]
    return out


@pytest.mark.parametrize("gemm", ["bf16x6", "fp32"])
def test_row_sharded_matrix_matches_whole(gemm, cuda_dev):
    from ltq_research_b200.liqk_v2 import _quantize_matrix_core
    from ltq_research_b200.shard import row_ranges
    W, H = synth(240, 512, 21)
    W, H = W.to(cuda_dev), H.to(cuda_dev)
    whole = _quantize_matrix_core(W, H, "TCQ3X", want_pack=True, gemm=gemm)
    rr = row_ranges(240, 2)
    assert rr == [(0, 128), (128, 240)]
    parts = _run_shards(lambda k, red: _quantize_matrix_core(W[rr[k][0]:rr[k][1]], H, "TCQ3X", want_pack=True,
                                                             gemm=gemm, row_reduce=red), 2)
    torch.cuda.synchronize()
    # every shard reaches the same suh and the same totals
    assert torch.equal(parts[0]["qdata"]["suh"], parts[1]["qdata"]["suh"])
    assert torch.equal(parts[0]["num"], parts[1]["num"]) and torch.equal(parts[0]["den"], parts[1]["den"])
    assert int(parts[0]["chol_info"]) == 0 and int(parts[1]["chol_info"]) == 0
    # against the whole matrix: the row sums only change order
    suh_eq = (parts[0]["qdata"]["suh"] == whole["qdata"]["suh"]).float().mean().item()
    assert suh_eq >= 0.99, suh_eq
    idx = torch.cat([p["pack"]["idx"] for p in parts])
    idx_eq = (idx == whole["pack"]["idx"]).float().mean().item()
    assert idx_eq >= 0.97, idx_eq
    rel_s = (parts[0]["num"] / parts[0]["den"]).item()
    rel_w = (whole["num"] / whole["den"]).item()
    assert abs(rel_s - rel_w) <= 0.01 * rel_w, (rel_s, rel_w)


def test_row_sharded_batch_merge_matvec(cuda_dev):
    from ltq_research_b200.batch import quantize_matrices
    from ltq_research_b200.formats import load_formats
    from ltq_research_b200.ltq_file import matvec
    from ltq_research_b200.shard import merge_row_shards, row_ranges
    fm = load_formats(["TCQ3X", "TCQ25X"], cuda_dev)
    mats = [synth(96, 512, 31), synth(64, 768, 32)]
    specs = ["TCQ3X", "TCQ25X"]
    ranges = [row_ranges(W.shape[0], 2) for W, _ in mats]

    def shard(k, red):
        jobs = [(W[rr[k][0]:rr[k][1]].to(cuda_dev), H.to(cuda_dev), sp) for (W, H), rr, sp in zip(mats, ranges, specs)]
        return quantize_matrices(jobs, n_streams=2, ltq_formats=fm, pack=False, row_reduce=red)
    parts = _run_shards(shard, 2)
    torch.cuda.synchronize()
    g = torch.Generator(device=cuda_dev).manual_seed(5)
    for j in range(len(mats)):
        lts = [parts[k][j]["ltq"] for k in range(2)]
        m = merge_row_shards(lts)
        K = m["suh"].shape[0]
        data = torch.zeros(((m["data"].numel() + 63) // 64) * 64, dtype=torch.uint8, device=cuda_dev)
        data[: m["data"].numel()] = m["data"]
        x = torch.randn(K, device=cuda_dev, generator=g)
        y = matvec(data, m["slices"], list(fm.values()), m["d_row"], m["e"], m["suh"], x)
        ys = []
        for lt in lts:
            d = torch.zeros(((lt["data"].numel() + 63) // 64) * 64, dtype=torch.uint8, device=cuda_dev)
            d[: lt["data"].numel()] = lt["data"]
            ys.append(matvec(d, lt["slices"], list(fm.values()), lt["d_row"], lt["e"], lt["suh"], x))
        assert torch.equal(y, torch.cat(ys))
        assert abs(parts[0][j]["rel_loss"] - parts[1][j]["rel_loss"]) == 0.0
