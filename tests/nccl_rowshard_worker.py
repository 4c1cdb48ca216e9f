"""Worker of tests/test_rowshard_nccl_gpu.py, one process per GPU under torchrun (NCCL over NVLink): matrices split by
rows across the ranks (shard.row_ranges), quantized with the row sums all-reduced (shard.nccl_row_reduce), the packed
shards gathered to rank 0 (shard.gather_ltq) and merged (shard.merge_row_shards); rank 0 also quantizes every matrix
whole and writes the comparison to the JSON file named by argv[1].

    torchrun --nproc-per-node 2 --master-addr 127.0.0.1 tests/nccl_rowshard_worker.py out.json
"""
import json
import os
import sys
from datetime import timedelta
from pathlib import Path

import torch
import torch.distributed as dist

ROOT = Path(__file__).resolve().parent.parent
sys.path.insert(0, str(ROOT))

from ltq_research_b200.batch import quantize_matrices  # noqa: E402
from ltq_research_b200.formats import load_formats  # noqa: E402
from ltq_research_b200.ltq_file import matvec  # noqa: E402
from ltq_research_b200.shard import gather_ltq, merge_row_shards, nccl_row_reduce, row_ranges  # noqa: E402
from tests.golden.matrix_inputs import synth  # noqa: E402

CASES = [(240, 512, "TCQ3X", 21), (96, 768, "TCQ275X", 22), (512, 1024, "TCQ25X", 23)]


def _padded(t, dev):
    d = torch.zeros(((t.numel() + 63) // 64) * 64, dtype=torch.uint8, device=dev)
    d[: t.numel()] = t.to(dev)
    return d


def main():
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    dev = torch.device("cuda", int(os.environ.get("LOCAL_RANK", "0")))
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=dev)
    fm = load_formats(sorted({c[2] for c in CASES}), dev)
    names = list(fm)
    mats = [synth(M, K, seed) for M, K, _, seed in CASES]  # CPU generator: the same inputs on every rank
    rr = [row_ranges(M, world) for M, _, _, _ in CASES]
    jobs = [(W[r[rank][0]:r[rank][1]].to(dev), H.to(dev), sp) for (W, H), r, (_, _, sp, _) in zip(mats, rr, CASES)]
    res = quantize_matrices(jobs, ltq_formats=fm, pack=False, row_reduce=nccl_row_reduce())
    got = gather_ltq({j * world + rank: r["ltq"] for j, r in enumerate(res)}, dst=0)
    rels = torch.tensor([r["rel_loss"] for r in res], dtype=torch.float64, device=dev)
    allrel = [torch.zeros_like(rels) for _ in range(world)]
    dist.all_gather(allrel, rels)
    out = {"world": world, "cases": []}
    if rank == 0:
        whole = quantize_matrices([(W.to(dev), H.to(dev), sp) for (W, H), (_, _, sp, _) in zip(mats, CASES)],
                                  ltq_formats=fm, pack=False)
        g = torch.Generator(device=dev).manual_seed(9)
        for j, (M, K, sp, _) in enumerate(CASES):
            shards = [got[j * world + r] for r in range(world)]
            m = merge_row_shards(shards, formats=[fm[n] for n in names])
            w = whole[j]["ltq"]
            x = torch.randn(K, device=dev, generator=g)
            y = matvec(_padded(m["data"], dev), m["slices"], [fm[n] for n in names], m["d_row"].to(dev),
                       m["e"].to(dev), m["suh"].to(dev), x)
            ys = torch.cat([matvec(_padded(s["data"], dev), s["slices"], [fm[n] for n in names], s["d_row"].to(dev),
                                   s["e"].to(dev), s["suh"].to(dev), x) for s in shards])
            yw = matvec(_padded(w["data"], dev), w["slices"], [fm[n] for n in names], w["d_row"], w["e"], w["suh"], x)
            out["cases"].append({
                "shape": [M, K], "format": sp,
                "rel_loss_ranks": [float(a[j]) for a in allrel], "rel_loss_whole": whole[j]["rel_loss"],
                "suh_equal_whole": float((m["suh"].to(dev) == w["suh"]).float().mean()),
                "merged_slices": m["slices"], "whole_slices": w["slices"],
                "merged_bytes": int(m["data"].numel()), "whole_bytes": int(w["data"].numel()),
                "merged_matvec_equals_shards": bool(torch.equal(y, ys)),
                "matvec_rel_diff_whole": float((y - yw).norm() / yw.norm())})
        Path(sys.argv[1]).write_text(json.dumps(out, indent=1))
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
