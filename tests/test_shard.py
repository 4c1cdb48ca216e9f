"""Sharding across ranks (ltq_research_b200.shard) on CPU: the longest-first assignment, and the end-of-run gather of
the packed .ltq tensors over a world-size-2 gloo process group (the same collective code runs over NCCL on the GPUs);
a rank that leaves before the gather makes the other rank's gather fail within the process-group timeout instead of
waiting for ever."""
import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

from ltq_research_b200.batch import estimated_seconds
from ltq_research_b200.shard import assign

LAYER = [(3072, 3072), (1024, 3072), (1024, 3072), (3072, 3072), (8192, 3072), (8192, 3072), (3072, 8192)]


def _shapes(n_layers=4):
    return [(M, K, "TCQ3X" if l % 2 == 0 else "TCQ25X") for l in range(n_layers) for M, K in LAYER]


def test_assign_is_complete_deterministic_and_balanced():
    shapes = _shapes()
    for world in (1, 2, 3, 8):
        a = assign(shapes, world)
        assert a == assign(shapes, world)
        assert sorted(i for lst in a for i in lst) == list(range(len(shapes)))
        cost = [estimated_seconds(*s) for s in shapes]
        loads = [sum(cost[i] for i in lst) for lst in a]
        assert max(loads) <= sum(cost) / world + max(cost) + 1e-12
    with pytest.raises(ValueError):
        assign(shapes, 0)


def _fake_ltq(i):
    g = torch.Generator().manual_seed(i)
    M, K = 16 * (1 + i % 3), 256
    return {"data": torch.randint(0, 256, (1000 + 64 * i,), generator=g, dtype=torch.uint8),
            "slices": [[0, M, i % 2, 0]],
            "d_row": torch.randn(M, generator=g).to(torch.float16),
            "e": torch.randint(-16, 16, (M, K // 256), generator=g, dtype=torch.int8),
            "suh": torch.randn(K, generator=g).to(torch.float16)}


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, mode, q):
    import datetime
    import torch.distributed as dist
    from ltq_research_b200.shard import gather_ltq
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=5))
    mine = assign(_shapes(2), world)[rank]
    if mode == "reduce":  # the row sums of row-sharded matrices, over the same collective
        from ltq_research_b200.shard import nccl_row_reduce
        t = torch.arange(5, dtype=torch.float32) * (rank + 1)
        nccl_row_reduce()(t)
        q.put((rank, "ok" if torch.equal(t, torch.arange(5, dtype=torch.float32) * 3) else "mismatch", None))
        dist.destroy_process_group()
        return
    if mode == "leave" and rank == 1:
        os._exit(0)  # leaves between steps, with no collective in flight
    try:
        out = gather_ltq({i: _fake_ltq(i) for i in mine}, dst=0)
    except Exception as e:  # noqa: BLE001
        q.put((rank, "error", type(e).__name__))
        return
    if rank == 0:
        ok = sorted(out) == list(range(len(_shapes(2))))
        for i, d in out.items():
            w = _fake_ltq(i)
            ok = ok and d["slices"] == w["slices"] and all(torch.equal(d[k], w[k]) for k in ("data", "d_row", "e", "suh"))
        q.put((rank, "ok" if ok else "mismatch", None))
    else:
        q.put((rank, "ok" if out is None else "unexpected", None))
    dist.destroy_process_group()


def _run(mode):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, mode, q)) for r in range(2)]
    for p in procs:
        p.start()
    n = 1 if mode == "leave" else 2
    res = sorted(q.get(timeout=120) for _ in range(n))
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    return res


def test_gather_ltq_world2_gloo():
    assert _run("ok") == [(0, "ok", None), (1, "ok", None)]


def test_gather_ltq_peer_leaves_gloo():
    res = _run("leave")
    assert res[0][0] == 0 and res[0][1] == "error", res


def test_row_reduce_world2_gloo():
    assert _run("reduce") == [(0, "ok", None), (1, "ok", None)]


def test_row_ranges():
    from ltq_research_b200.shard import row_ranges
    for M, world in ((96, 4), (1024, 3), (8192, 8), (16, 1), (48, 3)):
        rr = row_ranges(M, world)
        assert rr[0][0] == 0 and rr[-1][1] == M and len(rr) == world
        assert all(a1 == b0 for (_, a1), (b0, _) in zip(rr, rr[1:]))
        sizes = [r1 - r0 for r0, r1 in rr]
        assert all(n > 0 and n % 16 == 0 for n in sizes) and max(sizes) - min(sizes) <= 16
        assert sizes == sorted(sizes, reverse=True)
    for M, world in ((100, 2), (32, 3), (0, 1)):
        with pytest.raises(ValueError):
            row_ranges(M, world)


def test_merge_row_shards():
    """Shards' packed fields joined into one matrix: every shard's bytes start on a 64-byte boundary, slice rows and
    offsets move with them, d_row / e stack, and shards that disagree on suh are refused."""
    from ltq_research_b200.shard import merge_row_shards
    parts = [_fake_ltq(i) for i in (0, 1, 2)]
    for p in parts[1:]:
        p["suh"] = parts[0]["suh"].clone()
    parts[1]["slices"] = [[0, 8, 0, 0], [8, 32, 1, 64]]
    m = merge_row_shards(parts)
    rows = [0, 16, 48]
    offs, off = [], 0
    for p in parts:
        off += (-off) % 64
        offs.append(off)
        off += p["data"].numel()
    assert m["data"].numel() == off
    for p, r0, o in zip(parts, rows, offs):
        assert torch.equal(m["data"][o:o + p["data"].numel()], p["data"])
    assert m["slices"] == [[0, 16, 0, 0], [16, 24, 0, offs[1]], [24, 48, 1, offs[1] + 64], [48, 96, 0, offs[2]]]
    assert torch.equal(m["d_row"], torch.cat([p["d_row"] for p in parts]))
    assert torch.equal(m["e"], torch.cat([p["e"] for p in parts]))
    assert torch.equal(m["suh"], parts[0]["suh"])
    parts[2]["suh"] = parts[2]["suh"] + 1
    with pytest.raises(ValueError):
        merge_row_shards(parts)


def _pack_fmts(names):
    import numpy as np
    from ltq_research_b200.formats import load_formats
    from tests.test_oracle_golden import _ltq_fmt
    fm = load_formats(names, "cpu")
    return list(fm.values()), [_ltq_fmt(n, np.asarray(fm[n].gain_tab, np.float32)) for n in names]


def test_slice_region_sizes_match_library():
    """The region arithmetic of the coalescing merge gives the library's slice size for every .ltq format."""
    from ltq_research_b200 import _lib
    from ltq_research_b200.formats import TCQ_CONFIG
    from ltq_research_b200.shard import _slice_nbytes
    names = [n for n, c in TCQ_CONFIG.items() if c.get("tb") and int(c.get("pp", 0)) != 3]
    fmts, _ = _pack_fmts(names)
    for f in fmts:
        for R, K in ((16, 256), (48, 512), (96, 768), (208, 3072)):
            assert _slice_nbytes(R, K, f) == _lib.lib().ltq_slice_bytes(R, K, f.K, f.frac, f.h, f.sub), (f.name, R, K)


def test_merge_row_shards_coalesces_to_whole_packing():
    """Row shards packed separately and merged with their formats give the bytes and slice table of the whole matrix
    packed at once (the oracle's restatement of the reference's pack_slice): one format split 48 / 48 rows, and a
    two-format matrix whose second format spans the shard boundary."""
    import numpy as np
    from oracle import oracle as O
    from ltq_research_b200.shard import merge_row_shards
    fmts, ofmts = _pack_fmts(["TCQ3X", "TCQ25X"])
    g = np.random.default_rng(3)
    K = 512

    def codes(rows, of):
        idx = g.integers(0, of.n_labels * of.U, (rows, K))
        gi = g.integers(0, max(1 << of.h, 1), (rows, K))
        return idx, gi

    def packed(idx, gi, fi):
        return torch.from_numpy(np.frombuffer(O.pack_slice(idx, gi, ofmts[fi]), np.uint8).copy())

    def part(slices, rows):  # slices: [(r0, r1, fi, idx, gi)] -> ltq fields with 64-byte aligned slices
        data, table, off = [], [], 0
        for r0, r1, fi, idx, gi in slices:
            pad = (-off) % 64
            data.append(torch.zeros(pad, dtype=torch.uint8))
            off += pad
            b = packed(idx, gi, fi)
            table.append([r0, r1, fi, off])
            data.append(b)
            off += b.numel()
        return {"data": torch.cat(data), "slices": table, "d_row": torch.ones(rows, dtype=torch.float16),
                "e": torch.zeros(rows, K // 256, dtype=torch.int8), "suh": torch.ones(K, dtype=torch.float16)}

    # one format, two shards of 48 rows
    idx, gi = codes(96, ofmts[0])
    m = merge_row_shards([part([(0, 48, 0, idx[:48], gi[:48])], 48), part([(0, 48, 0, idx[48:], gi[48:])], 48)],
                         formats=fmts)
    assert m["slices"] == [[0, 96, 0, 0]]
    assert torch.equal(m["data"], packed(idx, gi, 0))
    # rows 0-16 TCQ3X, rows 16-96 TCQ25X; shards [0, 48) and [48, 96)
    i0, g0 = codes(16, ofmts[0])
    i1, g1 = codes(80, ofmts[1])
    a = part([(0, 16, 0, i0, g0), (16, 48, 1, i1[:32], g1[:32])], 48)
    b = part([(0, 48, 1, i1[32:], g1[32:])], 48)
    m = merge_row_shards([a, b], formats=fmts)
    whole = part([(0, 16, 0, i0, g0), (16, 96, 1, i1, g1)], 96)
    assert m["slices"] == whole["slices"]
    assert torch.equal(m["data"], whole["data"])
    # two slices of one format inside a shard stay two slices (as the whole matrix packed with those row slices)
    j0, h0 = codes(32, ofmts[0])
    j1, h1 = codes(16, ofmts[0])
    j2, h2 = codes(48, ofmts[0])
    a = part([(0, 32, 0, j0, h0), (32, 48, 0, j1, h1)], 48)
    b = part([(0, 48, 0, j2, h2)], 48)
    m = merge_row_shards([a, b], formats=fmts)
    whole = part([(0, 32, 0, j0, h0), (32, 96, 0, np.concatenate([j1, j2]), np.concatenate([h1, h2]))], 96)
    assert m["slices"] == whole["slices"] == [[0, 32, 0, 0], [32, 96, 0, m["slices"][1][3]]]
    assert torch.equal(m["data"], whole["data"])
