"""Quantizing a model across the GPUs of one node: one process per GPU, matrices sharded across ranks, no collective on
the data path, one gather of the packed .ltq results at the end.

Matrices are independent given their Hessian (the LDLQ feedback is row-local and the refits are per matrix,
src/liqk_v2.py:956-1180), so a model shards by whole matrices: `assign` gives every rank a share of the matrices,
longest first onto the least-loaded rank (the cost model of batch.estimated_seconds), deterministically, so every rank
computes the same assignment without communicating.  Each rank quantizes its share with batch.quantize_matrices.
`gather_ltq` then brings every rank's packed tensors (data, slice table, d_row, e, suh) to one rank with
torch.distributed — NCCL between the GPUs of a B200 node (NVLink / NVSwitch), gloo on CPU for the tests — as one
all-gather of sizes and headers followed by one gather of a flat byte buffer per rank.

Matrices can also be split by rows (many matrices of one shape, such as MoE experts, or fewer matrices than ranks):
`row_ranges` gives every rank a contiguous range of 16-row tiles, each rank quantizes its rows of every matrix with
batch.quantize_matrices(..., row_reduce=nccl_row_reduce(group)) — H is the whole matrix's Hessian on every rank, the
quantizer is row-local except for sums over rows (the column statistics of suh, the refit's Gram matrix and right-hand
side, its two losses, the final loss), which row_reduce adds up across the ranks, five all-reduces per matrix, so all
ranks reach the same suh — and `merge_row_shards` joins the shards' packed fields into one matrix.
"""
from __future__ import annotations

from typing import Dict, List, Optional, Sequence, Tuple

import torch

from .batch import estimated_seconds


def assign(shapes: Sequence[Tuple[int, int, object]], world: int) -> List[List[int]]:
    """Indices of `shapes` ((M, K, spec) per matrix) for each of `world` ranks: longest-processing-time first onto the
    least-loaded rank; ties go to the lower rank.  Deterministic: every rank computes the same lists."""
    if world < 1:
        raise ValueError("world must be >= 1")
    cost = [estimated_seconds(M, K, sp) for M, K, sp in shapes]
    order = sorted(range(len(shapes)), key=lambda i: (-cost[i], i))
    load = [0.0] * world
    out: List[List[int]] = [[] for _ in range(world)]
    for i in order:
        r = min(range(world), key=lambda k: (load[k], k))
        load[r] += cost[i]
        out[r].append(i)
    for lst in out:
        lst.sort()
    return out


def row_ranges(M: int, world: int, multiple: int = 16) -> List[Tuple[int, int]]:
    """Contiguous row ranges [r0, r1) of an M-row matrix for `world` ranks, for matrices sharded by rows (many experts
    of one shape, or too few matrices per rank): every boundary a multiple of `multiple` (16, the Viterbi tile's
    height), sizes within one multiple of each other, earlier ranks taking the larger ones.  Every rank gets rows
    (every rank takes part in the row sums): M >= world * multiple."""
    if world < 1 or multiple < 1 or M % multiple or M < world * multiple:
        raise ValueError(f"row_ranges: M = {M} must be a multiple of {multiple} and at least {world} x {multiple}")
    units = M // multiple
    q, rem = divmod(units, world)
    out, r0 = [], 0
    for k in range(world):
        n = (q + (1 if k < rem else 0)) * multiple
        out.append((r0, r0 + n))
        r0 += n
    return out


def nccl_row_reduce(group=None):
    """The row_reduce of batch.quantize_matrices for ranks that split matrices by rows: an in-place sum over `group`
    (NCCL between the GPUs of a node), issued on the current stream."""
    import torch.distributed as dist

    def reduce(t: torch.Tensor):
        dist.all_reduce(t, op=dist.ReduceOp.SUM, group=group)
    return reduce


def _region_words(f) -> List[int]:
    """u16 words per tile of the four SoA regions of a packed slice: code bits, bit planes, low bits, gain bits
    (src/ltq_file.py:79-102; each region starts on a 64-byte boundary, tiles by row group then 16-column block)."""
    if getattr(f, "frac", 0) == 3:
        raise ValueError(f"{f.name}: the EQ formats have no .ltq encoding")
    return [16, 16 * max(f.K - 2, 0), f.lsb_words() if f.K > 1 else 0, f.gain_words()]


def _slice_nbytes(rows: int, K: int, f, align: int = 64) -> int:
    off = 0
    for n in _region_words(f):
        off = -(-off // align) * align + 2 * (rows // 16) * (K // 16) * n
    return off


def _coalesce(pieces: Sequence[Tuple[torch.Tensor, int]], K: int, f, align: int = 64) -> torch.Tensor:
    """The bytes of one slice of format f made of consecutive slices [(bytes, rows)] of that format: region by region,
    the pieces' tiles one after the other (their row groups continue), as if packed in one piece."""
    out, off, src = [], 0, [0] * len(pieces)
    for n in _region_words(f):
        pad = (-off) % align
        if pad:
            out.append(torch.zeros(pad, dtype=torch.uint8, device=pieces[0][0].device))
            off += pad
        for i, (d, rows) in enumerate(pieces):
            s0 = -(-src[i] // align) * align
            nb = 2 * (rows // 16) * (K // 16) * n
            out.append(d[s0:s0 + nb])
            src[i] = s0 + nb
            off += nb
    return torch.cat(out) if out else torch.empty(0, dtype=torch.uint8, device=pieces[0][0].device)


def merge_row_shards(parts: Sequence[dict], align: int = 64, formats: Optional[Sequence] = None) -> dict:
    """One matrix's .ltq fields from the fields of its consecutive row shards (in row order, as quantize_matrices
    returns them under "ltq", on one device or on the host): d_row and e stacked; suh must be the same in every shard
    (the row-sharded refit makes it so).  Without `formats` the shards' packed data are concatenated, every shard
    starting on an `align`-byte boundary, slice rows and offsets moved accordingly.  With `formats` (the format of each
    slice index, as given to quantize_matrices' ltq_formats), a shard's last slice and the next shard's first slice
    become one slice when they have the same format (the cut between shards fell inside one row slice of the
    matrix), packed region by region; slices inside one shard stay as they are.  When every shard was quantized with
    the matrix's row slices cut at the shard boundaries, the result is laid out exactly as the whole matrix packed at
    once."""
    if not parts:
        raise ValueError("merge_row_shards: no shards")
    suh = parts[0]["suh"]
    for p in parts:
        if not torch.equal(p["suh"].to(suh.device), suh):
            raise ValueError("merge_row_shards: the shards disagree on suh")
    dev = parts[0]["data"].device
    d_row = torch.cat([p["d_row"] for p in parts])
    e = torch.cat([p["e"] for p in parts])
    if formats is None:
        data, slices, row0, off = [], [], 0, 0
        for p in parts:
            pad = (-off) % align
            if pad:
                data.append(torch.zeros(pad, dtype=torch.uint8, device=p["data"].device))
                off += pad
            for r0, r1, fi, o in p["slices"]:
                slices.append([r0 + row0, r1 + row0, fi, o + off])
            data.append(p["data"].reshape(-1))
            off += int(p["data"].numel())
            row0 += int(p["d_row"].shape[0])
        return {"data": torch.cat([d.to(dev) for d in data]), "slices": slices, "d_row": d_row, "e": e, "suh": suh}
    K = int(suh.numel())
    runs: List[list] = []  # [r0, r1, fi, [(bytes, rows), ...]]
    row0 = 0
    for p in parts:
        flat = p["data"].reshape(-1).to(dev)
        for k, (r0, r1, fi, o) in enumerate(sorted(p["slices"], key=lambda x: x[0])):
            piece = (flat[o:o + _slice_nbytes(r1 - r0, K, formats[fi], align)], r1 - r0)
            # only a shard's first slice may continue the previous shard's last one
            if k == 0 and runs and runs[-1][2] == fi and runs[-1][1] == r0 + row0:
                runs[-1][1] = r1 + row0
                runs[-1][3].append(piece)
            else:
                runs.append([r0 + row0, r1 + row0, fi, [piece]])
        row0 += int(p["d_row"].shape[0])
    data, slices, off = [], [], 0
    for r0, r1, fi, pieces in runs:
        pad = (-off) % align
        if pad:
            data.append(torch.zeros(pad, dtype=torch.uint8, device=dev))
            off += pad
        b = _coalesce(pieces, K, formats[fi], align)
        slices.append([r0, r1, fi, off])
        data.append(b)
        off += int(b.numel())
    return {"data": torch.cat(data), "slices": slices, "d_row": d_row, "e": e, "suh": suh}


_FIELDS = ("data", "d_row", "e", "suh")


def _pack_bytes(items: Dict[int, dict], device: torch.device) -> Tuple[torch.Tensor, list]:
    """Flatten {matrix index: ltq dict} into one uint8 buffer on `device` and a small header (index, field shapes /
    dtypes, slice table)."""
    parts, header = [], []
    for idx in sorted(items):
        d = items[idx]
        ent = {"index": int(idx), "slices": [list(map(int, s)) for s in d["slices"]], "fields": []}
        for k in _FIELDS:
            t = d[k].detach().contiguous()
            b = t.view(torch.uint8).reshape(-1) if t.numel() else torch.empty(0, dtype=torch.uint8, device=t.device)
            ent["fields"].append([k, str(t.dtype).replace("torch.", ""), list(t.shape), int(b.numel())])
            parts.append(b.to(device))
        header.append(ent)
    buf = torch.cat(parts) if parts else torch.empty(0, dtype=torch.uint8, device=device)
    return buf, header


def _unpack_bytes(buf: torch.Tensor, header: list) -> Dict[int, dict]:
    """Inverse of _pack_bytes.  Byte fields (the packed tiles, most of the volume) are views into `buf`; the small
    typed fields are copied, since their offsets in the flat buffer need not be aligned to their element size."""
    out, off = {}, 0
    for ent in header:
        d = {"slices": ent["slices"]}
        for k, dt, shape, n in ent["fields"]:
            b = buf[off:off + n]
            d[k] = (b if dt == "uint8" else b.clone().view(getattr(torch, dt))).reshape(shape)
            off += n
        out[ent["index"]] = d
    return out


def gather_ltq(local: Dict[int, dict], dst: int = 0, group=None) -> Optional[Dict[int, dict]]:
    """Gather every rank's packed .ltq tensors ({matrix index: {"data", "slices", "d_row", "e", "suh"}}) on rank
    `dst` as CPU tensors; other ranks get None.  Collective: every rank of `group` must call it, in the same order as
    its other collectives.  The byte buffers travel as uint8 tensors on the backend's device (CUDA for NCCL, CPU for
    gloo); sizes and headers with one all-gather of Python objects."""
    import torch.distributed as dist
    world = dist.get_world_size(group)
    rank = dist.get_rank(group)
    dev = torch.device("cuda", torch.cuda.current_device()) if dist.get_backend(group) == "nccl" else torch.device("cpu")
    buf, header = _pack_bytes(local, dev)
    meta = [None] * world
    dist.all_gather_object(meta, (int(buf.numel()), header), group=group)
    n_max = max(max(m[0] for m in meta), 1)
    send = torch.zeros(n_max, dtype=torch.uint8, device=dev)
    send[: buf.numel()] = buf
    if rank == dst:
        recv = [torch.empty(n_max, dtype=torch.uint8, device=dev) for _ in range(world)]
        dist.gather(send, recv, dst=dst, group=group)
        host = []
        for r in range(world):  # device buffers come back through pinned memory, all copies in flight at once
            if recv[r].is_cuda:
                h = torch.empty(meta[r][0], dtype=torch.uint8, pin_memory=True)
                h.copy_(recv[r][: meta[r][0]], non_blocking=True)
            else:
                h = recv[r][: meta[r][0]]
            host.append(h)
        if dev.type == "cuda":
            torch.cuda.current_stream(dev).synchronize()
        out: Dict[int, dict] = {}
        for r in range(world):
            out.update(_unpack_bytes(host[r], meta[r][1]))
        return out
    dist.gather(send, None, dst=dst, group=group)
    return None
