"""Quantizing a model across the GPUs of one node: one process per GPU, matrices sharded across ranks, no collective on
the data path, one gather of the packed .ltq results at the end.

Matrices are independent given their Hessian (the LDLQ feedback is row-local and the refits are per matrix,
src/liqk_v2.py:956-1180), so a model shards by whole matrices: `assign` gives every rank a share of the matrices,
longest first onto the least-loaded rank (the cost model of batch.estimated_seconds), deterministically, so every rank
computes the same assignment without communicating.  Each rank quantizes its share with batch.quantize_matrices.
`gather_ltq` then brings every rank's packed tensors (data, slice table, d_row, e, suh) to one rank with
torch.distributed — NCCL between the GPUs of a B200 node (NVLink / NVSwitch), gloo on CPU for the tests — as one
all-gather of sizes and headers followed by one gather of a flat byte buffer per rank.
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
