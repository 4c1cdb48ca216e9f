"""Concurrent quantization of many matrices on one B200.

The LDLQ sweep of one matrix is a chain of K/256 dependent block launches, each of M/16 CTAs that walk their rows
through 16 sub-blocks one after another; a single matrix therefore occupies a fraction of the 148 SMs for a time set
by its column count.  Independent matrices (the layers of a model, the experts of an MoE) are what fills the GPU: this
driver runs each matrix's whole quantize_matrix_liqk_v2 computation (rotation, Hessian factorisation, LDLQ, refits,
PACK fields) on one of several CUDA streams, with no host synchronisation until every matrix has been issued.  Matrices
are assigned longest-first to the least-loaded stream.  Results are the reference function's, bit for bit: the same
kernels and torch operations run on every stream.

The reference quantizes matrices one at a time (src/hybrid_quant.py, src/streaming_quant.py call
quantize_matrix_liqk_v2 per matrix, optionally from LIQK_PAR host threads); this is the single-process B200 form.
"""
from __future__ import annotations

from typing import Dict, List, Optional, Sequence, Tuple, Union

import torch

from . import _lib
from .formats import TCQ_CONFIG
from .liqk_v2 import _quantize_matrix_steps, check_gemm_errors

Spec = Union[str, Sequence[Tuple[int, int, str]]]


def _specs(spec: Spec) -> List[str]:
    return [spec] if isinstance(spec, str) else [sp for _, _, sp in spec]


def estimated_seconds(M: int, K: int, spec: Spec) -> float:
    """Rough B200 time of one matrix, for the longest-first assignment: the Viterbi at ~1.1 G weights/s for a four-slot
    plain format (scaled by slots x parity classes) plus the fp32 factorisations and refit products (~K^3 and M K^2)."""
    t = 0.0
    for sp in _specs(spec):
        c = TCQ_CONFIG[sp]
        g = 1 << c["h"]
        if c.get("n_cand"):
            g = min(g, int(c["n_cand"]))
        t += M * K * g * (2 if c.get("pp") else 1) / 4.0 / 1.1e9 / len(_specs(spec))
    return t + (3.0 * K ** 3 + 8.0 * M * K * K) / 50e12


_STREAMS: Dict[tuple, List[torch.cuda.Stream]] = {}


def _streams(dev: torch.device, n: int, role: str = "lane") -> List[torch.cuda.Stream]:
    """The driver's CUDA streams on `dev`, created once and reused by every call: the caching allocator keeps freed
    blocks per stream, so reusing the streams lets each call reuse the memory the previous calls cached (fresh streams
    on every call would allocate anew and grow the reserved memory call after call)."""
    key = (str(dev), n, role)
    if key not in _STREAMS:
        _STREAMS[key] = [torch.cuda.Stream(dev) for _ in range(n)]
    return _STREAMS[key]


def _record(obj, stream: torch.cuda.Stream):
    if torch.is_tensor(obj):
        if obj.is_cuda:
            obj.record_stream(stream)
    elif isinstance(obj, dict):
        for v in obj.values():
            _record(v, stream)
    elif isinstance(obj, (list, tuple)):
        for v in obj:
            _record(v, stream)


@torch.no_grad()
def quantize_matrices(jobs: Sequence[Tuple[torch.Tensor, torch.Tensor, Spec]], seed: int = 1337, damp: float = 0.02,
                      n_streams: int = 8, pack: bool = True, keep_w_hat: bool = False,
                      device: Optional[torch.device] = None, on_issued=None, ltq_formats: Optional[Dict] = None,
                      to_host: bool = False, gemm: str = "bf16x6", order: str = "lpt",
                      prep_ahead: bool = False, row_reduce=None) -> List[Dict]:
    """Quantize every (W [M, K], H [K, K], spec) of `jobs` as quantize_matrix_liqk_v2(W, H, spec, seed, damp) would,
    concurrently on `n_streams` CUDA streams.  W / H may be CUDA tensors or (pinned) host tensors, which are copied to
    the device on the matrix's stream.  Returns, per job: {"qdata", "pack" (the PACK["matrix"] fields, device tensors)
    when pack, "W_hat" when keep_w_hat, "rel_loss" (float)}.  One host synchronisation, after the last job is issued;
    on_issued(i), if given, is called after job i has been issued (for overlapping host work).
    ltq_formats ({name: LtqFormat}, e.g. formats.load_formats(menu, device)): each matrix is also packed into its .ltq
    data tensor on the device and verified there (ltq_file.pack_matrix_device), on the matrix's stream; the result
    gains "ltq": {"data" (uint8), "slices" ([r0, r1, format, offset] rows, format = position in ltq_formats),
    "d_row" fp16, "e" int8, "suh" fp16}, as pinned host tensors when to_host.  Raises torch.linalg.LinAlgError if a
    damped Hessian is not positive definite, RuntimeError if a packed matrix does not decode to its tile values.
    gemm: the mode of the LDLQ inter-block update and refit products (liqk_v2.GEMM_MODES): "bf16x6" (default) runs
    them as fp32-accurate split products on the tensor cores; "fp32" reproduces quantize_matrix_liqk_v2 bit for bit.
    order: the order in which the streams take jobs — "lpt" (default) longest estimated time first, "given" as listed.
    prep_ahead: issue each stream's next job's Hessian preparation on a second stream while the current job runs
    (measured on the bench's layer set: no gain once the device is saturated, so off by default).  The results depend
    on neither.
    row_reduce: every job is this rank's row slice of a matrix whose rows are split across ranks (shard.row_ranges),
    and row_reduce(t) sums t in place over those ranks (shard.nccl_row_reduce); see liqk_v2._quantize_matrix_steps.
    Every rank must pass the same matrices in the same order; the jobs are then taken as given, so that all ranks
    issue their sums in the same order whatever their slices' sizes."""
    if not jobs:
        return []
    dev = torch.device(device) if device is not None else None
    for W, H, _ in jobs:
        for t in (W, H):
            if t.is_cuda:
                dev = dev or t.device
    if dev is None:
        dev = torch.device("cuda", torch.cuda.current_device())
    if dev.type != "cuda":
        raise RuntimeError("quantize_matrices: a CUDA device is required; there is no CPU path")
    _lib.lib()
    main = torch.cuda.current_stream(dev)
    streams = _streams(dev, max(1, n_streams))
    cost = [estimated_seconds(W.shape[0], W.shape[1], sp) for W, _, sp in jobs]
    if row_reduce is not None:
        order = "given"
    if order == "lpt":
        pending = sorted(range(len(jobs)), key=lambda i: -cost[i])[::-1]  # pop() takes the longest remaining job
    elif order == "given":
        pending = list(range(len(jobs)))[::-1]  # pop() takes the jobs in the order given
    else:
        raise ValueError(f"order {order!r}: expected 'lpt' or 'given'")
    out: List[Optional[Dict]] = [None] * len(jobs)
    preps = _streams(dev, max(1, n_streams), "prep") if prep_ahead else streams

    def start(k: int) -> tuple:
        """Issue the next job's Hessian preparation (the generator's first step) on lane k's preparation stream."""
        i = pending.pop()
        W, H, sp = jobs[i]
        p, s = preps[k], streams[k]
        p.wait_stream(main)
        with torch.cuda.stream(p):
            Wd = W.to(dev, non_blocking=True) if not W.is_cuda else W
            Hd = H.to(dev, non_blocking=True) if not H.is_cuda else H
            for t in (W, H):
                if t.is_cuda:
                    t.record_stream(p)
                    t.record_stream(s)
            gen = _quantize_matrix_steps(Wd, Hd, sp, seed, damp, None, pack or ltq_formats is not None, None, gemm,
                                         row_reduce)
            next(gen)
            ev = torch.cuda.Event()
            ev.record(p)
        if p is not s:
            # what the preparation leaves to the later steps was allocated on p and is used and freed on s: the
            # allocator must not hand that memory to p again before s's work on it has run
            _record(dict(gen.gi_frame.f_locals), s)
        return i, gen, ev

    # every lane: one job in its block / refit steps on the lane's stream and, with prep_ahead, the next job's
    # preparation already issued on the lane's preparation stream (its single-CTA Cholesky leaves and
    # triangular-inverse kernels are latency-bound and overlap the other jobs' blocks).  Each round advances every
    # lane's current job by one step (one 256-column block, or the refits), so that every stream keeps work queued.
    cur: List[Optional[tuple]] = [None] * len(streams)
    nxt: List[Optional[tuple]] = [None] * len(streams)
    while pending or any(c is not None for c in cur) or any(n is not None for n in nxt):
        for k, s in enumerate(streams):
            if cur[k] is None:
                if nxt[k] is None and pending:
                    nxt[k] = start(k)
                if nxt[k] is not None:
                    i, gen, ev = nxt[k]
                    s.wait_event(ev)
                    cur[k] = (i, gen)
                    nxt[k] = start(k) if (prep_ahead and pending) else None
            if cur[k] is None:
                continue
            i, gen = cur[k]
            with torch.cuda.stream(s):
                try:
                    next(gen)
                except StopIteration as e:
                    r = e.value
                    if not keep_w_hat:
                        r.pop("W_hat")
                    if ltq_formats is not None:
                        r["ltq"] = _pack_job(r["pack"], ltq_formats, to_host)
                        if not pack:
                            r["pack"] = None
                    out[i] = r
                    cur[k] = None
                    if on_issued is not None:
                        on_issued(i)
    for s in streams + (preps if prep_ahead else []):
        main.wait_stream(s)
    for i, r in enumerate(out):
        _record(r, main)
    nd = torch.stack([torch.stack([r["num"], r["den"]]) for r in out]).cpu()
    check_gemm_errors(dev)
    info = torch.stack([r["chol_info"].reshape(()) for r in out]).cpu()
    bad = (torch.stack([r["ltq"]["bad"].reshape(()) for r in out]).cpu() if ltq_formats is not None
           else torch.zeros(len(out), dtype=torch.int64))
    res = []
    for i, r in enumerate(out):
        if int(info[i]) != 0:
            raise torch.linalg.LinAlgError(f"quantize_matrices: job {i}: the damped Hessian is not positive-definite")
        if int(bad[i]) != 0:
            raise RuntimeError(f"quantize_matrices: job {i}: the packed tiles disagree with the quantizer in "
                               f"{int(bad[i])} weights")
        d = {"qdata": r["qdata"], "rel_loss": float(nd[i, 0]) / float(nd[i, 1])}
        if pack:
            d["pack"] = r["pack"]
        if keep_w_hat:
            d["W_hat"] = r["W_hat"]
        if ltq_formats is not None:
            d["ltq"] = {k: v for k, v in r["ltq"].items() if k != "bad"}
        res.append(d)
    return res


def _pack_job(pm: dict, formats: Dict, to_host: bool) -> dict:
    """.ltq data of one matrix on the current stream: packed + verified slices, scales; optionally copied to pinned
    host memory (asynchronously, on the same stream)."""
    from .ltq_file import pack_matrix_device
    data, rows, bad = pack_matrix_device(pm, formats, verify=True)
    out = {"data": data, "slices": [[r0, r1, fi, o] for r0, r1, fi, o in rows], "d_row": pm["d_row"].to(torch.float16),
           "e": pm["e"].to(torch.int8), "suh": pm["suh"].to(torch.float16), "bad": bad}
    if to_host:
        for k in ("data", "d_row", "e", "suh"):
            h = torch.empty(out[k].shape, dtype=out[k].dtype, pin_memory=True)
            h.copy_(out[k], non_blocking=True)
            out[k] = h
    return out
