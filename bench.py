"""Benchmark of the LTQ TCQ quantizer hot path on B200 (one JSON line on rank 0).

Workload ("Llama-3.2-3B-shaped layer set"): a step is one decoder layer of seven matrices,
q 3072x3072, k / v 1024x3072, o 3072x3072, gate / up 8192x3072, down 3072x8192 (100.7 M weights), quantized as the
reference's quantize_matrix_liqk_v2 does (src/liqk_v2.py:1029-1198): FWHT-256 rotation with the column scale suh,
damped (0.02 x TCQ_DAMP_MULT 10 = 0.2) Cholesky factor U of the rotated Hessian, per-(row, block) scale fit, LDLQ over
256-column blocks with the two-pass tail-biting TCQ Viterbi (tb_window 32) per 16-column sub-block, c_row / suh refits,
then packed into .ltq tiles and verified on the device (src/ltq_file.py:79-148, 187-213).  Even layers use TCQ3X
(K = 3, 8 subsets, 4 gains per 16 weights), odd layers TCQ25X (K = 3 - 0.5, D2).  Synthetic seeded inputs with the
config's distributions: bf16 Student-t(5) x 0.02 weights with 0.5 % of input columns x 20; H = X^T X / 4096 of 4096
N(0, 1) activation rows with log-normal(0, 1) per-channel scales, one H per matrix.  Every rank quantizes its own layers
(weak scaling, no collective on the data path).  Metric: Mweights/s quantized (whole job).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl mine|reference]
    torchrun --nproc-per-node N bench.py --gpus N ...

--impl reference times the reference algorithm on the host cores: the CPU restatement of the reference Viterbi
(oracle/, the only CPU implementation that can run on the GPU box) on tiles of this workload's format and tail-biting
schedule, all host threads, bounded samples.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time
from pathlib import Path

import numpy as np
import torch

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "Mweights/s quantized"
WORKLOAD = "llama3.2-3b_layers_tcq3x_tcq25x_fwht_ldlq_damp0.2_tbwin32_pack"
LAYER = [("q_proj", 3072, 3072), ("k_proj", 1024, 3072), ("v_proj", 1024, 3072), ("o_proj", 3072, 3072),
         ("gate_proj", 8192, 3072), ("up_proj", 8192, 3072), ("down_proj", 3072, 8192)]
FORMATS = ("TCQ3X", "TCQ25X")
WEIGHTS_PER_LAYER = sum(m * k for _, m, k in LAYER)
TB_WINDOW = 32
ALU_SLOTS_PER_ACS = 2  # one path-metric add + half a compare + half a select (issue-slot accounting)


def layer_spec(layer: int) -> str:
    return FORMATS[layer % 2]


def make_matrix(M: int, K: int, seed: int, device) -> tuple:
    """bf16 Student-t(5) * 0.02 weights [M, K] with 0.5 % of the input columns x 20; H = X^T X / 4096 with
    X = N(0, 1) [4096, K] * exp(N(0, 1)) per column."""
    g = torch.Generator(device=device).manual_seed(seed)
    z = torch.randn(M, K, device=device, generator=g)
    chi2 = torch.zeros(M, K, device=device)
    for _ in range(5):
        chi2.add_(torch.randn(M, K, device=device, generator=g).square_())
    W = z.div_(chi2.div_(5.0).sqrt_()).mul_(0.02)
    del chi2
    cols = torch.randperm(K, device=device, generator=g)[: max(1, round(0.005 * K))]
    W[:, cols] *= 20.0
    W = W.to(torch.bfloat16)
    X = torch.randn(4096, K, device=device, generator=g) * torch.exp(torch.randn(1, K, device=device, generator=g))
    H = (X.T @ X) / 4096.0
    return W, H


def layer_jobs(layer: int, rank: int, device) -> list:
    spec = layer_spec(layer)
    return [(*make_matrix(M, K, 1_000_003 * rank + 1009 * layer + j, device), spec)
            for j, (_, M, K) in enumerate(LAYER)]


class ClockSampler:
    """nvidia-smi samples (SM clock, max clock, throttle reasons) while the timed region runs."""
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
              "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
              "clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.f = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
        self.p = None

    def __enter__(self):
        try:
            self.p = subprocess.Popen(["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.FIELDS}",
                                       "--format=csv,noheader,nounits", "-lms", "200"], stdout=self.f,
                                      stderr=subprocess.DEVNULL)
        except OSError:
            self.p = None
        return self

    def __exit__(self, *a):
        if self.p is not None:
            self.p.terminate()
            try:
                self.p.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.p.kill()

    def summary(self) -> dict:
        self.f.flush()
        rows = [r.split(",") for r in Path(self.f.name).read_text().splitlines() if r.strip()]
        os.unlink(self.f.name)
        sm, mx, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for r in rows:
            try:
                sm.append(float(r[1]))
                mx.append(float(r[2]))
            except (ValueError, IndexError):
                continue
            for nm, v in zip(names, r[5:9]):
                if v.strip().lower() == "active":
                    reasons.add(nm)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
        load = [v for v in sm if v > 0.5 * max(sm)] or sm
        return {"sm_mhz": statistics.median(load), "sm_max_mhz": max(mx), "reasons": sorted(reasons),
                "samples": len(sm)}


def measured_peaks() -> dict:
    p = ROOT / "MEASURED_PEAKS.json"
    return json.loads(p.read_text()) if p.exists() else {}


def alu_peak_gacs() -> tuple:
    sm_mhz = float(measured_peaks().get("sm_max_mhz", 1965.0))
    return 148 * 128 * sm_mhz * 1e6 / ALU_SLOTS_PER_ACS / 1e9, sm_mhz


# ------------------------------------------------------------------------------------------------
# CPU: the reference's own CPU Viterbi (src/tcq_proto.py:363-419, torch) from its install in baseline/_ref; where that
# install is absent, the oracle's C restatement of the reference Viterbi (oracle/tcq_oracle.c)
# ------------------------------------------------------------------------------------------------
CPU_TILES = 256           # tiles of 256 weights per CPU call, in both CPU legs
CPU_PASSES = 1.0 + 2.0 * TB_WINDOW / 256.0  # trellis passes per weight of the GPU step's schedule (windowed first pass)


def _cpu_threads() -> int:
    return len(os.sched_getaffinity(0))


def _cpu_tiles(n: int, seed: int = 0) -> tuple:
    rng = np.random.default_rng(seed)
    x = rng.standard_normal((n, 256)).astype(np.float32)
    w = (0.5 + rng.random(256)).astype(np.float32)
    return x, w


class _CpuViterbi:
    """One CPU leg: `run(x, w)` quantizes tiles x [n, 256] with position weights w [256]; `per_weight_passes` is how
    many trellis passes one call spends per weight; `desc` / `kind` / `threads` describe it.

    The reference's CPU implementation is its torch viterbi_ub (4 label subsets, no tail-biting): it runs the
    config-1 format of BASELINE (K = 2, 4 subsets, 2-bit gain index per 16 weights: 1024 states x 4 gain slots, the
    same add-compare-selects per weight and pass as the GPU step's TCQ3X / TCQ25X), one free pass per call; the GPU
    step's schedule needs CPU_PASSES passes per weight, so its rate is the pass rate / CPU_PASSES.  Without the
    reference install, the oracle's C restatement runs the GPU step's own TCQ3X two-pass tail-biting schedule."""

    def __init__(self):
        self.threads = _cpu_threads()
        from oracle.refroot import import_reference, reference_root
        root = reference_root()
        if root is not None:
            import_reference(root)
            os.environ["TCQ_NO_COMPILE"] = "1"  # its torch.compile step cannot build on these hosts (no Python headers)
            torch.set_num_threads(self.threads)
            import src.tcq_proto as tp
            u = json.loads((root / "results" / "universal_gaussian.json").read_text())["tcq_K2_h2"]
            self.tab = torch.tensor(u["tab"], dtype=torch.float32)
            self.gains = tp.make_gains(2, u["step"], "cpu")
            self.fn = tp.viterbi_ub
            self.kind, self.per_weight_passes = "reference", 1.0
            self.desc = ("the reference's torch viterbi_ub (src/tcq_proto.py:363-419, TCQ_NO_COMPILE=1, torch threads "
                         f"= {self.threads}) on config-1 tiles (K 2, h 2, sub 16, mask 359), one free pass per call, "
                         f"rate divided by {CPU_PASSES} passes per weight of the GPU step's schedule")
        else:
            from ltq_research_b200.formats import TCQ_CONFIG
            from ltq_research_b200.tcq_proto import make_gains
            self.c = TCQ_CONFIG["TCQ3X"]
            self.gains = make_gains(self.c["h"], self.c["step"], "cpu").numpy().astype(np.float32)
            self.fn = None
            self.kind, self.per_weight_passes = "port", CPU_PASSES
            self.desc = ("the C restatement of the reference Viterbi (oracle/tcq_oracle.c, OpenMP, "
                         f"{self.threads} threads) on TCQ3X tiles, two-pass tail-biting with window {TB_WINDOW}")

    def run(self, x, w):
        if self.fn is not None:
            xt = torch.from_numpy(x)
            self.fn(xt, self.tab, 2, 10, 359, self.gains, sub=16, wts=torch.from_numpy(w))
        else:
            from oracle import oracle as O
            c = self.c
            O.viterbi(x, np.asarray(c["lut"], np.float32), c["K"], 10, c["m"], self.gains, sub=16, wts=w,
                      m_extra=tuple(c["m_extra"]), tail_biting=True, tb_window=TB_WINDOW, return_code=True,
                      n_threads=self.threads)

    def rate(self, weights: int, seconds: float) -> float:
        """Mweights/s of the GPU step's schedule for `weights` weights quantized by calls that took `seconds`."""
        return weights / seconds / 1e6 * self.per_weight_passes / CPU_PASSES


def cpu_baseline_sample(seconds: float = 15.0) -> dict:
    """The CPU leg on rank 0 at N = 1: CPU_TILES tiles per call, calls until `seconds` have passed."""
    cv = _CpuViterbi()
    x, w = _cpu_tiles(CPU_TILES * 4)
    cv.run(x[:CPU_TILES], w)  # untimed first call
    done, calls, t0 = 0, 0, time.perf_counter()
    while time.perf_counter() - t0 < seconds:
        j = calls % 4
        cv.run(x[j * CPU_TILES:(j + 1) * CPU_TILES], w)
        done += CPU_TILES * 256
        calls += 1
    el = time.perf_counter() - t0
    return {"value": cv.rate(done, el), "unit": METRIC, "cores": cv.threads, "kind": cv.kind,
            "sample": f"{calls} calls of {CPU_TILES} tiles of 256 in {el:.1f} s: {cv.desc}; the Viterbi search only "
                      f"(the LDLQ / refit linear algebra of the GPU step is not timed on the CPU)"}


def run_reference(args, rank: int, world: int):
    """--impl reference: the reference's CPU implementation of the path on the host cores, rank 0 only; each step one
    call of CPU_TILES tiles (a bounded sample of one layer's sub-block tiles)."""
    if rank != 0:
        return
    cv = _CpuViterbi()
    n = CPU_TILES
    x, w = _cpu_tiles(n * (args.steps + args.warmup), seed=1)
    for k in range(args.warmup):
        cv.run(x[k * n:(k + 1) * n], w)
    t0 = time.perf_counter()
    for k in range(args.steps):
        s = (args.warmup + k) * n
        cv.run(x[s:s + n], w)
    el = time.perf_counter() - t0
    v = cv.rate(args.steps * n * 256, el)
    sample = f"{n} tiles of 256 per step: {cv.desc}; the Viterbi search only"
    line = {"metric": METRIC, "value": v, "unit": METRIC, "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": el / args.steps * 1e3, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "f32", "data": "synthetic", "impl": "reference",
            "config": {"workload": WORKLOAD, "tiles_per_step": n, "parallelism": "host threads",
                       "reference_scope": "Viterbi search of the path (the reference's CPU code for it); the GPU arm's "
                                          "step also includes rotation, factorisation, LDLQ feedback, refits, packing"},
            "cpu_baseline": {"value": v, "unit": METRIC, "cores": cv.threads, "kind": cv.kind, "sample": sample},
            "e2e": {"value": v, "unit": METRIC, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


# ------------------------------------------------------------------------------------------------
# GPU
# ------------------------------------------------------------------------------------------------

def union_ms(iv: list) -> float:
    tot, end = 0.0, -1e30
    for a, b in sorted(iv):
        if b <= end:
            continue
        tot += b - max(a, end)
        end = b
    return tot


def isolated_block_roofline(dev, spec: str, rows: int = 27648, timed: bool = True) -> dict:
    """One fused block launch over `rows` rows (a layer's worth of tile groups) timed alone: the block kernel at full
    occupancy, without the concurrent factorisation / GEMM kernels of the real step."""
    import ltq_research_b200.liqk_v2 as L
    g = torch.Generator(device=dev).manual_seed(7)
    W = torch.randn(rows, 256, device=dev, generator=g)
    A = torch.randn(256, 256, device=dev, generator=g) / 16
    U = torch.triu(A) + 4 * torch.eye(256, device=dev)
    Ui = torch.linalg.solve_triangular(U, torch.eye(256, device=dev), upper=True).contiguous()
    d_rb = torch.ones(rows, 1, device=dev)
    dw = (1.0 / torch.diagonal(U) ** 2).contiguous()
    G = torch.empty(rows, 256, device=dev)
    idx = torch.empty(rows, 256, dtype=torch.int16, device=dev)
    gi = torch.empty(rows, 256, dtype=torch.uint8, device=dev)
    br = L._BlockRunner(spec, rows, dev)
    for _ in range(2):
        br.run(W, 0, d_rb, 0, dw, U, Ui, G, idx, gi)
    if not timed:
        br.run(W, 0, d_rb, 0, dw, U, Ui, G, idx, gi)
        torch.cuda.synchronize()
        return {}
    ms = []
    for _ in range(3):
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        br.run(W, 0, d_rb, 0, dw, U, Ui, G, idx, gi)
        b.record()
        torch.cuda.synchronize()
        ms.append(a.elapsed_time(b))
    acs = br.acs_per_block()
    return {"format": spec, "rows": rows, "ms": statistics.median(ms),
            "achieved": acs / (statistics.median(ms) * 1e-3) / 1e9}


def _event_ms(fn, reps: int = 5) -> float:
    """Median device time of fn() (CUDA events on the current stream, after two untimed calls)."""
    for _ in range(2):
        fn()
    ms = []
    for _ in range(reps):
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        fn()
        b.record()
        torch.cuda.synchronize()
        ms.append(a.elapsed_time(b))
    return statistics.median(ms)


def aux_measurements(dev, fmts) -> dict:
    """The secondary paths on one GPU:
    * decode GEMV: y = W x from the packed tiles of a gate-shaped 8192 x 3072 TCQ3X matrix: the kernel alone
      (ltq_matvec_slice on the rotated input; weights / s and packed bytes / s) and the whole call (input rotation +
      kernel through ltq_file.matvec), each as 20 back-to-back calls;
    * rings: quantize_rings of a 2048 x 2560 bf16 table (20,480 rings, TCQ4X, rotation, three scale tries,
      tail-biting with a full first pass): values / s and the Viterbi's ACS rate (2 passes x 1024 x 4 slots x 3 tries
      per value);
    * DP-profile table kernel: lut_subs_quant over 2^20 sub-blocks with an 8192 x 64 table: sub-blocks / s;
    * the HBM-bound kernels of the path on a 16384 x 4096 matrix (268 MB in fp32, above the 126 MB L2), 10 back-to-back
      calls each, algorithmic bytes / s against MEASURED_PEAKS hbm_gbs: FWHT-256 with the column scale (fp32 in and
      out, 8 B / weight), the row-scale fit (4 B read), the .ltq pack of TCQ3X codes (idx + gi read, 3 B, tile bytes
      written) and the on-device verify decode (tile bytes + the fp32 reference values read)."""
    from ltq_research_b200.batch import quantize_matrices
    from ltq_research_b200.ltq_file import matvec, matvec_slice_device, rotate_input
    from ltq_research_b200.rings import quantize_rings
    from ltq_research_b200.tcq_proto import lut_subs_quant_cuda
    out = {"impl": "aux", "data": "synthetic (seeded)"}
    W, H = make_matrix(8192, 3072, 5, dev)
    r = quantize_matrices([(W, H, "TCQ3X")], ltq_formats=fmts, pack=False)[0]["ltq"]
    data = torch.zeros(((r["data"].numel() + 63) // 64) * 64, dtype=torch.uint8, device=dev)
    data[: r["data"].numel()] = r["data"]
    x = torch.randn(3072, device=dev)
    fl = list(fmts.values())
    xr = rotate_input(x, r["suh"])
    (r0, r1, fi, off), = r["slices"]
    y = torch.empty(8192, device=dev)
    reps = 20  # back-to-back calls between the events, so that host issue time does not count
    ms_k = _event_ms(lambda: [matvec_slice_device(data[off:], r1 - r0, 3072, fl[fi], r["d_row"], r["e"], xr, y=y)
                              for _ in range(reps)]) / reps
    ms = _event_ms(lambda: [matvec(data, r["slices"], fl, r["d_row"], r["e"], r["suh"], x) for _ in range(reps)]) / reps
    out["decode_gemv"] = {"shape": [8192, 3072], "format": "TCQ3X", "kernel_ms": ms_k, "call_ms": ms,
                          "gweights_per_s": 8192 * 3072 / ms_k / 1e6, "packed_gb_per_s": r["data"].numel() / ms_k / 1e6}
    g = torch.Generator().manual_seed(4)
    T = (torch.randn(2048, 2560, generator=g) * 0.03 * torch.exp(0.5 * torch.randn(2048, 1, generator=g))
         ).to(torch.bfloat16).to(dev)
    ms = _event_ms(lambda: quantize_rings(T, "TCQ4X", True), reps=3)
    n = T.numel()
    out["rings"] = {"table": [2048, 2560], "format": "TCQ4X:rot", "ms": ms, "mvalues_per_s": n / ms / 1e3,
                    "gacs_per_s": n * 2 * 1024 * 4 * 3 / ms / 1e6}
    S = 1 << 20
    xs = torch.randn(S, 16, device=dev)
    dh = torch.rand(S, 16, device=dev) + 0.1
    lut = torch.sort(torch.randn(8192, 64, device=dev), dim=0).values
    ms = _event_ms(lambda: lut_subs_quant_cuda(xs, dh, lut, 8191 / 8.0, 4095.5))
    out["lut_subs"] = {"sub_blocks": S, "table": [8192, 64], "ms": ms, "msub_blocks_per_s": S / ms / 1e3}
    out["hbm_kernels"] = hbm_kernels(dev, fmts["TCQ3X"])
    return out


def hbm_kernels(dev, f) -> dict:
    """Bandwidth of the path's HBM-bound kernels (see aux_measurements)."""
    from ltq_research_b200 import _lib
    from ltq_research_b200.liqk_v2 import fwht_rows_scaled
    from ltq_research_b200.ltq_file import decode_slice_device, pack_slice_device
    R, K = 16384, 4096
    n = R * K
    peak = float(measured_peaks().get("hbm_gbs", 0.0)) or None
    g = torch.Generator(device=dev).manual_seed(6)
    W = torch.randn(R, K, device=dev, generator=g)
    s = torch.rand(K, device=dev, generator=g) + 0.5
    Wr = torch.empty_like(W)
    d_row = torch.empty(R, device=dev)
    e = torch.empty((R, K // 256), dtype=torch.int8, device=dev)
    d_rb = torch.empty((R, K // 256), device=dev)
    idx = torch.randint(0, f.n_labels * f.U, (R, K), device=dev, generator=g, dtype=torch.int16)
    gi = torch.randint(0, 1 << f.h, (R, K), device=dev, generator=g, dtype=torch.uint8)
    data = pack_slice_device(idx, gi, f)
    buf = torch.zeros(((data.numel() + 63) // 64) * 64, dtype=torch.uint8, device=dev)
    buf[: data.numel()] = data
    ref = decode_slice_device(buf, R, K, f)
    bad = torch.zeros(1, dtype=torch.int64, device=dev)
    st = torch.cuda.current_stream(dev).cuda_stream
    L = _lib.lib()
    tb = data.numel()
    reps = 10
    kernels = {
        "fwht256": (lambda: fwht_rows_scaled(W, s, mode=1, out=Wr), 8 * n),
        "scale_fit": (lambda: L.ltq_scale_fit(W.data_ptr(), K, R, K, 1.1, 0.25, 5, None, d_row.data_ptr(),
                                              e.data_ptr(), d_rb.data_ptr(), st), 4 * n),
        "pack_slice": (lambda: pack_slice_device(idx, gi, f, out=buf), 3 * n + tb),
        "decode_verify": (lambda: decode_slice_device(buf, R, K, f, ref=ref, mismatches=bad), tb + 4 * n),
    }
    out = {"shape": [R, K], "format": f.name, "peak_gbs": peak}
    for name, (fn, nbytes) in kernels.items():
        ms = _event_ms(lambda: [fn() for _ in range(reps)]) / reps
        gbs = nbytes / ms / 1e6
        out[name] = {"ms": ms, "algorithmic_gb": nbytes / 1e9, "gb_per_s": gbs, "frac": gbs / peak if peak else None}
    torch.cuda.synchronize()
    assert int(bad) == 0, "hbm_kernels: the verify decode disagrees with its own reference"
    return out


def write_kernel_list(args, timed, fmts):
    """The timed layers quantized once more under torch.profiler (CUPTI activity records, device timestamps): per
    kernel name its launches, summed device time and share of the summed time, as a markdown table.  Kernels of
    different streams overlap, so the shares describe where device time goes, not wall-clock time."""
    from collections import defaultdict
    from torch.profiler import ProfilerActivity, profile
    from ltq_research_b200.batch import quantize_matrices
    with profile(activities=[ProfilerActivity.CUDA]) as prof:
        quantize_matrices(timed, n_streams=args.streams, ltq_formats=fmts, pack=False)
        torch.cuda.synchronize()
    agg = defaultdict(lambda: [0, 0.0])
    t0, t1 = float("inf"), 0.0
    for e in prof.events():
        if e.device_type != torch.autograd.DeviceType.CUDA or e.device_time_total <= 0:
            continue
        a = agg[e.name[:110]]
        a[0] += 1
        a[1] += e.device_time_total
        t0, t1 = min(t0, e.time_range.start), max(t1, e.time_range.end)
    tot = sum(v[1] for v in agg.values())
    lines = [f"| kernel | launches | device ms | share |", "|---|---|---|---|"]
    for name, (n, us) in sorted(agg.items(), key=lambda kv: -kv[1][1])[:40]:
        lines.append(f"| `{name}` | {n} | {us / 1e3:.1f} | {100 * us / tot:.1f} % |")
    head = (f"{args.steps} layers ({len(timed)} matrices), {args.streams} streams: {sum(v[0] for v in agg.values())} "
            f"launches, summed device time {tot / 1e3:.1f} ms over a {(t1 - t0) / 1e3:.1f} ms span\n\n")
    with open(args.kernel_list, "w") as f:
        f.write(head + "\n".join(lines) + "\n")
    print(head.strip(), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=8)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="mine", choices=["mine", "reference"])
    ap.add_argument("--streams", type=int, default=8)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--profile", action="store_true",
                    help="quantize one matrix of --rows x 3072 (TCQ3X) untimed, for ncu captures of its kernels")
    ap.add_argument("--rows", type=int, default=1024)
    ap.add_argument("--profile-block", default=None, metavar="FORMAT",
                    help="one fused block launch of FORMAT over --rows rows untimed (after two warm-up launches), for "
                         "ncu captures of ldlq_block_kernel")
    ap.add_argument("--profile-viterbi", default=None, metavar="FORMAT",
                    help="three stand-alone two-pass Viterbi calls (ltq_viterbi_tb) of FORMAT over the --rows / 16 "
                         "tiles of one sub-block, for ncu captures of vit_fwd_kernel")
    ap.add_argument("--aux", action="store_true",
                    help="time the secondary paths instead of the layer step (one JSON line): the decode GEMV from "
                         "packed tiles, ring quantization (config 5's path) and the DP-profile table kernel")
    ap.add_argument("--kernel-list", default=None, metavar="PATH",
                    help="after the warm-up, quantize the timed layers once under the CUDA profiler (CUPTI) and write "
                         "the per-kernel launch list (launches, total device time, share) to PATH as markdown")
    args = ap.parse_args()
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if args.warmup < 3:
        ap.error("--warmup must be at least 3 (untimed warm-up steps before the timed region)")
    if args.impl == "reference":
        run_reference(args, rank, world)
        return
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist = None
    if world > 1:
        import torch.distributed as dist
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=dev)

    from ltq_research_b200 import _lib
    import ltq_research_b200.liqk_v2 as Lq
    from ltq_research_b200.batch import quantize_matrices
    from ltq_research_b200.formats import load_formats
    fmts = load_formats(list(FORMATS), dev)

    if args.aux:
        print(json.dumps(aux_measurements(dev, fmts)), flush=True)
        return
    if args.profile_viterbi:
        r = Lq._TcqRunner(args.profile_viterbi, args.rows, dev)
        g = torch.Generator(device=dev).manual_seed(1)
        r.x.copy_(torch.randn(r.x.shape, device=dev, generator=g))
        dw = torch.rand(256, device=dev, generator=g) + 0.5
        for _ in range(3):
            r.run(dw)
        torch.cuda.synchronize()
        print(f"profile run: stand-alone Viterbi {args.profile_viterbi} over {r.nt} tiles", flush=True)
        return
    if args.profile_block:
        r = isolated_block_roofline(dev, args.profile_block, rows=args.rows, timed=False)
        print(f"profile run: fused block {args.profile_block} over {args.rows} rows", flush=True)
        return
    if args.profile:
        W, H = make_matrix(args.rows, 3072, 5, dev)
        r = quantize_matrices([(W, H, "TCQ3X")], ltq_formats=fmts)
        torch.cuda.synchronize()
        print(f"profile run: {args.rows} x 3072 TCQ3X, rel_loss {r[0]['rel_loss']:.5f}", flush=True)
        return

    def barrier():
        if dist is not None:
            dist.barrier()
        torch.cuda.synchronize()

    # inputs of the warm-up and timed layers, resident in HBM (each layer's H and W, ~0.7 GB, far above the 126 MB L2);
    # the warm-up quantizes --warmup layers untimed
    warm = [j for l in range(args.warmup) for j in layer_jobs(10_000 + l, rank, dev)]
    timed = [j for l in range(args.steps) for j in layer_jobs(l, rank, dev)]
    quantize_matrices(warm, n_streams=args.streams, ltq_formats=fmts, pack=False)
    barrier()

    if args.kernel_list:
        write_kernel_list(args, timed, fmts)
        return

    Lq.BLOCK_EVENTS = []
    k0 = _lib.kernels_launched()
    e_start, e_end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clk:
        barrier()
        t_wall = time.perf_counter()
        e_start.record()
        res = quantize_matrices(timed, n_streams=args.streams, ltq_formats=fmts, pack=False)
        e_end.record()
        barrier()
        t_wall = time.perf_counter() - t_wall
    launches = _lib.kernels_launched() - k0
    ev, Lq.BLOCK_EVENTS = Lq.BLOCK_EVENTS, None
    dev_ms = e_start.elapsed_time(e_end)
    iv = [(e_start.elapsed_time(a), e_start.elapsed_time(b)) for a, b, _, _ in ev]
    block_ms = union_ms(iv)
    block_acs = sum(c for _, _, c, _ in ev)
    block_weights = sum(w for _, _, _, w in ev)
    rel = [r["rel_loss"] for r in res]
    packed_bytes = sum(int(r["ltq"]["data"].numel()) for r in res)

    # end to end through the public API: pinned host inputs in, the packed .ltq tensors back in pinned host memory
    e2e_ms, h2d, d2h, e2e_same = None, 0, 0, None
    if not args.no_e2e:
        host = [(W.cpu().pin_memory(), H.cpu().pin_memory(), sp) for W, H, sp in timed]
        h2d = sum(W.numel() * W.element_size() + H.numel() * H.element_size() for W, H, _ in host)
        # one untimed pass through the same path first (pinned host output buffers, host-to-device staging; with
        # several GPUs also the gather, whose first call sets up NCCL's point-to-point connections)
        warm_h = quantize_matrices(host, n_streams=args.streams, ltq_formats=fmts, pack=False, to_host=dist is None)
        if dist is not None:
            from ltq_research_b200.shard import gather_ltq
            gather_ltq({rank * len(warm_h) + i: r["ltq"] for i, r in enumerate(warm_h)}, dst=0)
        del warm_h
        barrier()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        if dist is None:  # one GPU: the packed tensors come back to pinned host memory on the matrices' streams
            res_h = quantize_matrices(host, n_streams=args.streams, ltq_formats=fmts, pack=False, to_host=True)
            d2h = sum(sum(r["ltq"][k].numel() * r["ltq"][k].element_size() for k in ("data", "d_row", "e", "suh"))
                      for r in res_h)
        else:  # several GPUs: every rank's packed tensors go to rank 0 in one NCCL gather, then to its host memory
            from ltq_research_b200.shard import gather_ltq
            res_h = quantize_matrices(host, n_streams=args.streams, ltq_formats=fmts, pack=False)
            got = gather_ltq({rank * len(res_h) + i: r["ltq"] for i, r in enumerate(res_h)}, dst=0)
            if rank == 0:
                res_h = [{"ltq": got[i]} for i in range(len(res_h))]
                d2h = sum(sum(t.numel() * t.element_size() for k, t in d.items() if k in ("data", "d_row", "e", "suh"))
                          for d in got.values())
        b.record()
        barrier()
        e2e_ms = a.elapsed_time(b)
        # the host run's packed bytes against the device run's (the pipeline is deterministic: expected all equal)
        e2e_same = sum(int(torch.equal(r0["ltq"]["data"].cpu(), r1["ltq"]["data"].cpu()))
                       for r0, r1 in zip(res, res_h))
        del host, res_h

    t = torch.tensor([dev_ms, e2e_ms or 0.0], device=dev)
    if dist is not None:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    dev_ms, e2e_max = t.tolist()
    total = WEIGHTS_PER_LAYER * args.steps * world
    ms_step = dev_ms / args.steps
    value = total / (dev_ms * 1e-3) / 1e6
    clocks = clk.summary()
    iso = isolated_block_roofline(dev, "TCQ3X") if rank == 0 else None
    if rank == 0:
        peak, sm_mhz = alu_peak_gacs()
        achieved = block_acs / (block_ms * 1e-3) / 1e9
        prof = ROOT / "profiles" / "ldlq_block_config2.json"
        traffic = None
        if prof.exists():
            bpw = json.loads(prof.read_text()).get("dram_bytes_per_weight")
            if bpw:  # per average launch: weights x DRAM bytes per weight (ncu capture; mean of the two formats)
                traffic = float(np.mean(list(bpw.values()))) * block_weights / len(ev)
        # the CPU baseline is taken at N = 1 only (on rank 0), where the host cores are not shared with other ranks
        cpu = None if (args.no_cpu_baseline or world > 1) else cpu_baseline_sample()
        line = {
            "metric": METRIC, "value": value, "unit": METRIC, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms_step, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded, config-2 distributions)",
            "config": {"workload": WORKLOAD, "step": "one Llama-3.2-3B decoder layer, 7 matrices, 100.7 M weights",
                       "formats": "TCQ3X even layers / TCQ25X odd layers", "damp": 0.2, "tb_window": TB_WINDOW,
                       "streams": args.streams, "parallelism": f"dp{world} (own layers per rank)",
                       "l2": "inputs larger than L2 (0.7 GB per layer)", "wall_s": t_wall,
                       "rel_loss_mean": float(np.mean(rel)), "ltq_bytes": packed_bytes},
            "roofline": {"bound": "alu", "kernel": "ldlq_block_kernel (fused LDLQ block: Viterbi ACS)",
                         "achieved": achieved, "peak": peak, "unit": "GACS/s", "frac": achieved / peak,
                         "traffic": traffic,
                         "basis": f"sum of the launches' add-compare-selects / union of their CUDA-event intervals "
                                  f"({block_ms:.1f} ms of {dev_ms:.1f} ms) on the launching streams",
                         "peak_basis": f"148 SMs x 128 issue slots/clk x {sm_mhz:.0f} MHz (MEASURED_PEAKS sm_max_mhz) "
                                       f"/ {ALU_SLOTS_PER_ACS} slots per ACS",
                         "isolated": dict(iso, frac=iso["achieved"] / peak)},
            "cpu_baseline": cpu,
            "e2e": None if e2e_ms is None else {
                "value": total / (e2e_max * 1e-3) / 1e6, "unit": METRIC,
                "h2d_bytes_per_step": int(h2d // args.steps), "d2h_bytes_per_step": int(d2h // args.steps),
                "ltq_identical_to_timed_run": f"{e2e_same}/{len(res)} matrices"},
            "gpu_launches": int(launches),
            "clocks": clocks,
        }
        print(json.dumps(line), flush=True)
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
