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

    def __init__(self, port: bool = False):
        self.threads = _cpu_threads()
        from oracle.refroot import import_reference, reference_root
        root = None if port else reference_root()
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


def cpu_baseline_sample(seconds: float = 15.0, port: bool = False, port_seconds: float = 8.0) -> dict:
    """The CPU leg on rank 0 at N = 1: CPU_TILES tiles per call, calls until `seconds` have passed.  When it ran the
    reference's torch viterbi_ub, the oracle's C port is timed as well (`port_seconds`) and reported under "port", a
    second, labelled number."""
    cv = _CpuViterbi(port)
    x, w = _cpu_tiles(CPU_TILES * 4)
    cv.run(x[:CPU_TILES], w)  # untimed first call
    done, calls, t0 = 0, 0, time.perf_counter()
    while time.perf_counter() - t0 < seconds:
        j = calls % 4
        cv.run(x[j * CPU_TILES:(j + 1) * CPU_TILES], w)
        done += CPU_TILES * 256
        calls += 1
    el = time.perf_counter() - t0
    out = {"value": cv.rate(done, el), "unit": METRIC, "cores": cv.threads, "kind": cv.kind,
           "sample": f"{calls} calls of {CPU_TILES} tiles of 256 in {el:.1f} s: {cv.desc}; the Viterbi search only "
                     f"(the LDLQ / refit linear algebra of the GPU step is not timed on the CPU)"}
    if cv.kind == "reference" and port_seconds > 0:
        pt = cpu_baseline_sample(port_seconds, port=True, port_seconds=0)
        out["port"] = {k: pt[k] for k in ("value", "unit", "cores", "kind", "sample")}
    return out


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


def gemm_ldlq_compare(dev) -> dict:
    """tcgen05 six-product GEMM vs cuBLAS on the six-slot form, microseconds per call (see aux_measurements)."""
    from ltq_research_b200 import _lib
    L = _lib.lib()
    st = torch.cuda.current_stream(dev).cuda_stream
    peaks = measured_peaks()

    def med_us(fn):
        return _event_ms(lambda: [fn() for _ in range(5)], reps=10) / 5 * 1e3

    g = torch.Generator(device=dev).manual_seed(9)
    res = {}
    for M, N in ((1024, 256), (3072, 2816), (8192, 2816), (8192, 7936)):
        A3 = torch.randn(M, 768, device=dev, generator=g).to(torch.bfloat16)
        B3 = torch.randn(N, 768, device=dev, generator=g).to(torch.bfloat16)
        A6 = torch.cat([A3[:, 256 * i:256 * i + 256] for i in (0, 0, 1, 0, 1, 2)], 1).contiguous()
        B6 = torch.cat([B3[:, 256 * i:256 * i + 256] for i in (0, 1, 0, 2, 1, 0)], 1).contiguous()
        C = torch.randn(M, N, device=dev, generator=g)
        tc = med_us(lambda: L.ltq_gemm_bf16x6_tn(A3.data_ptr(), 768, B3.data_ptr(), 768, C.data_ptr(), N, M, N, 256,
                                                  -1.0, 1.0, None, st))
        cb = med_us(lambda: torch.addmm(C, A6, B6.T, beta=1, alpha=-1, out_dtype=torch.float32, out=C))
        tf = 2 * M * N * 1536 / (tc * 1e-6) / 1e12
        res[f"{M}x{N}"] = {"tcgen05_us": round(tc, 1), "cublas_us": round(cb, 1), "tcgen05_tflops": round(tf, 1),
                           "frac_of_bf16_burst": round(tf / peaks["bf16_tflops"], 3) if peaks.get("bf16_tflops") else None}
    return res


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
      written) and the on-device verify decode (tile bytes + the fp32 reference values read);
    * the LDLQ inter-block update's GEMM (W[:, c1:] -= acat @ bcat, K = 256 split in three bf16 parts, six products) at
      four (rows, columns) shapes: the tcgen05 kernel (ltq_gemm_bf16x6_tn on compact part operands) against cuBLAS
      (torch.addmm with fp32 output) on the K-concatenated six-slot operands of the same product, medians of 10 x 5
      back-to-back calls."""
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
    out["gemm_ldlq"] = gemm_ldlq_compare(dev)
    S = 1 << 20
    xs = torch.randn(S, 16, device=dev)
    dh = torch.rand(S, 16, device=dev) + 0.1
    lut = torch.sort(torch.randn(8192, 64, device=dev), dim=0).values
    ms = _event_ms(lambda: lut_subs_quant_cuda(xs, dh, lut, 8191 / 8.0, 4095.5))
    out["lut_subs"] = {"sub_blocks": S, "table": [8192, 64], "ms": ms, "msub_blocks_per_s": S / ms / 1e3}
    out["hbm_kernels"] = hbm_kernels(dev, fmts["TCQ3X"])
    return out


def hbm_kernels(dev, f, reps: int = 10, timed: bool = True) -> dict:
    """Bandwidth of the path's HBM-bound kernels (see aux_measurements).  timed=False: each kernel `reps` times,
    untimed (the profiling run of --profile-hbm)."""
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
    kernels = {
        "fwht256": (lambda: fwht_rows_scaled(W, s, mode=1, out=Wr), 8 * n),
        "scale_fit": (lambda: L.ltq_scale_fit(W.data_ptr(), K, R, K, 1.1, 0.25, 5, None, d_row.data_ptr(),
                                              e.data_ptr(), d_rb.data_ptr(), st), 4 * n),
        "pack_slice": (lambda: pack_slice_device(idx, gi, f, out=buf), 3 * n + tb),
        "decode_verify": (lambda: decode_slice_device(buf, R, K, f, ref=ref, mismatches=bad), tb + 4 * n),
    }
    out = {"shape": [R, K], "format": f.name, "peak_gbs": peak}
    if not timed:
        for name, (fn, nbytes) in kernels.items():
            for _ in range(reps):
                fn()
        torch.cuda.synchronize()
        return out
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


# ------------------------------------------------------------------------------------------------
# The other BASELINE configs (--workload): config 1 (the Gaussian Viterbi rig), config 3 (a Qwen3-8B-shaped model
# sharded by whole matrices, strong scaling), config 4 (a Qwen3-30B-A3B-shaped MoE, every matrix's rows split across
# the ranks), config 5 (a Gemma-style 262,144 x 2,560 embedding table as tail-biting rings, rows split across ranks).
# ------------------------------------------------------------------------------------------------
def synth_weight(M: int, K: int, seed: int, device) -> torch.Tensor:
    """bf16 Student-t(5) * 0.02 [M, K] with 0.5 % of the input columns x 20 (the config-2 weight distribution)."""
    g = torch.Generator(device=device).manual_seed(seed)
    W = torch.randn(M, K, device=device, generator=g)
    chi2 = torch.zeros(M, K, device=device)
    for _ in range(5):
        chi2.add_(torch.randn(M, K, device=device, generator=g).square_())
    W.div_(chi2.div_(5.0).sqrt_()).mul_(0.02)
    del chi2
    W[:, torch.randperm(K, device=device, generator=g)[: max(1, round(0.005 * K))]] *= 20.0
    return W.to(torch.bfloat16)


def synth_hessian(K: int, rows: int, seed: int, device) -> torch.Tensor:
    """H = X^T X / rows, X = N(0, 1) [rows, K] with log-normal(0, 1) per-channel scales (the config-2 Hessians)."""
    g = torch.Generator(device=device).manual_seed(seed)
    X = torch.randn(rows, K, device=device, generator=g) * torch.exp(torch.randn(1, K, device=device, generator=g))
    return (X.T @ X) / float(rows)


def qwen3_8b_matrices() -> list:
    """The 252 matrices of config 3 as (name, M, K, format, Hessian key): 36 layers of q / k / v (sharing the
    attention input's Hessian), o, gate / up (sharing the MLP input's) and down; formats cycle the 19-format TCQPQ menu
    (K = 2..5, 8- and 16-subset labels, D2 and D4 parity, 32-weight gain groups)."""
    from ltq_research_b200.formats import MENU_TCQPQ
    shapes = [("q_proj", 4096, 4096, "attn"), ("k_proj", 1024, 4096, "attn"), ("v_proj", 1024, 4096, "attn"),
              ("o_proj", 4096, 4096, "o"), ("gate_proj", 12288, 4096, "mlp"), ("up_proj", 12288, 4096, "mlp"),
              ("down_proj", 4096, 12288, "down")]
    return [(f"layers.{l}.{nm}", M, K, MENU_TCQPQ[(7 * l + j) % len(MENU_TCQPQ)], (l, hk))
            for l in range(36) for j, (nm, M, K, hk) in enumerate(shapes)]


def moe_layer_matrices(layer: int) -> list:
    """Config 4, one Qwen3-30B-A3B-shaped layer as (name, M, K, format, Hessian key): attention q 4096 x 2048,
    k / v 512 x 2048 (sharing the attention input's Hessian), o 2048 x 4096 at TCQ45X (4.5 bpw); 128 experts, each
    gate_up 1536 x 2048 (gate and up fused, as the reference's MoE path stores them) and down 2048 x 768 with Hessians
    of their own, at TCQ275X (2.75 bpw)."""
    out = [(f"layers.{layer}.q_proj", 4096, 2048, "TCQ45X", (layer, "attn")),
           (f"layers.{layer}.k_proj", 512, 2048, "TCQ45X", (layer, "attn")),
           (f"layers.{layer}.v_proj", 512, 2048, "TCQ45X", (layer, "attn")),
           (f"layers.{layer}.o_proj", 2048, 4096, "TCQ45X", (layer, "o"))]
    for e in range(128):
        out.append((f"layers.{layer}.experts.{e}.gate_up_proj", 1536, 2048, "TCQ275X", (layer, f"gu{e}")))
        out.append((f"layers.{layer}.experts.{e}.down_proj", 2048, 768, "TCQ275X", (layer, f"dn{e}")))
    return out


def _seed_of(key) -> int:
    """A stable seed from a matrix or Hessian key (independent of the rank that generates it)."""
    import zlib
    return zlib.crc32(repr(key).encode()) & 0x7FFFFFFF


def _block_roofline(ev: list, t0) -> dict:
    """The fused block kernel's live ACS rate over the launches in `ev` (BLOCK_EVENTS), timed from event t0."""
    peak, sm_mhz = alu_peak_gacs()
    if not ev:
        return None
    iv = [(t0.elapsed_time(a), t0.elapsed_time(b)) for a, b, _, _ in ev]
    ms = union_ms(iv)
    acs = sum(c for _, _, c, _ in ev)
    ach = acs / (ms * 1e-3) / 1e9
    return {"bound": "alu", "kernel": "ldlq_block_kernel (fused LDLQ block: Viterbi ACS)", "achieved": ach,
            "peak": peak, "unit": "GACS/s", "frac": ach / peak, "traffic": None,
            "basis": f"sum of the launches' add-compare-selects / union of their CUDA-event intervals ({ms:.1f} ms)",
            "peak_basis": f"148 SMs x 128 issue slots/clk x {sm_mhz:.0f} MHz / {ALU_SLOTS_PER_ACS} slots per ACS"}


def _timed(fn, barrier, local):
    """Run fn() between barriers, timed by CUDA events on the current stream; returns (result, ms, clocks)."""
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clk:
        barrier()
        a.record()
        r = fn()
        b.record()
        barrier()
    return r, a.elapsed_time(b), clk.summary(), a


def _max_over_ranks(dist, dev, *vals) -> list:
    t = torch.tensor([float(v) for v in vals], device=dev)
    if dist is not None:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return t.tolist()


def run_matrix_model(args, rank, world, dev, dist, barrier, local):
    """Config 3 (qwen3-8b) or 4 (qwen3-30b-a3b).  Inputs (W bf16, H fp32) are generated on the device from seeds of
    their matrix / Hessian keys, so every rank makes exactly its own share.
    qwen3-8b: the 252 matrices go to ranks whole (shard.assign, longest first), a step is the whole model, strong
    scaling (same model at every N), no collective until one NCCL gather of the packed .ltq tensors to rank 0.
    qwen3-30b-a3b: a step is one MoE layer (260 matrices); every matrix's rows are split across the ranks
    (shard.row_ranges, 16-row units) with the whole H on every rank and five all-reduces of row sums per matrix
    (shard.nccl_row_reduce), so every rank reaches the same suh; --steps layers are timed after --warmup layers."""
    from ltq_research_b200 import _lib
    import ltq_research_b200.liqk_v2 as Lq
    from ltq_research_b200.batch import quantize_matrices
    from ltq_research_b200.formats import MENU_TCQPQ, load_formats
    from ltq_research_b200.shard import assign, gather_ltq, nccl_row_reduce, row_ranges
    moe = args.workload == "qwen3-30b-a3b"
    by_rows = moe and args.moe_shard == "rows"
    if moe:
        warm_m = [m for l in range(args.warmup) for m in moe_layer_matrices(1000 + l)]
        timed_m = [m for l in range(args.steps) for m in moe_layer_matrices(l)]
        if by_rows:
            mine_w, mine_t = list(range(len(warm_m))), list(range(len(timed_m)))
            rows = {M: row_ranges(M, world)[rank] for M in {m[1] for m in warm_m + timed_m}}
            row_reduce = nccl_row_reduce() if world > 1 else None
        else:
            mine_w = assign([(M, K, sp) for _, M, K, sp, _ in warm_m], world)[rank]
            mine_t = assign([(M, K, sp) for _, M, K, sp, _ in timed_m], world)[rank]
            rows, row_reduce = None, None
        fmts = load_formats(["TCQ45X", "TCQ275X"], dev)
    else:
        allm = qwen3_8b_matrices()
        shard = assign([(M, K, sp) for _, M, K, sp, _ in allm], world)[rank]
        timed_m, mine_t = allm, shard
        # warm-up: for every format this rank will use, 256 rows of its first matrix of that format, --warmup times
        # (module loading, library handles); the memory pools grow in the untimed pass before the timing
        seen, mine_w = set(), []
        for i in shard:
            if allm[i][3] not in seen:
                seen.add(allm[i][3])
                mine_w.append(i)
        warm_m = allm
        rows, row_reduce = None, None
        fmts = load_formats(list(MENU_TCQPQ), dev)
    damp = 0.02
    hcache: dict = {}

    def jobs_of(mats, idx, max_rows=None):
        out = []
        for i in idx:
            name, M, K, sp, hk = mats[i]
            if hk not in hcache:
                hcache[hk] = synth_hessian(K, 1024 if moe and hk[1][:2] in ("gu", "dn") else 4096, _seed_of(hk), dev)
            W = synth_weight(M, K, _seed_of(name), dev)
            if rows is not None:
                r0, r1 = rows[M]
                W = W[r0:r1].contiguous()
            if max_rows is not None:
                W = W[:max_rows].contiguous()
            out.append((W, hcache[hk], sp))
        return out

    if moe:  # --warmup whole layers, once
        quantize_matrices(jobs_of(warm_m, mine_w), damp=damp, n_streams=args.streams, ltq_formats=fmts, pack=False,
                          row_reduce=row_reduce)
    else:
        warm = jobs_of(warm_m, mine_w, max_rows=256)
        for _ in range(args.warmup):
            quantize_matrices(warm, damp=damp, n_streams=args.streams, ltq_formats=fmts, pack=False)
        del warm
        hcache.clear()
    timed = jobs_of(timed_m, mine_t)
    weights_total = sum(M * K for _, M, K, _, _ in (timed_m[i] for i in range(len(timed_m))))
    weights_mine = sum(W.numel() for W, _, _ in timed)

    # end to end first (its untimed first pass also grows the streams' memory pools to the whole run's size and sets
    # up NCCL's point-to-point connections), then the device-resident timing
    e2e_ms, h2d, d2h = None, 0, 0
    host_need = sum(W.numel() * 2 for W, _, _ in timed) + sum(H.numel() * 4 for H in hcache.values())
    host_ram = os.sysconf("SC_PHYS_PAGES") * os.sysconf("SC_PAGE_SIZE")
    if not args.no_e2e and host_need * world > 0.6 * host_ram:
        print(f"rank {rank}: e2e skipped: {host_need * world / 1e9:.0f} GB of pinned inputs on a "
              f"{host_ram / 1e9:.0f} GB host", file=sys.stderr, flush=True)
        args.no_e2e = True
    if not args.no_e2e:
        # from pinned host memory to the packed tensors of every matrix in rank 0's host memory: host-to-device copies
        # on the matrices' streams, quantization, one NCCL gather of all ranks' packed tensors, device-to-host copies
        hosts = {}
        host = []
        for W, H, sp in timed:
            if id(H) not in hosts:
                hosts[id(H)] = H.cpu().pin_memory()
            host.append((W.cpu().pin_memory(), hosts[id(H)], sp))
        h2d = sum(W.numel() * 2 + H.numel() * 4 for W, H, _ in host)
        gid = [(i * world + rank if by_rows else i) for i in mine_t]

        def e2e():
            r = quantize_matrices(host, damp=damp, n_streams=args.streams, ltq_formats=fmts, pack=False,
                                  row_reduce=row_reduce, to_host=dist is None)
            if dist is None:
                return {g: x["ltq"] for g, x in zip(gid, r)}
            return gather_ltq({g: x["ltq"] for g, x in zip(gid, r)}, dst=0)
        e2e()  # untimed once
        got, e2e_ms, _, _ = _timed(e2e, barrier, local)
        if rank == 0 and got is not None:
            d2h = sum(sum(t.numel() * t.element_size() for k, t in d.items() if k in ("data", "d_row", "e", "suh"))
                      for d in got.values())
        del host, hosts, got
    else:  # the untimed pass that grows the memory pools
        quantize_matrices(timed, damp=damp, n_streams=args.streams, ltq_formats=fmts, pack=False,
                          row_reduce=row_reduce)
    barrier()
    Lq.BLOCK_EVENTS = []
    k0 = _lib.kernels_launched()
    res, dev_ms, clocks, t0 = _timed(lambda: quantize_matrices(timed, damp=damp, n_streams=args.streams,
                                                              ltq_formats=fmts, pack=False, row_reduce=row_reduce),
                                     barrier, local)
    launches = _lib.kernels_launched() - k0
    ev, Lq.BLOCK_EVENTS = Lq.BLOCK_EVENTS, None
    roof = _block_roofline(ev, t0)
    rel = float(np.mean([r["rel_loss"] for r in res]))
    packed = sum(int(r["ltq"]["data"].numel()) for r in res)
    dev_ms, e2e_max, per_rank_weights = _max_over_ranks(dist, dev, dev_ms, e2e_ms or 0.0, weights_mine)
    if rank != 0:
        return
    steps = 1 if not moe else args.steps
    line = {
        "metric": METRIC, "value": weights_total / (dev_ms * 1e-3) / 1e6, "unit": METRIC, "n_gpus": world,
        "steps": steps, "warmup": args.warmup, "ms_per_step": dev_ms / steps, "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic (seeded; config-2 weight and Hessian distributions)",
        "config": ({"workload": "qwen3-30b-a3b_moe_" + ("rowshard" if by_rows else "by_matrix") +
                                "_tcq45x_attn_tcq275x_experts",
                    "step": "one MoE layer: q 4096x2048, k/v 512x2048, o 2048x4096 at TCQ45X; 128 experts x "
                            "(gate_up 1536x2048, down 2048x768) at TCQ275X; 623 M weights",
                    "layers_timed": args.steps, "hessian_rows": "4096 (attention), 1024 per expert",
                    "parallelism": (f"rows of every matrix over {world} ranks, 5 NCCL all-reduces per matrix"
                                    if by_rows else f"whole matrices over {world} ranks (longest first), no "
                                    "data-path collective")}
                   if moe else
                   {"workload": "qwen3-8b_model_by_matrix_tcqpq_menu",
                    "step": "the whole model: 36 layers x (q/o 4096x4096, k/v 1024x4096, gate/up 12288x4096, down "
                            "4096x12288) = 6.946 G weights, formats cycling the 19-format TCQPQ menu",
                    "hessians": "one per input: attention (q/k/v), o, MLP (gate/up), down",
                    "parallelism": f"whole matrices over {world} ranks (longest first), no data-path collective",
                    "model_seconds": dev_ms / 1e3}) | {
            "damp": damp * 10, "tb_window": TB_WINDOW, "streams": args.streams, "weights_total": weights_total,
            "max_weights_per_rank": int(per_rank_weights), "rel_loss_mean_rank0": rel, "ltq_bytes_rank0": packed,
            "l2": "inputs larger than L2"},
        "roofline": roof, "cpu_baseline": None,
        "e2e": None if e2e_ms is None else {
            "value": weights_total / (e2e_max * 1e-3) / 1e6, "unit": METRIC, "seconds": e2e_max / 1e3,
            "h2d_bytes_per_step": int(h2d // steps), "d2h_bytes_per_step": int(d2h // steps),
            "scope": "pinned host W / H -> packed .ltq tensors of every matrix in rank 0's host memory"},
        "gpu_launches": int(launches), "clocks": clocks}
    print(json.dumps(line), flush=True)


def run_rings(args, rank, world, dev, dist, barrier, local):
    """Config 5: a 262,144 x 2,560 bf16 table (N(0, 0.03) x a log-normal(0, 0.5) row scale) quantized as 256-value
    tail-biting rings of TCQ4X after the Hadamard-256 rotation, three ring-scale tries (src/ple_quant.py:37-65).  The
    rows are split across the ranks (independent rings, no collective); a step is the whole table, strong scaling."""
    from ltq_research_b200 import _lib
    from ltq_research_b200.rings import quantize_rings
    from ltq_research_b200.shard import row_ranges
    R, C = args.ring_rows, 2560
    r0, r1 = row_ranges(R, world, multiple=16)[rank]

    def table(a, b, seed):
        g = torch.Generator(device=dev).manual_seed(seed)
        T = torch.empty(b - a, C, dtype=torch.bfloat16, device=dev)
        for c0 in range(0, b - a, 16384):  # row blocks, each from its own seed: any rank split gives the same table
            n = min(16384, b - a - c0)
            g.manual_seed(seed + a + c0)
            T[c0:c0 + n] = (torch.randn(n, C, device=dev, generator=g) * 0.03 *
                            torch.exp(0.5 * torch.randn(n, 1, device=dev, generator=g))).to(torch.bfloat16)
        return T

    Tm = table(r0, r1, 5)
    warm = Tm[: min(Tm.shape[0], (1 << 17) // (C // 256) + 1)]  # one full chunk of rings: the pool's working size
    for _ in range(args.warmup):
        quantize_rings(warm, "TCQ4X", True)
    barrier()
    k0 = _lib.kernels_launched()
    (out, _), dev_ms, clocks, _ = _timed(lambda: quantize_rings(Tm, "TCQ4X", True), barrier, local)
    launches = _lib.kernels_launched() - k0
    rel = float(((out.float() - Tm.float()).square().sum() / Tm.float().square().sum()).item())
    del out
    e2e_ms = None
    if not args.no_e2e:
        host = Tm.cpu().pin_memory()
        quantize_rings(host[:2048], "TCQ4X", True, device=dev)
        _, e2e_ms, _, _ = _timed(lambda: quantize_rings(host, "TCQ4X", True, device=dev), barrier, local)
    dev_ms, e2e_max = _max_over_ranks(dist, dev, dev_ms, e2e_ms or 0.0)
    if rank != 0:
        return
    values = R * C
    peak, sm_mhz = alu_peak_gacs()
    acs = values * 2 * 1024 * 4 * 3  # two full passes x 1024 states x 4 gain candidates x 3 scale tries
    line = {
        "metric": METRIC, "value": values / (dev_ms * 1e-3) / 1e6, "unit": METRIC, "n_gpus": world, "steps": 1,
        "warmup": args.warmup, "ms_per_step": dev_ms, "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded; N(0, 0.03) x log-normal(0, 0.5) row scale)",
        "config": {"workload": "ple_rings_262144x2560_tcq4x_rot_3tries", "table": [R, C], "format": "TCQ4X",
                   "rotation": "Hadamard-256 with signs(4242)", "tries": [0.9, 1.0, 1.12], "rel_mse": rel,
                   "parallelism": f"rows over {world} ranks, no collective", "unit_note": "weights = table values"},
        "roofline": {"bound": "alu", "kernel": "vit_fwd_kernel (stand-alone tail-biting Viterbi) and the whole step",
                     "achieved": acs / world / (dev_ms * 1e-3) / 1e9, "peak": peak, "unit": "GACS/s",
                     "frac": acs / world / (dev_ms * 1e-3) / 1e9 / peak, "traffic": None,
                     "basis": "per GPU: its values x 2 passes x 1024 states x 4 slots x 3 tries / the step's time"},
        "cpu_baseline": None,
        "e2e": None if e2e_ms is None else {
            "value": values / (e2e_max * 1e-3) / 1e6, "unit": METRIC, "seconds": e2e_max / 1e3,
            "h2d_bytes_per_step": int(values * 2), "d2h_bytes_per_step": int(values * 2),
            "scope": "pinned host table rows -> reconstructed rows in each rank's host memory"},
        "gpu_launches": int(launches), "clocks": clocks}
    print(json.dumps(line), flush=True)


def run_gaussian(args, rank, world, dev, dist, barrier, local):
    """Config 1, the reference's Gaussian rig (src/universal_bench.py:120-130 with the BASELINE choices): a 4096 x 4096
    N(0, 1) matrix from torch's CPU generator seeded 0 (rank r: seed r, weak scaling), cut into 65,536 tiles of
    16 x 16 (src/ltq_file.py:69-72), each divided by its fp16 RMS and quantized with the K = 2, 4-subset, 2-bit-gain
    tail-biting TCQ of results/universal_gaussian.json (full first pass, unit weights); per-weight MSE reported."""
    from ltq_research_b200 import _lib
    from ltq_research_b200.formats import GAUSSIAN_RIG_K2H2 as RIG
    from ltq_research_b200.tcq_proto import make_gains, viterbi_ub_cuda
    W = torch.randn(4096, 4096, generator=torch.Generator().manual_seed(rank)).to(dev)
    x = W.reshape(256, 16, 256, 16).permute(0, 2, 1, 3).reshape(-1, 256).contiguous()
    d = x.square().mean(dim=1, keepdim=True).sqrt().half().float()
    tab = torch.tensor(RIG["lut"], dtype=torch.float32, device=dev)
    gains = make_gains(RIG["h"], RIG["step"], dev)

    def step():
        return viterbi_ub_cuda(x / d, tab, 2, 10, 359, gains, sub=16, tail_biting=True) * d
    for _ in range(args.warmup):
        step()
    barrier()
    k0 = _lib.kernels_launched()

    def many():
        for _ in range(args.steps):
            r = step()
        return r
    rec, dev_ms, clocks, _ = _timed(many, barrier, local)
    launches = _lib.kernels_launched() - k0
    mse = float((rec - x).square().mean().item())
    e2e_ms = None
    if not args.no_e2e:
        hx = W.cpu().pin_memory()
        out = torch.empty(4096, 4096, pin_memory=True)

        def e2e():
            for _ in range(args.steps):
                Wd = hx.to(dev, non_blocking=True)
                xt = Wd.reshape(256, 16, 256, 16).permute(0, 2, 1, 3).reshape(-1, 256).contiguous()
                dd = xt.square().mean(dim=1, keepdim=True).sqrt().half().float()
                r = viterbi_ub_cuda(xt / dd, tab, 2, 10, 359, gains, sub=16, tail_biting=True) * dd
                out.copy_(r.reshape(256, 256, 16, 16).permute(0, 2, 1, 3).reshape(4096, 4096), non_blocking=True)
        _, e2e_ms, _, _ = _timed(e2e, barrier, local)
    dev_ms, e2e_max = _max_over_ranks(dist, dev, dev_ms, e2e_ms or 0.0)
    if rank != 0:
        return
    total = 4096 * 4096 * args.steps * world
    peak, sm_mhz = alu_peak_gacs()
    ach = 4096 * 4096 * args.steps * 8192 / (dev_ms * 1e-3) / 1e9
    line = {
        "metric": METRIC, "value": total / (dev_ms * 1e-3) / 1e6, "unit": METRIC, "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": dev_ms / args.steps, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded N(0, 1), CPU generator)",
        "config": {"workload": "gaussian_rig_4096x4096_tcq_k2_h2_tb", "tiles_per_step": 65536,
                   "format": "K 2, nu 10, mask 359, 4 subsets, h 2 (step 0.3), sub 16, tail-biting, full first pass",
                   "mse_per_weight": mse, "parallelism": f"dp{world} (one matrix per rank)",
                   "l2": "inputs 64 MB + survivor streams 1 GB per step (above L2)"},
        "roofline": {"bound": "alu", "kernel": "vit_fwd_kernel (stand-alone tail-biting Viterbi)",
                     "achieved": ach, "peak": peak, "unit": "GACS/s", "frac": ach / peak, "traffic": None,
                     "basis": "16.8 M weights x 8192 ACS (2 passes x 1024 states x 4 slots) per step / step time"},
        "cpu_baseline": None,
        "e2e": None if e2e_ms is None else {
            "value": total / (e2e_max * 1e-3) / 1e6, "unit": METRIC, "h2d_bytes_per_step": 4096 * 4096 * 4,
            "d2h_bytes_per_step": 4096 * 4096 * 4},
        "gpu_launches": int(launches), "clocks": clocks}
    print(json.dumps(line), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=8)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="mine", choices=["mine", "reference"])
    ap.add_argument("--workload", default="llama3.2-3b",
                    choices=["llama3.2-3b", "gaussian", "qwen3-8b", "qwen3-30b-a3b", "ple-rings"],
                    help="BASELINE config: llama3.2-3b (config 2, the headline; a step is one decoder layer), "
                         "gaussian (config 1), qwen3-8b (config 3, the whole model per step), qwen3-30b-a3b (config "
                         "4, one MoE layer per step), ple-rings (config 5, the whole table per step)")
    ap.add_argument("--ring-rows", type=int, default=262144, help="rows of the config-5 table")
    ap.add_argument("--moe-shard", default="rows", choices=["rows", "matrices"],
                    help="config 4: split every matrix's rows across the ranks (the config's row sharding), or give "
                         "each rank whole matrices (experts and attention, longest first; no collective)")
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
    ap.add_argument("--profile-gemm", action="store_true",
                    help="the tcgen05 six-product GEMM of the LDLQ update at 8192 x 2816 and 8192 x 7936 (K = 3 x 256), "
                         "three launches each, untimed, for ncu captures")
    ap.add_argument("--profile-hbm", action="store_true",
                    help="the HBM-bound kernels (FWHT-256, scale fit, pack, verify decode) on a 16384 x 4096 matrix, "
                         "three launches each, untimed, for ncu captures")
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
    if args.profile_gemm:
        from ltq_research_b200 import _lib
        L = _lib.lib()
        st = torch.cuda.current_stream(dev).cuda_stream
        g = torch.Generator(device=dev).manual_seed(9)
        for M, N in ((8192, 2816), (8192, 7936)):
            A3 = torch.randn(M, 768, device=dev, generator=g).to(torch.bfloat16)
            B3 = torch.randn(N, 768, device=dev, generator=g).to(torch.bfloat16)
            C = torch.randn(M, N, device=dev, generator=g)
            for _ in range(3):
                rc = L.ltq_gemm_bf16x6_tn(A3.data_ptr(), 768, B3.data_ptr(), 768, C.data_ptr(), N, M, N, 256, -1.0, 1.0,
                                          None, st)
                assert rc == 0, rc
        torch.cuda.synchronize()
        print("profile run: tcgen05 LDLQ-update GEMM, 8192 x 2816 and 8192 x 7936, 3 launches each", flush=True)
        return
    if args.profile_hbm:
        hbm_kernels(dev, fmts["TCQ3X"], reps=3, timed=False)
        print("profile run: HBM-bound kernels on 16384 x 4096, 3 launches each", flush=True)
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

    if args.workload != "llama3.2-3b":
        run = {"gaussian": run_gaussian, "qwen3-8b": run_matrix_model, "qwen3-30b-a3b": run_matrix_model,
               "ple-rings": run_rings}[args.workload]
        run(args, rank, world, dev, dist, barrier, local)
        if dist is not None:
            dist.barrier()
            dist.destroy_process_group()
        return

    # inputs of the warm-up and timed layers, resident in HBM (each layer's H and W, ~0.7 GB, far above the 126 MB L2);
    # the warm-up quantizes --warmup layers untimed; then, when the timed region holds more layers than the warm-up,
    # one untimed priming pass over the timed layers grows the streams' memory pools to the size the timed region's
    # concurrency needs (otherwise the timed region would time the caching allocator's device allocations)
    warm = [j for l in range(args.warmup) for j in layer_jobs(10_000 + l, rank, dev)]
    timed = [j for l in range(args.steps) for j in layer_jobs(l, rank, dev)]
    quantize_matrices(warm, n_streams=args.streams, ltq_formats=fmts, pack=False)
    primed = args.steps > args.warmup
    if primed:
        quantize_matrices(timed, n_streams=args.streams, ltq_formats=fmts, pack=False)
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
                       "pool_priming": ("one untimed pass over the timed layers after the warm-up (memory pools)"
                                        if primed else "none (warm-up >= timed layers)"),
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
