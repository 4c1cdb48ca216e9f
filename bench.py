"""Benchmark of the LTQ TCQ quantizer hot path on B200 (one JSON line on rank 0).

Workload ("Gaussian rig"): one fp32 4096 x 4096 matrix of N(0, 1) values (seed 0, one matrix
per rank: weak scaling), tiled 16 x 16 as src/ltq_file.py:69-72 does (65,536 tiles of 256), each tile divided by its
fp16 rms (scale multiplier 1.0, src/universal_bench.py:124), quantized by the joint TCQ Viterbi with the config-1
format (K = 2, 10-bit trellis memory, mask 359, 4 subsets, h = 2 -> 4 gains per 16 weights, table
results/universal_gaussian.json "tcq_K2_h2"), tail-biting, full-tile first pass.  A step = one quantization of that
matrix.  Metric: Mweights/s quantized (whole job, all ranks).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl mine|reference]
    torchrun --nproc-per-node N bench.py --gpus N ...

--impl reference times the reference algorithm on the host cores: the CPU restatement of the reference Viterbi
(oracle/, the only CPU implementation that can run on the GPU box), all host threads, bounded samples.
"""
from __future__ import annotations

import argparse
import json
import math
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

M_ROWS = M_COLS = 4096
TILE = 256
METRIC = "Mweights/s quantized"
WORKLOAD = "gaussian_rig_4096x4096_tcq_K2_h2_tailbiting"
ACS_PER_WEIGHT = 2 * 1024 * 4   # passes x states x gain slots (tb_window = 0: two full passes)
ALU_SLOTS_PER_ACS = 2           # one path-metric add + half a compare + half a select (issue-slot accounting)
L2_BYTES = 126 * 2 ** 20


def rig_format():
    d = json.loads((ROOT / "ltq_research_b200" / "data" / "tcq_formats.json").read_text())["formats"]["_config1_tcq_K2_h2"]
    return d


def make_tiles(seed: int, device) -> tuple[torch.Tensor, torch.Tensor]:
    """Seeded N(0,1) matrix -> tiles [65536, 256] divided by their fp16 rms, and the rms."""
    g = torch.Generator(device="cpu").manual_seed(seed)
    W = torch.randn(M_ROWS, M_COLS, generator=g)
    tiles = W.reshape(M_ROWS // 16, 16, M_COLS // 16, 16).permute(0, 2, 1, 3).reshape(-1, TILE).contiguous()
    d = tiles.square().mean(dim=1, keepdim=True).sqrt().half().float()
    return (tiles / d).to(device), d.to(device)


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


def cpu_baseline_sample(seconds: float = 15.0) -> dict:
    """The CPU restatement of the reference Viterbi (oracle/) on this host's cores, config-1 tiles, bounded sample."""
    from oracle import oracle as O
    fmt = rig_format()
    threads = len(os.sched_getaffinity(0))
    tiles, _ = make_tiles(0, "cpu")
    x = tiles.numpy()
    done, t0, i = 0, time.perf_counter(), 0
    step = max(threads, 8) * 2
    while time.perf_counter() - t0 < seconds and i + step <= x.shape[0]:
        O.viterbi(x[i:i + step], np.asarray(fmt["lut"], np.float32), 2, 10, 359,
                  np.asarray(fmt["gains_cpu"], np.float32), sub=16, tail_biting=True, n_threads=threads)
        done += step * TILE
        i += step
    el = time.perf_counter() - t0
    return {"value": done / el / 1e6, "unit": METRIC, "cores": threads, "kind": "port",
            "sample": f"{done // TILE} config-1 tiles (tail-biting, 2 passes) in {el:.1f} s with the C restatement of "
                      f"the reference Viterbi (oracle/tcq_oracle.c), {threads} threads"}


def run_reference(args, rank: int, world: int):
    """--impl reference: the reference algorithm on the host cores (the oracle port), rank 0 only."""
    if rank != 0:
        return
    from oracle import oracle as O
    fmt = rig_format()
    threads = len(os.sched_getaffinity(0))
    tiles, _ = make_tiles(0, "cpu")
    x = tiles.numpy()
    n = max(threads * 4, 64)  # tiles per step: a bounded sample of the config-1 matrix
    kw = dict(sub=16, tail_biting=True, n_threads=threads)
    lut, g = np.asarray(fmt["lut"], np.float32), np.asarray(fmt["gains_cpu"], np.float32)
    for k in range(args.warmup):
        O.viterbi(x[:n], lut, 2, 10, 359, g, **kw)
    t0 = time.perf_counter()
    for k in range(args.steps):
        s = (k * n) % (x.shape[0] - n)
        O.viterbi(x[s:s + n], lut, 2, 10, 359, g, **kw)
    el = time.perf_counter() - t0
    v = args.steps * n * TILE / el / 1e6
    line = {"metric": METRIC, "value": v, "unit": METRIC, "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": el / args.steps * 1e3, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "f32", "data": "synthetic", "impl": "reference",
            "config": {"workload": WORKLOAD, "tiles_per_step": n, "parallelism": "host threads"},
            "cpu_baseline": {"value": v, "unit": METRIC, "cores": threads, "kind": "port",
                             "sample": f"{n} config-1 tiles per step, tail-biting, C restatement of the reference "
                                       f"Viterbi (oracle/tcq_oracle.c), {threads} threads"},
            "e2e": {"value": v, "unit": METRIC, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="mine", choices=["mine", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--profile", action="store_true", help="one quantization of --tiles tiles, no timing (ncu runs)")
    ap.add_argument("--tiles", type=int, default=0, help="with --profile: tiles of the config-1 matrix to quantize")
    args = ap.parse_args()
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        run_reference(args, rank, world)
        return
    args.warmup = max(args.warmup, 3)
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist = None
    if world > 1:
        import torch.distributed as dist
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=dev)

    from ltq_research_b200.tcq_proto import viterbi_ub_cuda
    fmt = rig_format()
    small = torch.tensor(fmt["lut"], device=dev)
    gains = torch.tensor(fmt["gains_cpu"], device=dev)
    x, d = make_tiles(rank, dev)
    kw = dict(K=2, nu=10, m=359, sub=16, tail_biting=True, return_code=True)
    if args.profile:
        xs = x[: args.tiles] if args.tiles else x
        rec, gi, idx = viterbi_ub_cuda(xs, small, gains=gains, **kw)
        torch.cuda.synchronize()
        assert torch.equal(rec, gains[gi.long()] * small[idx.long()])
        print(f"profile run: {xs.shape[0]} tiles", flush=True)
        return
    flush = torch.empty(2 * L2_BYTES // 4, dtype=torch.float32, device=dev)

    def step(xx):
        return viterbi_ub_cuda(xx, small, gains=gains, **kw)

    def barrier():
        if dist is not None:
            dist.barrier()
        torch.cuda.synchronize()

    for _ in range(args.warmup):
        step(x)
    barrier()
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    with ClockSampler(local) as clk:
        barrier()
        t_wall = time.perf_counter()
        for k in range(args.steps):
            flush.fill_(float(k))  # L2 flush between timed steps (outside the step's events)
            starts[k].record()
            rec, gi, idx = step(x)
            ends[k].record()
        barrier()
        t_wall = time.perf_counter() - t_wall
    dev_ms = sum(s.elapsed_time(e) for s, e in zip(starts, ends))
    # one Viterbi pass timed alone (forward ACS + traceback kernels), for the ACS roofline
    pass_ms = []
    from ltq_research_b200.tcq_proto import viterbi_ub_cuda as vu
    for k in range(3):
        flush.fill_(float(k))
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        vu(x, small, 2, 10, 359, gains, sub=16, return_end_state=True)
        b.record()
        torch.cuda.synchronize()
        pass_ms.append(a.elapsed_time(b))
    # end to end through the public API: pinned host tiles in, reconstruction and codes back to the host
    xh = x.cpu().pin_memory()
    rec_h = torch.empty(x.shape, dtype=torch.float32).pin_memory()
    code_h = torch.empty(x.shape, dtype=torch.int32).pin_memory()
    e2e_ms = []
    for k in range(max(3, args.steps // 2)):
        flush.fill_(float(k))
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        xd = xh.to(dev, non_blocking=True)
        r, gi, idx = step(xd)
        rec_h.copy_(r, non_blocking=True)
        code_h.copy_((gi << 16) | idx, non_blocking=True)
        b.record()
        torch.cuda.synchronize()
        e2e_ms.append(a.elapsed_time(b))
    # correctness guard on the timed output: recompute one tile sample through the same path
    assert torch.equal(rec, gains[gi.long()] * small[idx.long()])

    t = torch.tensor([dev_ms, statistics.median(pass_ms), statistics.median(e2e_ms)], device=dev)
    if dist is not None:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    dev_ms, pass_med, e2e_med = t.tolist()
    weights_per_rank = M_ROWS * M_COLS
    total = weights_per_rank * world
    ms_step = dev_ms / args.steps
    value = total / (ms_step * 1e-3) / 1e6
    e2e_value = total / (e2e_med * 1e-3) / 1e6
    clocks = clk.summary()
    if rank == 0:
        peaks = measured_peaks()
        sm_mhz = float(peaks.get("sm_max_mhz", 1965.0))
        alu_peak = 148 * 128 * sm_mhz * 1e6 / ALU_SLOTS_PER_ACS / 1e9  # GACS/s at full issue of every SMSP
        acs_per_pass = weights_per_rank * ACS_PER_WEIGHT / 2
        achieved = acs_per_pass / (pass_med * 1e-3) / 1e9
        prof = ROOT / "profiles" / "vit_fwd_config1.json"
        traffic = json.loads(prof.read_text()).get("dram_bytes_per_pass") if prof.exists() else None
        cpu = None if args.no_cpu_baseline else cpu_baseline_sample()
        line = {
            "metric": METRIC, "value": value, "unit": METRIC, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms_step, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": {"workload": WORKLOAD, "matrix": [M_ROWS, M_COLS], "tiles_per_rank": weights_per_rank // TILE,
                       "format": "K=2 nu=10 m=359 nl=4 h=2 sub=16 tail-biting tb_window=0",
                       "parallelism": f"dp{world} (one matrix per rank)", "l2": "flushed between timed steps",
                       "wall_s": t_wall},
            "roofline": {"bound": "alu", "kernel": "viterbi pass (vit_fwd_kernel + vit_tb_kernel)",
                         "achieved": achieved, "peak": alu_peak, "unit": "GACS/s", "frac": achieved / alu_peak,
                         "traffic": traffic,
                         "peak_basis": f"148 SMs x 128 issue slots/clk x {sm_mhz:.0f} MHz (MEASURED_PEAKS sm_max_mhz) "
                                       f"/ {ALU_SLOTS_PER_ACS} slots per ACS"},
            "cpu_baseline": cpu,
            "e2e": {"value": e2e_value, "unit": METRIC, "h2d_bytes_per_step": int(xh.numel() * 4),
                    "d2h_bytes_per_step": int(rec_h.numel() * 4 + code_h.numel() * 4)},
            "gpu_launches": 4 * args.steps,
            "clocks": clocks,
        }
        print(json.dumps(line), flush=True)
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
