#!/usr/bin/env python
"""Benchmark of the B200 W4A8 ConvRot qlinear (the driver's contract: one JSON line on rank 0).

Workload (per GPU): the qlinear shape sweep at DiT width 5120 -- projections (K, N) in
{(5120, 5120), (5120, 13824), (13824, 5120)} at M in {256, 2048, 16384, 65536} tokens, bf16 activations (N(0, 1), 0.5%
outlier channels x20), int4 group-128 weights with fp16 scales.  One step = one W4A8 linear (rotate+quantise, decode,
tcgen05 GEMM + epilogue) at each of the 12 points.  Inputs are resident in HBM; each step streams ~8 GB, far more than
the 126 MB L2, so no step reads the previous one's data from L2.

Multi-GPU (torchrun, one rank per GPU): the path is token-wise, so each rank runs the same sweep on its own token shard
with no data-path collective ("scaling": "weak"); the time is the max over ranks, `value` the ops of all ranks / time.

  value     whole-job int8 TOPS (2*M*N*K per linear), device-timed over the K timed steps
  e2e       the same metric through the public API `qlinear.linear` with pinned HOST input and output: every step
            copies each point's activations host->device and its output device->host inside the timed region
  roofline  the GEMM kernel (dominant): algorithmic ops per launch / its CUDA-event duration, against the int8 peak
            (2x the measured bf16 dense peak of MEASURED_PEAKS.json); rotate+quantise reported likewise against HBM
  cpu_baseline  the oracle (a numpy restatement of the reference's CPU qlinear) on a bounded row sample, all host
            cores, extrapolated per token (the path is token-wise) to the same sweep

`--impl reference` runs only the reference's CPU algorithm (the oracle port) on rank 0 and prints its line.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
SWEEP = [(5120, 5120), (5120, 13824), (13824, 5120)]  # (K, N)
MS = [256, 2048, 16384, 65536]
METRIC = "W4A8 qlinear int8 TOPS"


def load_package():
    import importlib.util

    name = "minimax_h3_turbo_b200"
    if name in sys.modules:
        return sys.modules[name]
    pkg = ROOT / "minimax-h3-turbo_b200"
    spec = importlib.util.spec_from_file_location(name, pkg / "__init__.py", submodule_search_locations=[str(pkg)])
    mod = importlib.util.module_from_spec(spec)
    sys.modules[name] = mod
    spec.loader.exec_module(mod)
    return mod


def sweep_points(ms):
    return [(k, n, m) for (k, n) in SWEEP for m in ms]


def ops_of(points):
    return sum(2.0 * m * n * k for (k, n, m) in points)


def peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return {"hbm_gbs": d["hbm_gbs"], "bf16": d["bf16_tflops"], "bf16_sustained": d.get("bf16_tflops_sustained"),
                "source": "measured"}
    return {"hbm_gbs": 6650.0, "bf16": 1590.0, "bf16_sustained": 1400.0, "source": "fallback"}


# ------------------------------------------------------------------------------------------------ clocks
class ClockSampler:
    """nvidia-smi samples (every 50 ms) of SM clock and throttle reasons while the timed region runs."""

    FIELDS = ("clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
              "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
              "clocks_event_reasons.sw_power_cap")

    def __init__(self, device_index: int):
        import torch

        self.sel = str(device_index)
        try:  # the physical GPU behind this CUDA device: match its UUID in nvidia-smi's list
            want = str(torch.cuda.get_device_properties(device_index).uuid).lower().replace("gpu-", "")
            out = subprocess.run(["nvidia-smi", "--query-gpu=index,uuid", "--format=csv,noheader"], capture_output=True,
                                 text=True, timeout=20).stdout.strip().splitlines()
            rows = [[c.strip() for c in line.split(",")] for line in out if line.strip()]
            hit = [r[0] for r in rows if len(r) > 1 and r[1].lower().replace("gpu-", "") == want]
            if hit:
                self.sel = hit[0]
            elif len(rows) == 1:
                self.sel = rows[0][0]
        except Exception:
            pass
        self.proc = None

    def start(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                                          "-lms", "50", "-i", self.sel], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL,
                                         text=True)
        except OSError:
            self.proc = None

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            out, _ = self.proc.communicate(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
            out, _ = self.proc.communicate()
        sm, smax, power, reasons = [], [], [], set()
        names = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")
        for line in out.strip().splitlines():
            f = [c.strip() for c in line.split(",")]
            if len(f) < 8:
                continue
            try:
                sm.append(float(f[0]))
                smax.append(float(f[1]))
                power.append(float(f[2]))
            except ValueError:
                continue
            for nm, v in zip(names, f[4:8]):
                if v.lower() == "active":
                    reasons.add(nm)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(smax) if smax else None,
                "power_w_max": max(power) if power else None, "samples": len(sm), "reasons": sorted(reasons)}


# ------------------------------------------------------------------------------------------------ CPU (oracle) leg
_CPU_WEIGHTS = {}


def cpu_reference_rate(ms, rows: int, reps: int = 1, seed: int = 0):
    """The reference's CPU algorithm (oracle port) on a bounded sample: per projection, one full weight decode (the
    reference decodes on every call) plus quantise + exact int8 GEMM + epilogue on `rows` rows.  Extrapolated per token
    (token-wise path) to the sweep: t(M) = t_decode + M * t_row.  Returns (TOPS, detail)."""
    import numpy as np

    sys.path.insert(0, str(ROOT))
    from oracle import qlinear_oracle as orc

    total_t, detail = 0.0, []
    for (k, n) in SWEEP:
        key = (k, n, seed)
        if key not in _CPU_WEIGHTS:  # generated once per process, outside the timed part
            _CPU_WEIGHTS[key] = orc.synth_weight_int4_g128(n, k, seed=seed + k + n)
        q, s_rel, s_ch, cb = _CPU_WEIGHTS[key]
        x = orc.synth_activation(rows, k, seed=seed, outlier_frac=0.005)
        t_dec, t_rows = [], []
        for _ in range(reps):
            t0 = time.perf_counter()
            grid = orc.decode_int8_grid(q, s_rel, "fp16", cb, 128)
            t1 = time.perf_counter()
            codes, xs = orc.quantize_rows(x, "bf16")
            acc = orc.int8_mm(codes, grid)
            orc.epilogue(acc, xs, s_ch, None, "bf16")
            t2 = time.perf_counter()
            t_dec.append(t1 - t0)
            t_rows.append((t2 - t1) / rows)
        td, tr = min(t_dec), min(t_rows)
        for m in ms:
            total_t += td + m * tr
        detail.append({"K": k, "N": n, "decode_s": round(td, 4), "per_row_ms": round(tr * 1e3, 4)})
    return ops_of(sweep_points(ms)) / total_t / 1e12, detail


def run_reference(args, rank):
    if rank != 0:
        return
    import numpy as np  # noqa: F401

    cores = os.cpu_count() or 1
    ms = args.ms
    rows = args.ref_rows
    vals = []
    for i in range(args.warmup + args.steps):
        v, detail = cpu_reference_rate(ms, rows)
        if i >= args.warmup:
            vals.append(v)
    value = statistics.median(vals)
    line = {"metric": METRIC, "value": value, "unit": "TOPS", "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": ops_of(sweep_points(ms)) / (value * 1e12) * 1e3, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "int8", "data": "synthetic", "impl": "reference",
            "config": config_dict(ms, args.gpus),
            "cpu_baseline": {"value": value, "unit": "TOPS", "cores": cores, "kind": "port",
                             "sample": f"{rows} rows per projection + one full weight decode per projection, per-token "
                                       f"extrapolation to the sweep (numpy oracle of the reference CPU path, {cores} threads)",
                             "detail": detail},
            "e2e": {"value": value, "unit": "TOPS", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def config_dict(ms, world):
    return {"workload": "config2 qlinear sweep per GPU: (K,N) in " + str(SWEEP) + f" x M in {ms}",
            "model": "H3 DiT W4A8 ConvRot qlinear (width 5120, FFN 13824)", "weights": "int4 group-128, fp16 scales",
            "activations": "bf16 N(0,1), 0.5% outlier channels x20", "global_tokens_per_point": [m * world for m in ms],
            "parallelism": f"token-shard x{world}", "l2": "inputs larger than L2 (each step streams ~8 GB)"}


# ------------------------------------------------------------------------------------------------ GPU leg
def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="h3b", choices=["h3b", "reference"])
    ap.add_argument("--ms", default=",".join(map(str, MS)))
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--cpu-rows", type=int, default=256)
    ap.add_argument("--ref-rows", type=int, default=256)
    ap.add_argument("--detail", default="", help="write per-point timings to this JSON file")
    args = ap.parse_args()
    args.ms = [int(v) for v in args.ms.split(",") if v]
    rank, world, local = int(os.environ.get("RANK", 0)), int(os.environ.get("WORLD_SIZE", 1)), int(os.environ.get("LOCAL_RANK", 0))
    if args.warmup < 3:
        print("bench.py: --warmup must be >= 3", file=sys.stderr)
        sys.exit(2)
    if args.impl == "reference":
        run_reference(args, rank)
        return

    import torch
    import torch.distributed as dist
    from datetime import timedelta

    load_package()
    from minimax_h3_turbo_b200 import _lib
    from minimax_h3_turbo_b200.h3 import qlinear as ql
    from minimax_h3_turbo_b200.h3.synth import synthetic_activation, synthetic_w4a8

    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=dev)
    L = _lib.lib()
    stream = torch.cuda.current_stream(dev)
    sp = stream.cuda_stream
    points = sweep_points(args.ms)

    # ---- resident inputs: weights per projection, activations per (K, M) (the two K=5120 projections share them)
    weights, grids = {}, {}
    for (k, n) in SWEEP:
        w = synthetic_w4a8(n, k, seed=k + n, device=dev)
        weights[(k, n)] = (w, ql._WeightArgs(w))
        grids[(k, n)] = torch.empty(n, k, dtype=torch.int8, device=dev)
    acts = {}
    for (k, m) in sorted({(k, m) for (k, _, m) in points}):
        acts[(k, m)] = synthetic_activation(m, k, seed=1000 * rank + k + m, device=dev)
    outs = {p: torch.empty(p[2], p[1], dtype=torch.bfloat16, device=dev) for p in points}
    mmax, kmax = max(args.ms), max(k for k, _ in SWEEP)
    codes = torch.empty(mmax * kmax, dtype=torch.int8, device=dev)
    xs = torch.empty(mmax, dtype=torch.float32, device=dev)

    def step(evs=None):
        """One pass of the hot path over every sweep point: KA (rotate+quantise), decode, KB (GEMM + epilogue)."""
        for i, (k, n, m) in enumerate(points):
            w, a = weights[(k, n)]
            x = acts[(k, m)]
            if evs is not None:
                evs[i][0].record(stream)
            _lib.check(L.h3b_rotq(x.data_ptr(), _lib.BF16, m, k, k, 256, 0, 0, codes.data_ptr(), k, xs.data_ptr(), sp), "rotq")
            if evs is not None:
                evs[i][1].record(stream)
            g = grids[(k, n)]
            _lib.check(L.h3b_decode_grid(a.q.data_ptr(), n, k, a.ldq, a.s.data_ptr(), a.s_dtype, a.lds, a.cb.data_ptr(), 128,
                                         g.data_ptr(), k, sp), "decode")
            if evs is not None:
                evs[i][2].record(stream)
            o = outs[(k, n, m)]
            _lib.check(L.h3b_int8_gemm_epilogue(codes.data_ptr(), k, xs.data_ptr(), m, g.data_ptr(), k, a.s_ch.data_ptr(), None,
                                                o.data_ptr(), _lib.BF16, n, n, k, 0, sp), "gemm")
            if evs is not None:
                evs[i][3].record(stream)

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize(dev)

    for _ in range(args.warmup):
        step()
    barrier()

    # ---- timed region: K steps, per-kernel events on the launching stream, clocks sampled throughout
    evs = [[[torch.cuda.Event(enable_timing=True) for _ in range(4)] for _ in points] for _ in range(args.steps)]
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    clocks = ClockSampler(local)
    clocks.start()
    barrier()
    t0.record(stream)
    for s in range(args.steps):
        step(evs[s])
    t1.record(stream)
    barrier()
    clk = clocks.stop()
    elapsed_ms = t0.elapsed_time(t1)
    t_local = torch.tensor([elapsed_ms], device=dev, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(t_local, op=dist.ReduceOp.MAX)
    t_max_ms = float(t_local.item())

    # per-kernel device time over the timed region
    per_point = []
    tot = {"rotq": 0.0, "decode": 0.0, "gemm": 0.0}
    for i, (k, n, m) in enumerate(points):
        r = sum(evs[s][i][0].elapsed_time(evs[s][i][1]) for s in range(args.steps)) / args.steps
        d = sum(evs[s][i][1].elapsed_time(evs[s][i][2]) for s in range(args.steps)) / args.steps
        g = sum(evs[s][i][2].elapsed_time(evs[s][i][3]) for s in range(args.steps)) / args.steps
        tot["rotq"] += r
        tot["decode"] += d
        tot["gemm"] += g
        per_point.append({"K": k, "N": n, "M": m, "rotq_ms": r, "decode_ms": d, "gemm_ms": g,
                          "gemm_tops": 2.0 * m * n * k / (g * 1e-3) / 1e12, "linear_tops": 2.0 * m * n * k / ((r + d + g) * 1e-3) / 1e12,
                          "rotq_gbs": (3.0 * m * k + 4 * m) / (r * 1e-3) / 1e9})
    ops_step = ops_of(points)
    value = world * ops_step * args.steps / (t_max_ms * 1e-3) / 1e12
    pk = peaks()
    int8_peak = 2.0 * pk["bf16"]
    gemm_tops = ops_step / (tot["gemm"] * 1e-3) / 1e12
    rotq_bytes = sum(3.0 * m * k + 4.0 * m for (k, _, m) in points)
    rotq_gbs = rotq_bytes / (tot["rotq"] * 1e-3) / 1e9
    traffic = None
    tf = ROOT / "profiles" / "traffic.json"
    if tf.exists():
        try:
            t = json.loads(tf.read_text()).get("gemm_i8_kernel")
            if t and t.get("bytes_per_op"):
                traffic = t["bytes_per_op"] * ops_step / len(points)  # average bytes per GEMM launch at this workload
        except Exception:
            traffic = None

    # ---- e2e through the public API with pinned host buffers (copies inside the timed region)
    e2e = None
    if not args.no_e2e:
        big_in = max(m * k for (k, _, m) in points)
        big_out = max(m * n for (_, n, m) in points)
        hin = torch.empty(big_in, dtype=torch.bfloat16, pin_memory=True)
        hout = torch.empty(big_out, dtype=torch.bfloat16, pin_memory=True)
        kb, mb = max(((k, m) for (k, _, m) in points), key=lambda t: t[0] * t[1])
        hin[: kb * mb].copy_(acts[(kb, mb)].view(-1))  # realistic values for every point (prefix views of this buffer)
        h2d = sum(m * k * 2 for (k, _, m) in points)
        d2h = sum(m * n * 2 for (_, n, m) in points)

        def e2e_step():
            for (k, n, m) in points:
                w, _ = weights[(k, n)]
                xd = hin[: m * k].view(m, k).to(dev, non_blocking=True)
                y = ql.linear(xd, w)
                hout[: m * n].view(m, n).copy_(y, non_blocking=True)

        e2e_step()
        barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e2e_steps = max(1, min(args.steps, 3))
        barrier()
        e0.record(stream)
        for _ in range(e2e_steps):
            e2e_step()
        e1.record(stream)
        barrier()
        te = torch.tensor([e0.elapsed_time(e1)], device=dev, dtype=torch.float64)
        if world > 1:
            dist.all_reduce(te, op=dist.ReduceOp.MAX)
        e2e = {"value": world * ops_step * e2e_steps / (float(te.item()) * 1e-3) / 1e12, "unit": "TOPS",
               "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h, "steps": e2e_steps,
               "path": "qlinear.linear (public API) per point; pinned host input/output, copies on the compute stream"}

    # ---- CPU baseline (rank 0, single GPU only)
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu:
        cores = os.cpu_count() or 1
        v, detail = cpu_reference_rate(args.ms, args.cpu_rows)
        cpu = {"value": v, "unit": "TOPS", "cores": cores, "kind": "port",
               "sample": f"{args.cpu_rows} rows per projection + one full weight decode per projection, per-token "
                         f"extrapolation to the sweep (numpy oracle of the reference CPU path, {cores} threads)",
               "detail": detail}

    if args.detail and rank == 0:
        Path(args.detail).parent.mkdir(parents=True, exist_ok=True)
        Path(args.detail).write_text(json.dumps({"points": per_point, "totals_ms_per_step": tot, "clocks": clk}, indent=1))

    if rank == 0:
        line = {"metric": METRIC, "value": value, "unit": "TOPS", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
                "ms_per_step": t_max_ms / args.steps, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
                "dtype": "int8", "data": "synthetic", "config": config_dict(args.ms, world),
                "roofline": {"bound": "tensor", "kernel": "gemm_i8_kernel", "achieved": gemm_tops, "peak": int8_peak,
                             "unit": "TOPS", "frac": gemm_tops / int8_peak, "traffic": traffic,
                             "peak_note": f"int8 dense = 2 x {pk['source']} bf16 dense ({pk['bf16']} TFLOP/s burst)",
                             "frac_of_sustained": gemm_tops / (2.0 * pk["bf16_sustained"]) if pk.get("bf16_sustained") else None},
                "rotq_roofline": {"bound": "hbm", "kernel": "rotq_kernel", "achieved": rotq_gbs, "peak": pk["hbm_gbs"],
                                  "unit": "GB/s", "frac": rotq_gbs / pk["hbm_gbs"]},
                "kernel_ms_per_step": tot, "cpu_baseline": cpu, "e2e": e2e, "clocks": clk,
                "gpu_launches": 3 * len(points) * args.steps}
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
