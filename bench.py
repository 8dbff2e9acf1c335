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

  sharded_block  BASELINE config 5 (59440 tokens, 4 W4A8 DiT blocks) token-sharded over the N ranks: tokens/s, ms per
            forward, the W4A8 linears / attention / exposed key-value exchange per forward, NCCL ranks, and (N > 1) a
            check of 256 gathered rows against the whole sequence recomputed on rank 0 alone
  block     (N = 1) BASELINE config 3: one DiT block on 12290 tokens, tokens/s

`--impl reference` runs the reference's own CPU qlinear (staged under oracle/_ref by oracle/make_ref.py; the numpy port
of it when absent) on rank 0, and times the reference's portable CUDA path beside it.
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
WORKLOADS = ("sweep", "block", "stream", "longseq")
# (K, N, M) -> DRAM bytes read + written by that point's GEMM launch (ncu, one capture of the sweep's launches)
GEMM_DRAM_BYTES = {(5120, 5120, 256): 14918400, (5120, 5120, 2048): 36766976 + 5376,
                   (5120, 5120, 16384): 197843968 + 149336576, (5120, 5120, 65536): 704727296 + 654303744,
                   (5120, 13824, 256): 37935616, (5120, 13824, 2048): 85519360 + 23642368,
                   (5120, 13824, 16384): 332693504 + 413625088, (5120, 13824, 65536): 1164723200 + 1776166144,
                   (13824, 5120, 256): 40125696, (13824, 5120, 2048): 155100672 + 8222720,
                   (13824, 5120, 16384): 1039225600 + 160625152, (13824, 5120, 65536): 4936572672 + 723166976}
HID, HEADS, HEAD_DIM, FFN = 5120, 40, 128, 13824  # DiT width, attention heads x head dim, SwiGLU width
BLOCK_LINEARS = [(HID, 3 * HID), (HID, HID), (HID, 2 * FFN), (FFN, HID)]  # (K, N): qkv, out, fc1, fc2 (SwiGLU input)
BLOCK_OPS_PER_TOKEN = sum(2.0 * k * n for k, n in BLOCK_LINEARS)  # 634.4 M
# token sequences: latent frames x patch rows x patch cols of video + audio tokens, and how many blocks run on them
SEQS = {"block": (31, 26, 15, 200, 1),  # 5 s 832x480: 12090 + 200 = 12290 tokens, one block
        "longseq": (241, 20, 12, 1600, 4)}  # 40 s 640x384: 57840 + 1600 = 59440 tokens, four blocks
STREAM_BLOCKS, STREAM_TOKENS, STREAM_RESIDENT, STREAM_RING, STREAM_PREFETCH = 48, 4096, 4, 3, 2
E2E_ROWS = 8192  # tokens per chunk of the end-to-end leg's pipeline


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
        """Start sampling and wait (up to 5 s) for the first sample, so the timed region that follows is covered."""
        import threading

        self.lines, self.t_begin, self.t_end = [], None, None
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                                          "-lms", "50", "-i", self.sel], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL,
                                         text=True)
        except OSError:
            self.proc = None
            return
        first = threading.Event()

        def reader():
            for line in self.proc.stdout:
                self.lines.append((time.monotonic(), line))
                first.set()

        self.thread = threading.Thread(target=reader, daemon=True)
        self.thread.start()
        first.wait(5.0)

    def begin(self):
        self.t_begin = time.monotonic()

    def end(self):
        self.t_end = time.monotonic()

    def stop(self):
        """Median SM clock and active throttle reasons of the samples taken between begin() and end() (the nearest
        sample when the region is shorter than the 50 ms sampling period)."""
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        self.thread.join(timeout=5)
        lines = list(self.lines)
        b = self.t_begin if self.t_begin is not None else -1e18
        e = self.t_end if self.t_end is not None else 1e18
        inside = [ln for t, ln in lines if b <= t <= e + 0.05]
        window = "timed region"
        if not inside and lines:
            mid = (b + e) / 2 if self.t_begin is not None and self.t_end is not None else lines[-1][0]
            inside = [min(lines, key=lambda tl: abs(tl[0] - mid))[1]]
            window = "nearest sample (timed region shorter than the sampling period)"
        sm, smax, power, reasons = [], [], [], set()
        names = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")
        for line in inside:
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
                "power_w_max": max(power) if power else None, "samples": len(sm), "window": window,
                "reasons": sorted(reasons)}


# ------------------------------------------------------------------------------------------------ CPU (oracle) leg
_CPU_WEIGHTS = {}


CPU_WEIGHT_ROWS = 1024  # output channels of each weight the CPU sample decodes and multiplies


def cpu_projection_times(projs, rows: int, reps: int = 1, seed: int = 0, wrows: int = CPU_WEIGHT_ROWS):
    """The reference's CPU algorithm (oracle port) on a bounded sample: per (K, N) projection, the weight decode (the
    reference decodes on every call), the quantiser on `rows` tokens, and the exact int8 GEMM + epilogue of those tokens,
    with the decode and the GEMM run on the first `wrows` output channels and scaled by N / wrows (both are linear in
    N; the quantiser is not scaled).  Returns [(K, N, t_decode_s, t_per_row_s)]: the path is token-wise, so a call on M
    rows costs t_decode + M * t_per_row."""
    sys.path.insert(0, str(ROOT))
    from oracle import qlinear_oracle as orc

    res = []
    for (k, n) in projs:
        key = (k, n, seed)
        if key not in _CPU_WEIGHTS:  # generated once per process, outside the timed part
            _CPU_WEIGHTS[key] = orc.synth_weight_int4_g128(n, k, seed=seed + k + n)
        q, s_rel, s_ch, cb = _CPU_WEIGHTS[key]
        nr = min(n, wrows)
        qs, ss, cs = q[:nr], s_rel[:nr], s_ch[:nr]
        x = orc.synth_activation(rows, k, seed=seed, outlier_frac=0.005)
        t_dec, t_rows = [], []
        for _ in range(reps):
            t0 = time.perf_counter()
            grid = orc.decode_int8_grid(qs, ss, "fp16", cb, 128)
            t1 = time.perf_counter()
            codes, xs = orc.quantize_rows(x, "bf16")
            t2 = time.perf_counter()
            acc = orc.int8_mm(codes, grid)
            orc.epilogue(acc, xs, cs, None, "bf16")
            t3 = time.perf_counter()
            t_dec.append((t1 - t0) * n / nr)
            t_rows.append(((t2 - t1) + (t3 - t2) * n / nr) / rows)
        res.append((k, n, min(t_dec), min(t_rows)))
    return res


def cpu_reference_rate(ms, rows: int, reps: int = 1, seed: int = 0):
    """CPU TOPS of the sweep, extrapolated per token from cpu_projection_times.  Returns (TOPS, detail)."""
    total_t, detail = 0.0, []
    for (k, n, td, tr) in cpu_projection_times(SWEEP, rows, reps, seed):
        total_t += sum(td + m * tr for m in ms)
        detail.append({"K": k, "N": n, "decode_s": round(td, 4), "per_row_ms": round(tr * 1e3, 4)})
    return ops_of(sweep_points(ms)) / total_t / 1e12, detail


def cpu_block_rate(tokens: int, n_blocks: int, rows: int):
    """CPU tokens/s of n_blocks DiT blocks on `tokens` rows counting only the four W4A8 linears (attention, norms and
    RoPE excluded, so this is an upper bound on the CPU block rate), extrapolated per token.  Returns (tokens/s, detail)."""
    total_t, detail = 0.0, []
    for (k, n, td, tr) in cpu_projection_times(BLOCK_LINEARS, rows):
        total_t += n_blocks * (td + tokens * tr)
        detail.append({"K": k, "N": n, "decode_s": round(td, 4), "per_row_ms": round(tr * 1e3, 4)})
    return tokens / total_t, detail


def load_reference():
    """The reference's own qlinear module (h3turbo/h3/qlinear.py, unchanged) staged under oracle/_ref/ by
    oracle/make_ref.py, or None when it has not been staged."""
    import importlib

    ref = ROOT / "oracle" / "_ref"
    if not (ref / "h3turbo" / "h3" / "qlinear.py").is_file():
        return None
    if str(ref) not in sys.path:
        sys.path.insert(0, str(ref))
    ql = importlib.import_module("h3turbo.h3.qlinear")
    types = importlib.import_module("h3turbo.h3.types")
    return ql, types


def reference_weight(types, k, n, seed, device):
    """The benchmark's int4 group-128 weight (the oracle's seeded generator) as the reference's own W4A8Weight."""
    import torch

    sys.path.insert(0, str(ROOT))
    from oracle import qlinear_oracle as orc

    q, s_rel, s_ch, cb = orc.synth_weight_int4_g128(n, k, seed=seed)
    return types.W4A8Weight(torch.from_numpy(q).to(device), torch.from_numpy(s_rel).to(device),
                            torch.from_numpy(s_ch).to(device), torch.from_numpy(cb).to(device), 128, 256)


def reference_activation(m, k, seed, device):
    import torch

    sys.path.insert(0, str(ROOT))
    from oracle import qlinear_oracle as orc

    bits = orc.synth_activation(m, k, seed=seed, outlier_frac=0.005)
    return torch.from_numpy(bits.view("int16").copy()).view(torch.bfloat16).to(device)


def reference_cuda_rate(ql, types, ms, reps=1):
    """TOPS of the reference's own portable CUDA path -- qlinear.linear(..., backend="torch"): its cuBLAS rotation,
    "ck" quantiser, per-call int8 grid decode and torch._int_mm (cuBLASLt), qlinear.py:380-424 -- over the whole sweep
    on cuda:0, one warm-up pass then `reps` timed passes (CUDA events).  Its comfy_kitchen kernels are absent."""
    import torch

    dev = torch.device("cuda", 0)
    pts = sweep_points(ms)
    ws = {(k, n): reference_weight(types, k, n, k + n, dev) for (k, n) in SWEEP}
    xs = {(k, m): reference_activation(m, k, 1000 + k + m, dev) for (k, _, m) in pts}

    def one():
        for (k, n, m) in pts:
            ql.linear(xs[(k, m)], ws[(k, n)], None, backend="torch", quant_mode="ck")

    one()
    torch.cuda.synchronize(dev)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(reps):
        one()
    e1.record()
    torch.cuda.synchronize(dev)
    return ops_of(pts) * reps / (e0.elapsed_time(e1) * 1e-3) / 1e12


def run_reference(args, rank):
    """The reference arm: the reference's own CPU qlinear (oracle/_ref) on the host cores, each step a bounded sample of
    the sweep -- the three projections at M = --ref-rows tokens (2048, a point of the sweep) -- timed as executed.  The
    reference's portable CUDA path is timed over the full sweep beside it.  Without oracle/_ref the numpy port of the
    reference CPU path (oracle/qlinear_oracle.py) stands in, labelled kind "port"."""
    if rank != 0:
        return
    if args.workload != "sweep":
        run_reference_dit(args)
        return
    import torch

    cores = os.cpu_count() or 1
    torch.set_num_threads(cores)
    rows = args.ref_rows
    staged = load_reference()
    sample = [(k, n, rows) for (k, n) in SWEEP]
    if staged is not None:
        ql, types = staged
        ws = {(k, n): reference_weight(types, k, n, k + n, "cpu") for (k, n) in SWEEP}
        xs = {k: reference_activation(rows, k, 1000 + k + rows, "cpu") for (k, _) in SWEEP}

        def step():
            for (k, n, m) in sample:
                ql.linear(xs[k], ws[(k, n)], None, backend="torch", quant_mode="ck")
        kind, what = "reference", "h3turbo.h3.qlinear.linear(x, w, backend='torch', quant_mode='ck') on CPU (the reference's own code)"
    else:
        sys.path.insert(0, str(ROOT))
        from oracle import qlinear_oracle as orc

        wn = {(k, n): orc.synth_weight_int4_g128(n, k, seed=k + n) for (k, n) in SWEEP}
        xn = {k: orc.synth_activation(rows, k, seed=1000 + k + rows, outlier_frac=0.005) for (k, _) in SWEEP}

        def step():
            for (k, n, m) in sample:
                q, s_rel, s_ch, cb = wn[(k, n)]
                orc.linear(xn[k], "bf16", q, s_rel, "fp16", s_ch, cb, 128)
        kind, what = "port", "numpy restatement of the reference CPU qlinear (oracle/qlinear_oracle.py)"
    times = []
    for i in range(args.warmup + args.steps):
        t0 = time.perf_counter()
        step()
        if i >= args.warmup:
            times.append(time.perf_counter() - t0)
    t_step = statistics.median(times)
    value = ops_of(sample) / t_step / 1e12
    cuda = None
    if staged is not None and not args.no_ref_cuda:
        try:
            if torch.cuda.is_available():
                cuda = {"value": reference_cuda_rate(ql, types, args.ms), "unit": "TOPS", "points": "the full sweep",
                        "what": "the reference's portable CUDA path, qlinear.linear(backend='torch') on cuda:0: cuBLAS "
                                "rotation, ck quantiser, per-call grid decode, torch._int_mm (its comfy_kitchen kernels "
                                "are not available)"}
        except Exception as e:  # a library limitation of the reference must not cost the CPU measurement
            cuda = {"value": None, "error": repr(e)[:300]}
    line = {"metric": METRIC, "value": value, "unit": "TOPS", "n_gpus": args.gpus, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": t_step * 1e3, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "int8", "data": "synthetic", "impl": "reference",
            "config": config_dict(args.ms, args.gpus),
            "cpu_baseline": {"value": value, "unit": "TOPS", "cores": cores, "kind": kind,
                             "sample": f"each step: the three sweep projections at M = {rows} tokens (points of the sweep), "
                                       f"timed as executed with {cores} threads: {what}"},
            "reference_cuda_path": cuda,
            "e2e": {"value": value, "unit": "TOPS", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def run_reference_dit(args):
    """Reference arm of the DiT workloads: the block's four W4A8 linears through the reference's own CPU qlinear on a
    bounded token sample (attention, norms and RoPE excluded: an upper bound on the reference's CPU block rate)."""
    import torch

    tokens, nb, _, metric, cfg = dit_shape(args.workload)
    cores = os.cpu_count() or 1
    torch.set_num_threads(cores)
    staged = load_reference()
    rows = args.ref_rows
    if staged is None:
        v, detail = cpu_block_rate(tokens, nb, rows)
        kind, t_ms, sample = "port", tokens / v * 1e3, f"numpy port, {rows}-token sample, extrapolated"
    else:
        ql, types = staged
        ws = [reference_weight(types, k, n, 7 + k + n, "cpu") for (k, n) in BLOCK_LINEARS]
        xs = [reference_activation(rows, k * (2 if j == 3 else 1), 11 + k, "cpu") for j, (k, _) in enumerate(BLOCK_LINEARS)]
        times = []
        for i in range(args.warmup + args.steps):
            t0 = time.perf_counter()
            for j, w in enumerate(ws):
                ql.linear(xs[j], w, None, backend="torch", quant_mode="ck", input_act="swiglu" if j == 3 else None)
            if i >= args.warmup:
                times.append(time.perf_counter() - t0)
        t_ms = statistics.median(times) * 1e3
        v = rows / (t_ms * 1e-3) / nb
        kind, sample = "reference", (f"the block's four W4A8 linears (qkv, out, fc1, fc2 with SwiGLU input) through the "
                                     f"reference's own CPU qlinear on {rows} tokens, timed as executed ({cores} threads); "
                                     f"tokens/s of {nb} block(s); attention, norms and RoPE excluded (an upper bound)")
    cfg = dict(cfg, parallelism=f"{args.gpus} GPU(s) requested; the CPU arm runs on rank 0's host cores")
    line = {"metric": metric, "value": v, "unit": "tokens/s", "n_gpus": args.gpus, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": t_ms, "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "int8", "data": "synthetic", "impl": "reference", "config": cfg,
            "cpu_baseline": {"value": v, "unit": "tokens/s", "cores": cores, "kind": kind, "sample": sample},
            "e2e": {"value": v, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def config_dict(ms, world):
    return {"workload": "config2 qlinear sweep per GPU: (K,N) in " + str(SWEEP) + f" x M in {ms}",
            "model": "H3 DiT W4A8 ConvRot qlinear (width 5120, FFN 13824)", "weights": "int4 group-128, fp16 scales",
            "activations": "bf16 N(0,1), 0.5% outlier channels x20", "global_tokens_per_point": [m * world for m in ms],
            "parallelism": f"token-shard x{world}", "l2": "inputs larger than L2 (each step streams ~8 GB)"}


def dit_shape(workload):
    """(tokens, blocks, video tokens, metric, config) of a DiT workload."""
    if workload == "stream":
        t, nb, vid = STREAM_TOKENS, STREAM_BLOCKS, STREAM_TOKENS
        cfg = {"workload": f"config4 weight streaming: {nb} W4A8 DiT blocks (width {HID}, {HEADS}x{HEAD_DIM} heads, "
                           f"FFN {FFN} SwiGLU) held in a pinned host h3t store, {STREAM_RESIDENT} resident + a "
                           f"{STREAM_RING}-slot ring on the GPU, prefetch {STREAM_PREFETCH}; M={t} tokens",
               "model": "H3 DiT block stack, W4A8 int4 group-128 fp16 scales", "tokens": t, "blocks": nb}
        return t, nb, vid, "DiT 48-block stack tokens/s, weights streamed from pinned host", cfg
    f, h, w, audio, nb = SEQS[workload]
    vid = f * h * w
    t = vid + audio
    name = "config3 one DiT block" if workload == "block" else "config5 long sequence, 4 DiT blocks"
    cfg = {"workload": f"{name}: M={t} tokens ({f}x{h}x{w} video + {audio} audio), width {HID}, {HEADS}x{HEAD_DIM} heads, "
                       f"FFN {FFN} SwiGLU, W4A8 linears, bf16 attention/norms, AdaLN modulation precomputed",
           "model": "H3 DiT block, W4A8 int4 group-128 fp16 scales", "tokens": t, "blocks": nb}
    return t, nb, vid, f"DiT block tokens/s ({name})", cfg


# ------------------------------------------------------------------------------------------------ DiT workloads (GPU)
def synthetic_block(seed, dev):
    """Random W4A8 block at DiT width (int4 group-128 from N(0, 0.02), fp16 scales) with bf16 norm weights."""
    import torch
    from minimax_h3_turbo_b200.h3.synth import synthetic_w4a8
    from minimax_h3_turbo_b200.h3.types import BlockWeights

    g = torch.Generator(device=dev).manual_seed(seed)
    norm = lambda n: (1.0 + 0.1 * torch.randn(n, generator=g, device=dev)).to(torch.bfloat16)  # noqa: E731
    lin = [synthetic_w4a8(n, k, seed=seed * 10 + j, device=dev) for j, (k, n) in enumerate(BLOCK_LINEARS)]
    return BlockWeights(qkv=lin[0], out=lin[1], fc1=lin[2], fc2=lin[3], norm1=norm(HID), norm2=norm(HID),
                        q_norm=norm(HEAD_DIM), k_norm=norm(HEAD_DIM))


def synthetic_modulation(seed, dev):
    """Precomputed AdaLN outputs: six [2, HID] bf16 N(0, 1) rows (row 0: video tokens, row 1: audio tokens)."""
    import torch
    from minimax_h3_turbo_b200.h3 import block as blk

    g = torch.Generator(device=dev).manual_seed(seed)
    return blk.Modulation(*(torch.randn(2, HID, generator=g, device=dev).to(torch.bfloat16) for _ in range(6)))


def dit_sequence(frames, hh, ww, audio, start, stop, dev):
    """RoPE tables and modulation segments of rows [start, stop) of a video + audio token sequence."""
    import torch
    from minimax_h3_turbo_b200.h3 import block as blk

    pos = blk.video_audio_positions(frames, hh, ww, audio, dev)[start:stop]
    inv_freq = 1.0 / (10000.0 ** (torch.arange(16, device=dev, dtype=torch.float32) / 16))
    cos, sin = blk.rope_tables(pos, inv_freq, torch.bfloat16)
    vid = frames * hh * ww
    segs = []
    for a, b, row in ((0, vid, 0), (vid, vid + audio, 1)):
        a, b = max(a, start), min(b, stop)
        if b > a:
            segs.append((a - start, b - start, row))
    return cos, sin, segs


class TimedLinear:
    """The W4A8 qlinear with CUDA events around each call on the launching stream (when `on`)."""

    def __init__(self):
        from minimax_h3_turbo_b200.h3 import qlinear as ql

        self.ql, self.on, self.events, self.calls = ql, False, [], 0

    def _run(self, x, w, input_act):
        from minimax_h3_turbo_b200.h3 import block as blk

        if isinstance(x, blk.Prenorm):  # qkv / fc1: RMSNorm + modulation fused into the quantiser
            return blk.prenorm_linear(x, w)
        return self.ql.linear(x, w, input_act=input_act)

    def __call__(self, x, w, input_act=None):
        import torch

        if not self.on:
            return self._run(x, w, input_act)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        y = self._run(x, w, input_act)
        e1.record()
        self.events.append((e0, e1))
        self.calls += 1
        return y

    def ms(self):
        return sum(a.elapsed_time(b) for a, b in self.events)


def dit_common_fields(pk, lin_ops, lin_ms, attn_flops, total_ms, steps):
    """Roofline of the qlinear share and of the block as a whole (per rank, per step)."""
    int8_peak, bf16_peak = 2.0 * pk["bf16"], pk["bf16"]
    lin_tops = lin_ops / (lin_ms / steps * 1e-3) / 1e12 if lin_ms > 0 else None
    bound_ms = (lin_ops / (int8_peak * 1e12) + attn_flops / (bf16_peak * 1e12)) * 1e3
    rest_ms = (total_ms - lin_ms) / steps
    return {"roofline": {"bound": "tensor", "kernel": "W4A8 qlinear (rotq + decode + gemm_i8 per call)", "achieved": lin_tops,
                         "peak": int8_peak, "unit": "TOPS", "frac": lin_tops / int8_peak if lin_tops else None, "traffic": None,
                         "peak_note": f"int8 dense = 2 x {pk['source']} bf16 dense ({pk['bf16']} TFLOP/s burst)"},
            "block_roofline": {"bound_ms": bound_ms, "measured_ms": total_ms / steps, "frac": bound_ms / (total_ms / steps),
                               "basis": "linear ops / int8 peak + attention flops / bf16 peak, per rank per step"},
            "split_ms_per_step": {"qlinear": lin_ms / steps, "attention_norms_rope_gathers": rest_ms,
                                  "attention_tflops_if_all_rest": attn_flops / (rest_ms * 1e-3) / 1e12 if rest_ms > 0 else None}}


class PhaseProbe:
    """CUDA events at the attention's phase boundaries (DiTBlock's probe): per block call, the exposed key/value
    exchange time (kv_ready after qk_ready, or after local_done when the local attention overlaps the exchange) and
    the attention time (the rest of qk_ready -> attn_done)."""

    def __init__(self):
        self.on, self.calls, self.cur = False, [], None

    def __call__(self, tag):
        import torch

        if not self.on:
            return
        if tag == "qk_ready":
            self.cur = {}
            self.calls.append(self.cur)
        ev = torch.cuda.Event(enable_timing=True)
        ev.record()
        self.cur[tag] = ev

    def totals_ms(self):
        exch = attn = 0.0
        for c in self.calls:
            if "kv_ready" not in c:
                attn += c["qk_ready"].elapsed_time(c["attn_done"])
                continue
            start = c.get("local_done", c["qk_ready"])
            exch += start.elapsed_time(c["kv_ready"])
            attn += c["kv_ready"].elapsed_time(c["attn_done"])
            if "local_done" in c:
                attn += c["qk_ready"].elapsed_time(c["local_done"])
        return exch, attn


def dit_measure(workload, steps, warmup, rank, world, local, group, kv_exchange="gather", kv_groups=1, e2e=True,
                check_rows=0):
    """Configs 3 and 5 on the kernels: DiT blocks on a video + audio sequence, token-sharded over `world` ranks (keys
    and values exchanged per block, the final hidden states all-gathered at the sequence boundary).  Times `steps`
    forwards (after `warmup`) with CUDA events, max over ranks; per phase: the W4A8 linears, the exposed key/value
    exchange, attention.  check_rows > 0 (several ranks): rank 0 recomputes the whole sequence alone and compares that
    many rows, spread over every shard, of the gathered output.  Returns the record (on every rank)."""
    import torch
    import torch.distributed as dist

    load_package()
    from minimax_h3_turbo_b200.h3 import block as blk

    dev = torch.device("cuda", local)
    frames, hh, ww, audio, nb = SEQS[workload]
    tokens, _, _, metric, cfg = dit_shape(workload)
    a, b = blk.shard_rows(tokens, world, rank)
    spec = blk.ShardSpec(a, b, tokens, group=group if world > 1 else None, world=world, rank=rank)
    cos, sin, segs = dit_sequence(frames, hh, ww, audio, a, b, dev)
    weights = [synthetic_block(100 + i, dev) for i in range(nb)]  # the same seeds on every rank: replicated weights
    mods = [synthetic_modulation(200 + i, dev) for i in range(nb)]
    gx = torch.Generator(device=dev).manual_seed(7)
    x_all = torch.randn(tokens, HID, generator=gx, device=dev).to(torch.bfloat16)
    x0 = x_all[a:b].contiguous()
    if not check_rows or world == 1 or rank != 0:
        del x_all
    x = torch.empty_like(x0)
    lin, probe = TimedLinear(), PhaseProbe()
    block = blk.DiTBlock(HEADS, HEAD_DIM, linear=lin, kv_exchange=kv_exchange, fuse_norm=True, kv_groups=kv_groups,
                         probe=probe)
    stream = torch.cuda.current_stream(dev)

    def forward(xin):
        x.copy_(xin)
        y = x
        for i in range(nb):
            y = block(y, weights[i], mods[i], segs, cos, sin, spec)
        return blk.gather_rows(y, spec)

    def barrier():
        if world > 1:
            dist.barrier(group=group)
        torch.cuda.synchronize(dev)

    def max_over_ranks(v):
        t = torch.tensor([v], device=dev, dtype=torch.float64)
        if world > 1:
            dist.all_reduce(t, op=dist.ReduceOp.MAX, group=group)
        return float(t.item())

    for _ in range(warmup):
        forward(x0)
    barrier()
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    clocks = ClockSampler(local)
    clocks.start()
    barrier()
    clocks.begin()
    lin.on = probe.on = True
    t0.record(stream)
    for _ in range(steps):
        out = forward(x0)
    t1.record(stream)
    barrier()
    clocks.end()
    lin.on = probe.on = False
    clk = clocks.stop()
    t_ms = max_over_ranks(t0.elapsed_time(t1))
    lin_ms = max_over_ranks(lin.ms()) / steps
    exch_ms, attn_ms = probe.totals_ms()
    exch_ms, attn_ms = max_over_ranks(exch_ms) / steps, max_over_ranks(attn_ms) / steps
    finite = bool(torch.isfinite(out.float()).all().item()) and tuple(out.shape) == (tokens, HID)
    rows = b - a
    kv_bytes = 2 * (tokens - rows) * HEADS * HEAD_DIM * 2  # keys + values this rank receives per block
    rec = {"workload": cfg["workload"], "tokens": tokens, "blocks": nb, "n_gpus": world,
           "tokens_per_s": tokens * steps / (t_ms * 1e-3), "ms_per_forward": t_ms / steps, "steps": steps,
           "warmup": warmup, "qlinear_ms_per_forward": lin_ms, "attention_ms_per_forward": attn_ms,
           "kv_exchange": kv_exchange if world > 1 else "none (one GPU)",
           "kv_exchange_exposed_ms_per_forward": exch_ms,
           "kv_bytes_in_per_rank_per_block": kv_bytes,
           "kv_exchange_gbs_per_rank": (kv_bytes * nb / (exch_ms * 1e-3) / 1e9) if exch_ms > 0 else None,
           "rest_ms_per_forward": t_ms / steps - lin_ms - attn_ms - exch_ms,
           "rows_per_rank": [e - s for s, e in (blk.shard_rows(tokens, world, r) for r in range(world))],
           "backend": dist.get_backend(group) if world > 1 else None, "nccl_ranks": world if world > 1 else 0,
           "output_finite": finite, "clocks": clk,
           "linear_tops_per_rank": nb * rows * BLOCK_OPS_PER_TOKEN / (lin_ms * 1e-3) / 1e12 if lin_ms > 0 else None,
           "attention_tflops_per_rank": nb * 4.0 * rows * tokens * HEADS * HEAD_DIM / (attn_ms * 1e-3) / 1e12
           if attn_ms > 0 else None}
    if world > 1:  # the link this exchange runs on: one all-gather of a K/V-sized shard, alone, best of 5
        shard = torch.empty(rows, 2 * HEADS * HEAD_DIM, dtype=torch.bfloat16, device=dev)
        full = torch.empty(world * rows, 2 * HEADS * HEAD_DIM, dtype=torch.bfloat16, device=dev)
        best = float("inf")
        for _ in range(6):
            barrier()
            g0, g1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            g0.record(stream)
            dist.all_gather_into_tensor(full, shard, group=group)
            g1.record(stream)
            barrier()
            best = min(best, max_over_ranks(g0.elapsed_time(g1)))
        rec["allgather_probe"] = {"bytes_in_per_rank": kv_bytes, "ms": best,
                                  "gbs_in_per_rank": kv_bytes / (best * 1e-3) / 1e9,
                                  "what": "one NCCL all_gather_into_tensor of this rank's keys+values shard, alone"}
        del shard, full
    if check_rows and world > 1:
        idx = torch.linspace(0, tokens - 1, check_rows, device=dev).round().long()
        got = out[idx].float()
        if rank == 0:  # the same sequence on this GPU alone
            ref_block = blk.DiTBlock(HEADS, HEAD_DIM, fuse_norm=True)
            cos1, sin1, segs1 = dit_sequence(frames, hh, ww, audio, 0, tokens, dev)
            y = x_all.clone()
            for i in range(nb):
                y = ref_block(y, weights[i], mods[i], segs1, cos1, sin1)
            want, x_in = y[idx].float(), x_all[idx].float()
            rec["check"] = {"rows": check_rows, "max_rel": float((got - want).abs().max() / want.abs().max()),
                            "rel_l2_of_update": float((got - want).norm() / (want - x_in).norm()),
                            "bit_identical": bool(torch.equal(got, want)),
                            "vs": "the same rows of the whole sequence recomputed on rank 0 alone (one GPU, no exchange)"}
            del y, x_all
        barrier()
    if e2e:
        hin = torch.empty(rows, HID, dtype=torch.bfloat16, pin_memory=True)
        hin.copy_(x0)
        hout = torch.empty(tokens, HID, dtype=torch.bfloat16, pin_memory=True)
        e_steps = max(1, min(steps, 2))
        barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(e_steps):
            y = forward(hin.to(dev, non_blocking=True))
            if rank == 0:
                hout.copy_(y, non_blocking=True)
        e1.record(stream)
        barrier()
        te = max_over_ranks(e0.elapsed_time(e1))
        rec["e2e"] = {"value": tokens * e_steps / (te * 1e-3), "unit": "tokens/s", "h2d_bytes_per_step": tokens * HID * 2,
                      "d2h_bytes_per_step": tokens * HID * 2, "steps": e_steps,
                      "path": "DiTBlock over qlinear.linear; each rank copies its input rows in from pinned host memory, "
                              "rank 0 copies the gathered [tokens, 5120] output out"}
    rec["_lin_calls"] = lin.calls
    rec["_metric"], rec["_cfg"] = metric, cfg
    del weights, out, x, x0
    torch.cuda.empty_cache()
    return rec


def run_dit(args, rank, world, local):
    """Configs 3 and 5 as their own bench line (`--workload block|longseq`)."""
    import torch
    import torch.distributed as dist
    from datetime import timedelta

    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=dev)
    group = dist.group.WORLD if world > 1 else None
    rec = dit_measure(args.workload, args.steps, args.warmup, rank, world, local, group, args.kv_exchange,
                      args.kv_groups, e2e=not args.no_e2e, check_rows=256 if world > 1 else 0)
    tokens, nb = rec["tokens"], rec["blocks"]
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu:
        cores = os.cpu_count() or 1
        v, detail = cpu_block_rate(tokens, nb, args.cpu_rows)
        cpu = {"value": v, "unit": "tokens/s", "cores": cores, "kind": "port",
               "sample": f"the four W4A8 linears only (attention, norms, RoPE excluded: an upper bound), {args.cpu_rows} "
                         f"tokens and {CPU_WEIGHT_ROWS} output channels per projection, scaled per channel, per-token "
                         f"extrapolation ({cores} threads)", "detail": detail}
    rows = tokens // world
    lin_ops = nb * rows * BLOCK_OPS_PER_TOKEN
    attn_flops = nb * 4.0 * rows * tokens * HEADS * HEAD_DIM
    fields = dit_common_fields(peaks(), lin_ops, rec["qlinear_ms_per_forward"] * args.steps, attn_flops,
                               rec["ms_per_forward"] * args.steps, args.steps)
    if rank == 0:
        cfg = dict(rec["_cfg"], parallelism=f"token-shard x{world} (contiguous rows, K/V exchange: {rec['kv_exchange']}, "
                                            f"output all-gather)", rows_per_rank=rec["rows_per_rank"],
                   l2="inputs larger than L2 (each block streams ~0.6 GB of weights+activations per rank)")
        detail = {k: v for k, v in rec.items() if not k.startswith("_") and k not in ("e2e", "clocks")}
        line = {"metric": rec["_metric"], "value": rec["tokens_per_s"], "unit": "tokens/s", "n_gpus": world,
                "steps": args.steps, "warmup": args.warmup, "ms_per_step": rec["ms_per_forward"],
                "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "int8", "data": "synthetic",
                "config": cfg, **fields, "phases": detail, "cpu_baseline": cpu, "e2e": rec.get("e2e"),
                "clocks": rec["clocks"],
                # per block: 4 W4A8 linears (rotate+quantise -- with the RMSNorm+modulation for qkv and fc1 --, decode,
                # GEMM each), 1 q/k norm+RoPE, 2 gated residuals, with the overlapped or ring exchange the merges
                "gpu_launches": 3 * rec["_lin_calls"] + 3 * nb * args.steps +
                (2 * nb * args.steps if world > 1 and args.kv_exchange == "overlap" else 0) +
                (world * nb * args.steps if world > 1 and args.kv_exchange == "ring" else 0)}
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def pick_store_dir(need_bytes, want=None):
    import shutil
    import tempfile

    cands = [want] if want else [tempfile.gettempdir(), "/dev/shm", str(ROOT)]
    for d in cands:
        try:
            if d and os.path.isdir(d) and shutil.disk_usage(d).free > 1.1 * need_bytes:
                return Path(d)
        except OSError:
            continue
    raise SystemExit(f"bench.py: no directory among {cands} has {need_bytes / 1e9:.1f} GB free for the h3t store")


def run_stream(args, rank, world, local):
    """Config 4: a 48-block stack from a pinned host h3t store through the StreamingProvider (4 resident blocks + a
    3-slot ring), against the same stack fully resident, a copy-only pass, and a pinned host->device copy peak."""
    if world > 1:
        raise SystemExit("bench.py: the stream workload runs on one GPU (each rank would need its own host store)")
    import torch

    load_package()
    from minimax_h3_turbo_b200.h3 import block as blk
    from minimax_h3_turbo_b200.h3 import stream as sm
    from minimax_h3_turbo_b200.h3.config import H3Config
    from minimax_h3_turbo_b200.h3.store import H3TFile
    from minimax_h3_turbo_b200.h3.synth import synthetic_store_tensors
    from minimax_h3_turbo_b200.h3.writer import write_h3t

    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    stream = torch.cuda.current_stream(dev)
    tokens, nb, _, metric, cfgd = dit_shape("stream")
    hcfg = H3Config(hidden=HID, layers=nb, refiner_layers=0, heads=HEADS, head_dim=HEAD_DIM, ffn=FFN, quant_group=128)
    est = nb * 164e6
    path = pick_store_dir(est, args.store_dir) / f"h3b_bench_stack_{os.getpid()}.h3t"
    tw = time.perf_counter()
    write_h3t(path, hcfg, synthetic_store_tensors(hcfg, group=128, scale_dtype="fp16", seed=11, with_globals=False, device=dev),
              quant={"format": "asym_w4a8_int8", "group_size": 128, "convrot_groupsize": 256})
    write_s = time.perf_counter() - tw
    store = H3TFile(path)
    try:
        mod = synthetic_modulation(300, dev)
        f, h, w = 16, 16, 16  # 4096 video tokens
        cos, sin, segs = dit_sequence(f, h, w, 0, 0, tokens, dev)
        x0 = torch.randn(tokens, HID, generator=torch.Generator(device=dev).manual_seed(5), device=dev).to(torch.bfloat16)
        x = torch.empty_like(x0)
        block = blk.DiTBlock(HEADS, HEAD_DIM)

        def forward(p, compute=True):
            x.copy_(x0)
            y = x
            p.begin_forward()
            for i in range(nb):
                wi = p.acquire(i)
                if compute:
                    y = block(y, wi, mod, segs, cos, sin)
                p.release(i)
            p.end_forward()
            return y

        def timed(p, compute=True, clocks=None):
            for _ in range(args.warmup):
                forward(p, compute)
            torch.cuda.synchronize(dev)
            s0 = p.stats()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            if clocks:
                clocks.start()
                clocks.begin()
            e0.record(stream)
            for _ in range(args.steps):
                y = forward(p, compute)
            e1.record(stream)
            torch.cuda.synchronize(dev)
            if clocks:
                clocks.end()
            clk = clocks.stop() if clocks else None
            s1 = p.stats()
            d = {k: s1[k] - s0[k] for k in ("acquires", "waits", "wait_s", "copies", "bytes")}
            return e0.elapsed_time(e1) / args.steps, d, y, clk

        # pinned host -> device link peak: one cudaMemcpyAsync of 1 GiB from pinned memory, best of 5
        hb = torch.empty(1 << 30, dtype=torch.uint8, pin_memory=True)
        db = torch.empty_like(hb, device=dev)
        best = float("inf")
        for _ in range(6):
            c0, c1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            c0.record(stream)
            db.copy_(hb, non_blocking=True)
            c1.record(stream)
            torch.cuda.synchronize(dev)
            best = min(best, c0.elapsed_time(c1))
        link_gbs = hb.numel() / (best * 1e-3) / 1e9
        del hb, db

        clocks = ClockSampler(local)
        with sm.StreamingProvider(store, dev, resident=STREAM_RESIDENT, ring=STREAM_RING, prefetch=STREAM_PREFETCH,
                                  pin=True) as p:
            t_stream, d_stream, y_stream, clk = timed(p, True, clocks)
            t_copy, d_copy, _, _ = timed(p, False)
            kinds = sorted(set(p.stats()["host_kinds"]))
            # e2e through the public API: activations in from pinned host memory, the result back out
            hin = torch.empty(tokens, HID, dtype=torch.bfloat16, pin_memory=True)
            hin.copy_(x0)
            hout = torch.empty_like(hin)
            torch.cuda.synchronize(dev)
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e_steps = max(1, min(args.steps, 2))
            e0.record(stream)
            for _ in range(e_steps):
                x0.copy_(hin, non_blocking=True)
                hout.copy_(forward(p, True), non_blocking=True)
            e1.record(stream)
            torch.cuda.synchronize(dev)
            t_e2e = e0.elapsed_time(e1) / e_steps
        with sm.StreamingProvider(store, dev, resident=nb, ring=1, prefetch=0, pin=False) as p:
            t_res, _, y_res, _ = timed(p, True)
        same = bool(torch.equal(y_stream, y_res))
        nbytes = store.block_nbytes
    finally:
        store.close()
        path.unlink(missing_ok=True)

    h2d_gbs = d_stream["bytes"] / args.steps / (t_stream * 1e-3) / 1e9
    copy_gbs = d_copy["bytes"] / args.steps / (t_copy * 1e-3) / 1e9
    pk = peaks()
    lin_ops = nb * tokens * BLOCK_OPS_PER_TOKEN
    cpu = None
    if not args.no_cpu:
        cores = os.cpu_count() or 1
        v, detail = cpu_block_rate(tokens, nb, args.cpu_rows)
        cpu = {"value": v, "unit": "tokens/s", "cores": cores, "kind": "port",
               "sample": f"the four W4A8 linears only (attention, norms excluded: an upper bound), {args.cpu_rows} rows per "
                         f"projection and {CPU_WEIGHT_ROWS} output channels, scaled per channel, per-token extrapolation to {nb} blocks ({cores} threads)",
               "detail": detail}
    cfgd = dict(cfgd, block_nbytes=nbytes, store_bytes=nb * nbytes, host_kinds=kinds, store_write_s=round(write_s, 1),
                parallelism="one GPU")
    line = {"metric": metric, "value": tokens / (t_stream * 1e-3), "unit": "tokens/s", "n_gpus": 1, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": t_stream, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "int8", "data": "synthetic", "config": cfgd,
            "roofline": {"bound": "h2d", "kernel": "host->device block copies (copy engine)", "achieved": h2d_gbs,
                         "peak": link_gbs, "unit": "GB/s", "frac": h2d_gbs / link_gbs, "traffic": None,
                         "peak_note": "pinned 1 GiB cudaMemcpyAsync measured in this run"},
            "streaming": {"ms_per_forward_streamed": t_stream, "ms_per_forward_resident": t_res,
                          "ms_per_forward_copy_only": t_copy, "streamed_vs_resident": t_res / t_stream,
                          "hidden_copy_frac": 1.0 - (t_stream - t_res) / t_copy, "h2d_gbs_streamed": h2d_gbs,
                          "h2d_gbs_copy_only": copy_gbs, "link_peak_gbs": link_gbs,
                          "bytes_per_forward": d_stream["bytes"] / args.steps, "waits_per_forward": d_stream["waits"] / args.steps,
                          "wait_s_per_forward": d_stream["wait_s"] / args.steps, "streamed_equals_resident": same,
                          "linear_tops_resident": lin_ops / (t_res * 1e-3) / 1e12, "int8_peak": 2.0 * pk["bf16"]},
            "cpu_baseline": cpu,
            "e2e": {"value": tokens / (t_e2e * 1e-3), "unit": "tokens/s", "h2d_bytes_per_step": tokens * HID * 2,
                    "d2h_bytes_per_step": tokens * HID * 2, "steps": e_steps,
                    "path": "activations in from pinned host memory, 48 streamed blocks, result out to pinned host memory"},
            "clocks": clk, "gpu_launches": 12 * nb * args.steps}
    print(json.dumps(line), flush=True)


# ------------------------------------------------------------------------------------------------ GPU leg: the sweep
def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="h3b", choices=["h3b", "reference"])
    ap.add_argument("--ms", default=",".join(map(str, MS)))
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--cpu-rows", type=int, default=256)
    ap.add_argument("--ref-rows", type=int, default=2048, help="reference arm: tokens per projection in each step's sample")
    ap.add_argument("--no-ref-cuda", action="store_true", help="reference arm: skip timing the reference's CUDA path")
    ap.add_argument("--detail", default="", help="write per-point timings to this JSON file")
    ap.add_argument("--workload", default="sweep", choices=WORKLOADS,
                    help="sweep: config 2 (default); block: config 3; stream: config 4; longseq: config 5")
    ap.add_argument("--store-dir", default="", help="stream workload: directory for the temporary ~7.9 GB h3t store")
    ap.add_argument("--kv-groups", type=int, default=1, help="block/longseq over several GPUs: head groups of the K/V all-gather")
    ap.add_argument("--kv-exchange", default="gather", choices=["gather", "overlap", "ring"],
                    help="DiT blocks on several GPUs: keys/values exchanged point-to-point behind the local attention "
                         "(overlap), all-gathered first (gather), or passed round a ring")
    ap.add_argument("--no-official", action="store_true", help="sweep line: skip the official-geometry record")
    ap.add_argument("--dit-steps", type=int, default=5, help="sweep line: timed forwards of the config-5 record (config 3: twice as many)")
    ap.add_argument("--e2e-rows", type=int, default=E2E_ROWS, help="sweep line: tokens per chunk of the end-to-end pipeline")
    ap.add_argument("--no-dit", action="store_true", help="sweep line: skip the config-5 (and, on one GPU, config-3) records")
    args = ap.parse_args()
    args.ms = [int(v) for v in args.ms.split(",") if v]
    rank, world, local = int(os.environ.get("RANK", 0)), int(os.environ.get("WORLD_SIZE", 1)), int(os.environ.get("LOCAL_RANK", 0))
    if args.warmup < 3:
        print("bench.py: --warmup must be >= 3", file=sys.stderr)
        sys.exit(2)
    if args.impl == "reference":
        run_reference(args, rank)
        return
    if args.workload in ("block", "longseq"):
        run_dit(args, rank, world, local)
        return
    if args.workload == "stream":
        run_stream(args, rank, world, local)
        return
    run_sweep(args, rank, world, local)


OFFICIAL = {"qkv": (5376, 21504, False), "out": (7168, 5376, False), "fc1": (5376, 28672, False),
            "fc2": (14336, 5376, True)}  # (K, N, SwiGLU input): hidden 5376, 56 x 128 heads, FFN 14336


def official_points(dev, ms=(256, 4096), reps=10):
    """The four projections of the official H3 DiT (h3turbo/h3/config.py:12-31) in the real checkpoint format, one W4A8
    linear each through qlinear.linear (device-resident bf16 activations), at M = 256 and 4096: CUDA-event time of
    `reps` calls after 3 warm-up calls.  Context beside the headline sweep, not part of `value`."""
    import torch
    from minimax_h3_turbo_b200.h3 import qlinear as ql
    from minimax_h3_turbo_b200.h3.synth import synthetic_activation, synthetic_w4a8_fp8

    out = []
    for name, (k, n, sw) in OFFICIAL.items():
        w = synthetic_w4a8_fp8(n, k, seed=k + n, device=dev)
        for m in ms:
            x = synthetic_activation(m, 2 * k if sw else k, seed=m + k, device=dev)
            act = "swiglu" if sw else None
            for _ in range(3):
                ql.linear(x, w, input_act=act)
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            for _ in range(reps):
                ql.linear(x, w, input_act=act)
            e1.record()
            torch.cuda.synchronize(dev)
            us = e0.elapsed_time(e1) / reps * 1e3
            out.append({"proj": name, "K": k, "N": n, "M": m, "swiglu_input": sw, "us": round(us, 1),
                        "tops": 2.0 * m * n * k / (us * 1e-6) / 1e12})
        del w
    return {"format": "fp8 e4m3 group-16 scales, 16-level codebook", "points": out}


def measure_int8_peak(dev, n=8192, reps=10):
    """Dense int8 tensor-core throughput of the library GEMM on this GPU: torch._int_mm (cuBLASLt) on n^3, best of
    `reps` launches timed with CUDA events."""
    import torch

    try:
        g = torch.Generator(device=dev).manual_seed(0)
        a = torch.randint(-128, 128, (n, n), generator=g, device=dev, dtype=torch.int32).to(torch.int8)
        b = torch.randint(-128, 128, (n, n), generator=g, device=dev, dtype=torch.int32).to(torch.int8)
        bt = b.t()  # column-major operand, the layout cuBLASLt's int8 kernels take
        for _ in range(3):
            torch._int_mm(a, bt)
        best = float("inf")
        for _ in range(reps):
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            torch._int_mm(a, bt)
            e1.record()
            torch.cuda.synchronize(dev)
            best = min(best, e0.elapsed_time(e1))
        del a, b, bt
        return {"tops": 2.0 * n ** 3 / (best * 1e-3) / 1e12, "how": f"torch._int_mm (cuBLASLt) {n}^3 int8 -> int32, best of {reps}"}
    except Exception as e:  # a library limitation must not cost the main measurement
        return {"tops": None, "error": repr(e)[:200]}


def run_sweep(args, rank, world, local):
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

    # small M: the W4A8 GEMM decodes the int4 weight in its producer warps (no decode pass); large M: decode pass, then
    # the int8 GEMM -- exactly what h3b_w4a8_gemm (and qlinear.linear) do for each point
    fused = {(k, n, m): bool(L.h3b_w4a8_gemm_decodes_in_kernel(m, n, k, weights[(k, n)][1].q.data_ptr(),
                                                                weights[(k, n)][1].ldq, weights[(k, n)][1].s_dtype, 128))
             for (k, n, m) in points}

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
            o = outs[(k, n, m)]
            if fused[(k, n, m)]:
                if evs is not None:
                    evs[i][2].record(stream)
                _lib.check(L.h3b_w4a8_gemm(codes.data_ptr(), k, xs.data_ptr(), m, a.q.data_ptr(), a.ldq, a.s.data_ptr(),
                                           a.s_dtype, a.lds, a.s_ch.data_ptr(), a.cb.data_ptr(), 128, None, o.data_ptr(),
                                           _lib.BF16, n, n, k, 0, g.data_ptr(), g.numel(), sp), "w4a8 gemm")
            else:
                _lib.check(L.h3b_decode_grid(a.q.data_ptr(), n, k, a.ldq, a.s.data_ptr(), a.s_dtype, a.lds, a.cb.data_ptr(),
                                             128, g.data_ptr(), k, sp), "decode")
                if evs is not None:
                    evs[i][2].record(stream)
                _lib.check(L.h3b_int8_gemm_epilogue(codes.data_ptr(), k, xs.data_ptr(), m, g.data_ptr(), k, a.s_ch.data_ptr(),
                                                    None, o.data_ptr(), _lib.BF16, n, n, k, 0, sp), "gemm")
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
    clocks.begin()
    t0.record(stream)
    for s in range(args.steps):
        step(evs[s])
    t1.record(stream)
    barrier()
    clocks.end()
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
        per_point.append({"K": k, "N": n, "M": m, "decode_in_gemm": fused[(k, n, m)], "rotq_ms": r, "decode_ms": d, "gemm_ms": g,
                          "gemm_tops": 2.0 * m * n * k / (g * 1e-3) / 1e12, "linear_tops": 2.0 * m * n * k / ((r + d + g) * 1e-3) / 1e12,
                          "rotq_gbs": (3.0 * m * k + 4 * m) / (r * 1e-3) / 1e9})
    ops_step = ops_of(points)
    value = world * ops_step * args.steps / (t_max_ms * 1e-3) / 1e12
    pk = peaks()
    int8_peak = 2.0 * pk["bf16"]
    gemm_tops = ops_step / (tot["gemm"] * 1e-3) / 1e12
    rotq_bytes = sum(3.0 * m * k + 4.0 * m for (k, _, m) in points)
    rotq_gbs = rotq_bytes / (tot["rotq"] * 1e-3) / 1e9
    # DRAM bytes (read + write) of the GEMM launch of each point, measured with ncu on a B200 (dram__bytes_read.sum +
    # dram__bytes_write.sum of that kernel, this sweep's command): the average launch of the sweep, or None when a
    # point of this run was not measured
    traffic = (sum(GEMM_DRAM_BYTES[p] for p in points) / len(points)) if all(p in GEMM_DRAM_BYTES for p in points) else None

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

        # pipelined like a serving loop: host->device copies on one copy stream, device->host on another, compute on
        # the current stream.  Each point goes through in chunks of at most E2E_ROWS tokens (the linear is token-wise,
        # so a chunk is an exact sub-problem) over three device input slots, so the upload of chunk j + 1 and the
        # download of chunk j - 1 run while chunk j computes: the host link, not the order of the copies, bounds it
        kmax = max(k for (k, _, _) in points)
        rows = args.e2e_rows
        chunks = [(i, k, n, r0, min(m, r0 + rows)) for i, (k, n, m) in enumerate(points) for r0 in range(0, m, rows)]
        s_in, s_out = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
        nslot = 3
        dbuf = [torch.empty(min(big_in, rows * kmax), dtype=torch.bfloat16, device=dev) for _ in range(nslot)]
        slot_free = [None] * nslot  # compute-done event of the chunk that last read each slot

        def e2e_step():
            for j, (i, k, n, r0, r1) in enumerate(chunks):
                w, _ = weights[(k, n)]
                slot = j % nslot
                rows = r1 - r0
                xd = dbuf[slot][: rows * k].view(rows, k)
                if slot_free[slot] is None:
                    s_in.wait_stream(stream)
                else:
                    s_in.wait_event(slot_free[slot])
                with torch.cuda.stream(s_in):
                    xd.copy_(hin[r0 * k: r1 * k].view(rows, k), non_blocking=True)
                    ready = torch.cuda.Event()
                    ready.record(s_in)
                stream.wait_event(ready)
                y = ql.linear(xd, w)
                done = torch.cuda.Event()
                done.record(stream)
                slot_free[slot] = done
                s_out.wait_event(done)
                with torch.cuda.stream(s_out):
                    hout[r0 * n: r1 * n].view(rows, n).copy_(y, non_blocking=True)
                y.record_stream(s_out)
            stream.wait_stream(s_out)  # the step ends when its last result is in host memory

        e2e_step()
        barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e2e_steps = max(1, min(args.steps, 3))
        barrier()
        e0.record(stream)
        s_in.wait_stream(stream)
        for _ in range(e2e_steps):
            e2e_step()
        e1.record(stream)
        barrier()
        te = torch.tensor([e0.elapsed_time(e1)], device=dev, dtype=torch.float64)
        if world > 1:
            dist.all_reduce(te, op=dist.ReduceOp.MAX)
        e2e = {"value": world * ops_step * e2e_steps / (float(te.item()) * 1e-3) / 1e12, "unit": "TOPS",
               "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h, "steps": e2e_steps,
               "path": "qlinear.linear (public API) per point; pinned host input/output; uploads, compute and downloads "
                       "pipelined on three streams (two device input slots)"}

    # ---- CPU baseline (rank 0, single GPU only)
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu:
        cores = os.cpu_count() or 1
        v, detail = cpu_reference_rate(args.ms, args.cpu_rows)
        cpu = {"value": v, "unit": "TOPS", "cores": cores, "kind": "port",
               "sample": f"{args.cpu_rows} tokens and {CPU_WEIGHT_ROWS} output channels per projection (decode, quantise, "
                         f"int8 GEMM, epilogue), scaled per output channel and extrapolated per token to the sweep "
                         f"(numpy oracle of the reference CPU path, {cores} threads)",
               "detail": detail}

    # ---- a measured int8 denominator beside 2 x bf16: cuBLASLt's int8 GEMM (torch._int_mm) at 8192^3, best of 10
    int8_lib = measure_int8_peak(dev)

    # ---- the official H3 geometry in the real checkpoint format (fp8 e4m3 group-16 scales), through qlinear.linear
    official = None if args.no_official else official_points(dev)

    # ---- the DiT records: config 5 token-sharded over the N ranks (every N), config 3 on one GPU
    del weights, grids, acts, outs, codes, xs
    torch.cuda.empty_cache()
    sharded = block3 = None
    if not args.no_dit:
        group = dist.group.WORLD if world > 1 else None
        rec = dit_measure("longseq", args.dit_steps, 3, rank, world, local, group, args.kv_exchange, args.kv_groups,
                          e2e=False, check_rows=256 if world > 1 else 0)
        sharded = {k: v for k, v in rec.items() if not k.startswith("_")}
        if world == 1:
            rec3 = dit_measure("block", 2 * args.dit_steps, 3, rank, world, local, None, e2e=False)
            block3 = {k: v for k, v in rec3.items() if not k.startswith("_")}

    if args.detail and rank == 0:
        Path(args.detail).parent.mkdir(parents=True, exist_ok=True)
        Path(args.detail).write_text(json.dumps({"points": per_point, "totals_ms_per_step": tot, "clocks": clk}, indent=1))

    if rank == 0:
        line = {"metric": METRIC, "value": value, "unit": "TOPS", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
                "ms_per_step": t_max_ms / args.steps, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
                "dtype": "int8", "data": "synthetic", "config": config_dict(args.ms, world),
                "roofline": {"bound": "tensor", "kernel": "int8 GEMM (gemm_i8_pair_kernel for large M, gemm_w4s_kernel with "
                                                           "the int4 decode for small M)", "achieved": gemm_tops, "peak": int8_peak,
                             "unit": "TOPS", "frac": gemm_tops / int8_peak, "traffic": traffic,
                             "peak_note": f"int8 dense = 2 x {pk['source']} bf16 dense ({pk['bf16']} TFLOP/s burst)",
                             "frac_of_sustained": gemm_tops / (2.0 * pk["bf16_sustained"]) if pk.get("bf16_sustained") else None,
                             "int8_library_peak": int8_lib,
                             "frac_of_int8_library": gemm_tops / int8_lib["tops"] if int8_lib.get("tops") else None},
                "rotq_roofline": {"bound": "hbm", "kernel": "rotq_kernel", "achieved": rotq_gbs, "peak": pk["hbm_gbs"],
                                  "unit": "GB/s", "frac": rotq_gbs / pk["hbm_gbs"]},
                "kernel_ms_per_step": tot, "cpu_baseline": cpu, "e2e": e2e, "clocks": clk,
                "gpu_launches": sum(2 if fused[p] else 3 for p in points) * args.steps,
                "sharded_block": sharded, "block": block3, "official": official}
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
