#!/usr/bin/env python
"""Benchmark of the EXL3 trellis-decode GEMV path on B200 (driver contract: one JSON line).

Workload (the config its metric is quoted on): the dense EXL3 GEMV
sweep, shapes (out x in) 2048x7168, 7168x2048, 4096x14336, rates K in {2, 3, 4} (n = 32, 48,
64), batch M in {1, 2, 4, 8, 16, 64}: 54 projections.  One step runs every projection over a
ring of distinct weight copies whose total exceeds twice the 126 MB L2, so no launch reads a
weight another left in L2.  Weights are seeded random trellis words with sign-only scales (the
reference's synthetic-bank recipe, src/exl3/synth.zig:16-41): the decode cost does not depend on
the values.  Activations are bf16 N(0,1).

metric: compressed-HBM GB/s of the GEMVs (algorithmic bytes: trellis + suh + svh + x + y per
launch) over the device time of the step, graph-replayed with inputs resident in HBM.  e2e: the
same bytes over the time of the same projections called one by one through the C ABI with the
activations copied from pinned host memory and the outputs copied back, inside the timed region.
Rows from 16 go through the tensor-core projection (sx_linear_gemm); fewer through the decode
GEMV (sx_linear_ex with static weights).  At N > 1 every rank runs its own sweep (the projections
do not shard: replicas), value sums the ranks' bytes over the slowest rank's time.  roofline: the
headline launch (4096x14336 K2 M=1 gemv_kernel) against the measured HBM copy bandwidth.

Riding along: "moe" (configs[2]: the 512-expert decode layer, T = 1/8/64 tokens per rank; expert
parallel over the ranks at N > 1), and at N = 1 "moe_prefill" (configs[3]: 8192 tokens, Zipf
routing, tensor-core path) and "ffn_stack_deepseek" (configs[4]: 16 layers, rate-grouped K1/K2
routed experts, T = 1/8/64/4096).

--impl reference times the reference's CPU decode + matmul (`format.project`,
src/exl3/expert_exl3.zig:546; Zig is not installed, so its C++ restatement in oracle/) on the
host cores over the M = 1 projections of the sweep.
"""

import argparse
import ctypes
import json
import os
import subprocess
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

SHAPES = [(7168, 2048), (2048, 7168), (14336, 4096)]  # (in, out): out x in = 2048x7168, 7168x2048, 4096x14336
RATES = [32, 48, 64]
ROWS = [1, 2, 4, 8, 16, 64]
L2_BYTES = 126 * 1024 * 1024
GEMM_ROWS = 16  # sweep rows at or above this go through the tensor-core projection
# DRAM traffic of the headline launch comes from a committed record of one ncu capture, which
# names the digest of the kernel sources it was taken on; a changed kernel reports no traffic.
TRAFFIC_RECORD = os.path.join(ROOT, "profiles", "roofline_traffic.txt")
GEMV_SOURCES = ["sx_gemv_impl.cuh", "sx_core.cuh", "sx_decode.cuh", "sx_common.cuh", "sx_gemv.cu", "sx_gemv_mcg_nb1.cu"]
METRIC = "EXL3 GEMV compressed-HBM GB/s (% peak); MoE layer tokens/s at 1/2/4/8 B200"
UNIT = "GB/s"


def alg_bytes(in_f, out_f, n, m):
    return in_f * out_f * n // 128 + 2 * (in_f + out_f) + 2 * m * in_f + 2 * m * out_f


def sweep_config(world):
    """The workload both arms report on (the reference arm times a bounded sample of it)."""
    return {"workload": "gemv_sweep (BASELINE configs[1])", "shapes_out_x_in": ["2048x7168", "7168x2048", "4096x14336"],
            "n": RATES, "rows": ROWS, "codebook": "mcg", "window": 16,
            "l2": "ring of distinct weight copies > 2x L2 per (shape, rate)", "parallelism": f"replicas x{world}"}


def source_digest(names):
    """sha256 (16 hex digits) over the named kernel sources, in order (missing names skipped)."""
    import hashlib

    h = hashlib.sha256()
    for name in names:
        path = os.path.join(ROOT, "sushi_b200", "csrc", name)
        if os.path.exists(path):
            with open(path, "rb") as f:
                h.update(name.encode() + b"\0" + f.read())
    return h.hexdigest()[:16]


def recorded_traffic(kernel_key, sources):
    """(DRAM bytes per launch, provenance) of the kernel's last ncu capture, or (None, why):
    the record's lines are `key bytes digest command...`; a digest other than the current
    sources' means the capture was of an older kernel."""
    digest = source_digest(sources)
    try:
        with open(TRAFFIC_RECORD) as f:
            for line in f:
                parts = line.split(None, 3)
                if len(parts) >= 3 and parts[0] == kernel_key:
                    if parts[2] != digest:
                        return None, f"stale: captured on sources {parts[2]}, current {digest}"
                    return int(parts[1]), "ncu dram__bytes_read.sum + dram__bytes_write.sum, one capture: " + (
                        parts[3].strip() if len(parts) > 3 else "")
    except OSError:
        pass
    return None, f"no capture recorded for sources {digest}"


def host_cpu():
    """(model name, usable host threads) of this machine."""
    model = "unknown"
    try:
        with open("/proc/cpuinfo") as f:
            for line in f:
                if line.startswith("model name"):
                    model = line.split(":", 1)[1].strip()
                    break
    except OSError:
        pass
    try:
        cores = len(os.sched_getaffinity(0))
    except AttributeError:
        cores = os.cpu_count() or 1
    return model, cores


def measured_peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), float(p.get("bf16_tflops", 1618.5)), "measured"
    except Exception:
        return 6650.0, 1590.0, "fallback"


class ClockSampler:
    """nvidia-smi clocks and throttle reasons sampled every 50 ms while running."""

    def __init__(self, index):
        self.index = index
        self.samples = []
        self.proc = None
        self.thread = None

    def __enter__(self):
        q = ("clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown,"
             "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
             "clocks_event_reasons.sw_power_cap")
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={q}", "--format=csv,noheader,nounits", "-lms", "50", "-i", str(self.index)],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
            # nvidia-smi takes a moment to start: wait for its first line (at most 3 s), then keep
            # only the lines taken from here on, inside the timed region
            t_end = time.time() + 3.0
            while not self.samples and time.time() < t_end:
                time.sleep(0.005)
            self.samples.clear()
        except Exception:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) >= 7:
                self.samples.append(parts)

    def __exit__(self, *exc):
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()

    def summary(self):
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        sm = [float(s[0]) for s in self.samples if s[0].replace(".", "").isdigit()]
        mx = [float(s[1]) for s in self.samples if s[1].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for s in self.samples for i in range(4) if s[3 + i].lower() == "active"})
        return {"sm_mhz": float(np.median(sm)) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(self.samples)}


def dist_env():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return world, rank, local


# ---------------------------------------------------------------------------------------------
def run_reference(args):
    """The reference's CPU decode + matmul (oracle restatement) on the host cores."""
    world, rank, _ = dist_env()
    if rank != 0:
        return
    from oracle import oracle as orc
    from oracle import synth

    model, cores = host_cpu()
    orc.set_num_threads(cores)  # torch.distributed.run sets OMP_NUM_THREADS=1; use every host core
    threads = orc.num_threads()
    packs = []
    for (in_f, out_f) in SHAPES:
        for n in RATES:
            tr, su, sv = synth.random_bank(in_f * 7 + n, 1, in_f, out_f, n)
            packs.append((in_f, out_f, n, tr[0], su[0], sv[0], synth.activations(n, 1, in_f)))
    sample = packs  # every (shape, rate) at M = 1: 9 projections per step
    for _ in range(args.warmup):
        in_f, out_f, n, tr, su, sv, x = sample[0]
        orc.project(x, tr, su, sv, in_f, out_f, n, orc.CB_MCG, 16)
    t0 = time.perf_counter()
    total = 0
    for _ in range(args.steps):
        for in_f, out_f, n, tr, su, sv, x in sample:
            orc.project(x, tr, su, sv, in_f, out_f, n, orc.CB_MCG, 16)
            total += alg_bytes(in_f, out_f, n, 1)
    dt = time.perf_counter() - t0
    value = total / dt / 1e9
    config = sweep_config(world)
    config["reference_sample"] = "rows M = 1 of every (shape, rate); the CPU path costs M times the M = 1 time"
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": dt / args.steps * 1e3, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "u16 trellis -> f32 accumulate", "data": "synthetic (seeded random trellis words)",
        "config": config,
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": threads, "kind": "port", "cpu_model": model,
                         "sample": "each step: the sweep's 9 (shape, rate) projections at M = 1 (rows cost the CPU "
                                   "path proportionally; format.project restated in C++, OpenMP over output tiles)"},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------------------------------------
def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-moe", action="store_true")
    ap.add_argument("--profile", default=None, choices=["gemv", "moe", "gemm", "prefill"],
                    help="a small fixed case for ncu: --warmup launches, then --steps launches, no graphs")
    ap.add_argument("--profile-tokens", type=int, default=8, help="tokens of the --profile moe layer")
    ap.add_argument("--profile-rows", type=int, default=1024, help="rows of the --profile gemm projection")
    ap.add_argument("--profile-shape", default="4096x14336", choices=["4096x14336", "2048x7168", "7168x2048"],
                    help="out x in of the --profile gemm projection")
    args = ap.parse_args()
    if args.impl == "reference":
        return run_reference(args)
    if args.profile:
        return run_profile(args)

    import torch
    import torch.distributed as dist

    import sushi_b200 as sx
    from sushi_b200 import _lib
    from oracle import synth

    world, rank, local = dist_env()
    torch.cuda.set_device(local)
    if world > 1:
        import datetime

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=torch.device("cuda", local))
    L = _lib.load()
    # graphs are captured on a side stream; every launch of the bench runs on it
    stream = torch.cuda.Stream()
    torch.cuda.set_stream(stream)
    sptr = ctypes.c_void_p(stream.cuda_stream)
    dec = sx.Decode(sx.Codebook.MCG, 16).c()

    # ---------------- weights: a ring of distinct copies per (shape, rate)
    rings = {}
    for (in_f, out_f) in SHAPES:
        for n in RATES:
            size = in_f * out_f * n // 128
            copies = max(2, -(-2 * L2_BYTES // size))
            tr = torch.randint(-32768, 32768, (copies, in_f // 16, out_f // 16, n), dtype=torch.int16, device="cuda")
            su = (torch.randint(0, 2, (copies, in_f), device="cuda").half() * 2 - 1) * 0.05
            sv = torch.randint(0, 2, (copies, out_f), device="cuda").half() * 2 - 1
            projs = [_lib.SxProj(tr[c].data_ptr(), su[c].data_ptr(), sv[c].data_ptr(), 1, in_f, out_f, n, 0)
                     for c in range(copies)]
            rings[(in_f, out_f, n)] = (tr, su, sv, projs)
    maxm = max(ROWS)
    xbuf = {in_f: torch.randn((maxm, in_f), device="cuda").to(torch.bfloat16) for in_f, _ in SHAPES}
    ybuf = {out_f: torch.empty((maxm, out_f), device="cuda", dtype=torch.bfloat16) for _, out_f in SHAPES}
    configs = [(in_f, out_f, n, m) for (in_f, out_f) in SHAPES for n in RATES for m in ROWS]

    gemm_ws = torch.empty(max(in_f for in_f, _ in SHAPES) * maxm * 2 + 256, dtype=torch.uint8, device="cuda")

    def launch(in_f, out_f, n, m, proj):
        if m >= GEMM_ROWS:  # the tensor-core path (sx_linear_gemm) from 16 rows
            st = L.sx_linear_gemm(sptr, ctypes.byref(proj), ctypes.byref(dec), xbuf[in_f].data_ptr(), 2, m,
                                  ybuf[out_f].data_ptr(), gemm_ws.data_ptr(), gemm_ws.numel())
        else:  # the decode GEMV; weights are loaded once, so launches may overlap the previous one's tail
            st = L.sx_linear_ex(sptr, ctypes.byref(proj), ctypes.byref(dec), xbuf[in_f].data_ptr(), 2, m,
                                ybuf[out_f].data_ptr(), 1)
        if st:
            raise RuntimeError(f"{L.sx_status_name(st).decode()} {L.sx_last_error_detail().decode()} "
                               f"(out {out_f} in {in_f} n {n} rows {m})")

    # one graph per config: every ring copy once (each launch reads weights no recent launch read)
    graphs, launches_per_step, bytes_per_step = [], 0, 0
    for (in_f, out_f, n, m) in configs:
        projs = rings[(in_f, out_f, n)][3]
        for p in projs:  # warm (sets kernel attributes) before capture
            launch(in_f, out_f, n, m, p)
        torch.cuda.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=stream):
            for p in projs:
                launch(in_f, out_f, n, m, p)
        graphs.append((g, len(projs), alg_bytes(in_f, out_f, n, m) * len(projs)))
        launches_per_step += len(projs) * (2 if m >= GEMM_ROWS else 1)  # GEMM: prep + MMA kernel
        bytes_per_step += alg_bytes(in_f, out_f, n, m) * len(projs)
    torch.cuda.synchronize()

    def step(events=None):
        for i, (g, _, _) in enumerate(graphs):
            if events is not None:
                events[i][0].record(stream)
            g.replay()
            if events is not None:
                events[i][1].record(stream)

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    per_cfg = [[torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)] for _ in graphs]
    cfg_ms = np.zeros(len(graphs))
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    with ClockSampler(local) as clocks:
        t0 = torch.cuda.Event(enable_timing=True)
        t1 = torch.cuda.Event(enable_timing=True)
        t0.record(stream)
        for _ in range(args.steps):
            step(per_cfg)
            torch.cuda.synchronize()
            cfg_ms += np.array([a.elapsed_time(b) for a, b in per_cfg])
        t1.record(stream)
        torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    kernel_ms = float(cfg_ms.sum()) / args.steps  # device time of the GEMV launches per step
    total_ms = t0.elapsed_time(t1) / args.steps
    if world > 1:
        tt = torch.tensor([kernel_ms], device="cuda")
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        kernel_ms = float(tt.item())
    value = world * bytes_per_step / (kernel_ms * 1e-3) / 1e9

    # ---------------- e2e: the C ABI called per projection with pinned host activations
    hx = {in_f: torch.randn((maxm, in_f)).to(torch.bfloat16).pin_memory() for in_f, _ in SHAPES}
    hy = {out_f: torch.empty((maxm, out_f), dtype=torch.bfloat16).pin_memory() for _, out_f in SHAPES}
    h2d = sum(2 * m * in_f for (in_f, _, _, m) in configs)
    d2h = sum(2 * m * out_f for (_, out_f, _, m) in configs)
    e2e_bytes = sum(alg_bytes(*c) for c in configs)

    def e2e_step(k):
        for (in_f, out_f, n, m) in configs:
            projs = rings[(in_f, out_f, n)][3]
            xbuf[in_f][:m].copy_(hx[in_f][:m], non_blocking=True)
            launch(in_f, out_f, n, m, projs[k % len(projs)])
            hy[out_f][:m].copy_(ybuf[out_f][:m], non_blocking=True)

    for k in range(args.warmup):
        e2e_step(k)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for k in range(args.steps):
        e2e_step(k + 7)
    e1.record(stream)
    torch.cuda.synchronize()
    e2e_ms = e0.elapsed_time(e1) / args.steps
    if world > 1:
        tt = torch.tensor([e2e_ms], device="cuda")
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        e2e_ms = float(tt.item())
    e2e_value = world * e2e_bytes / (e2e_ms * 1e-3) / 1e9

    hbm_peak, tf_peak, peak_kind = measured_peaks()
    per_config = {}
    for (in_f, out_f, n, m), (g, copies, b), ms in zip(configs, graphs, cfg_ms / args.steps):
        per_config[f"{out_f}x{in_f}_n{n}_m{m}"] = round(b / (ms * 1e-3) / 1e9, 1)
    headline = per_config.get("4096x14336_n32_m1")
    traffic, traffic_src = recorded_traffic("gemv_kernel<MCG,32,1,W16>:4096x14336:m1", GEMV_SOURCES)
    dense0 = config0_bench(L, torch, stream, sptr, dec, args, hbm_peak)

    out = {
        "metric": METRIC, "value": round(value, 2), "unit": UNIT, "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(kernel_ms, 4), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "u16 trellis (K=2/3/4) decoded to f16, bf16 activations, f32 accumulate",
        "data": "synthetic (seeded random trellis words, sign-only scales; bf16 N(0,1) activations)",
        "config": sweep_config(world),
        # The dominant kernel at the metric's headline config: gemv_kernel on 4096x14336 K2 M=1;
        # achieved = its algorithmic bytes per launch over its average launch time in this run's
        # timed graphs; traffic = DRAM bytes read + written per launch from one ncu capture of the
        # same kernel sources (null when the kernel changed since).
        "roofline": {"bound": "hbm", "achieved": headline, "peak": hbm_peak, "unit": "GB/s",
                     "frac": round(headline / hbm_peak, 4) if headline else None, "traffic": traffic,
                     "traffic_source": traffic_src,
                     "algorithmic_bytes_per_launch": alg_bytes(14336, 4096, 32, 1), "peak_kind": peak_kind,
                     "kernel": "sx::gemv_kernel<MCG,32,1,W16> 4096x14336 M=1"},
        "sweep_gbs": round(bytes_per_step / (kernel_ms * 1e-3) / 1e9, 2),
        "e2e": {"value": round(e2e_value, 2), "unit": UNIT, "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h},
        "gpu_launches": launches_per_step * args.steps,
        "clocks": clocks.summary(),
        "headline_4096x14336_k2_m1_gbs": headline,
        "dense_4096x4096": dense0,
        "per_config_gbs": per_config,
        "wall_ms_per_step": round(total_ms, 3),
    }

    if world > 1:
        out["ep_parity"] = ep_parity(sx, torch)
    if not args.no_moe:
        out["moe"] = moe_bench(sx, _lib, torch, args, stream, sptr, hbm_peak)
        out["moe_prefill"] = prefill_bench(sx, torch, args, stream, tf_peak)
        if world > 1:
            out["moe_ep"] = ep_efficiency(sx, _lib, torch, args, stream, sptr, hbm_peak, tf_peak, out)
        out["ffn_stack_deepseek"] = deepseek_bench(sx, torch, args, stream, tf_peak)

    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        out["cpu_baseline"] = cpu_baseline()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    if rank == 0:
        print(json.dumps(out), flush=True)


def config0_bench(L, torch, stream, sptr, dec, args, hbm_peak):
    """one dense 4096x4096 linear at K2 (n32, MCG w16), batch 1, through the
    decode GEMV; a ring of distinct weight copies (> 2x L2) in a CUDA graph.  Compressed-HBM GB/s
    on the algorithmic bytes (trellis + suh + svh + x + y) and its fraction of the measured HBM
    copy bandwidth.  (Its parity, on the quantizer's own pack of that weight, is a GPU test.)"""
    from sushi_b200 import _lib

    in_f, out_f, n = 4096, 4096, 32
    size = in_f * out_f * n // 128
    copies = max(2, -(-2 * L2_BYTES // size))
    tr = torch.randint(-32768, 32768, (copies, in_f // 16, out_f // 16, n), dtype=torch.int16, device="cuda")
    su = (torch.randint(0, 2, (copies, in_f), device="cuda").half() * 2 - 1) * 0.05
    sv = torch.randint(0, 2, (copies, out_f), device="cuda").half() * 2 - 1
    projs = [_lib.SxProj(tr[c].data_ptr(), su[c].data_ptr(), sv[c].data_ptr(), 1, in_f, out_f, n, 0)
             for c in range(copies)]
    x = torch.randn((1, in_f), device="cuda").to(torch.bfloat16)
    y = torch.empty((1, out_f), device="cuda", dtype=torch.bfloat16)

    def run():
        for p in projs:
            st = L.sx_linear_ex(sptr, ctypes.byref(p), ctypes.byref(dec), x.data_ptr(), 2, 1, y.data_ptr(), 1)
            if st:
                raise RuntimeError(L.sx_status_name(st).decode())

    run()
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=stream):
        run()
    for _ in range(max(3, args.warmup)):
        g.replay()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    reps = max(5, args.steps)
    e0.record(stream)
    for _ in range(reps):
        g.replay()
    e1.record(stream)
    torch.cuda.synchronize()
    us = e0.elapsed_time(e1) * 1e3 / (reps * copies)
    del g
    gbs = alg_bytes(in_f, out_f, n, 1) / (us * 1e-6) / 1e9
    return {"workload": "configs[0]: 4096x4096 K2 (n32) M=1, decode GEMV", "us_per_launch": round(us, 3),
            "gbs": round(gbs, 1), "hbm_frac_of_measured": round(gbs / hbm_peak, 4),
            "algorithmic_bytes_per_launch": alg_bytes(in_f, out_f, n, 1), "copies": copies}


def ep_parity(sx, torch):
    """Expert-parallel correctness at N > 1, outside the timed regions: a seeded 64-expert layer
    (hidden 512, intermediate 256, K2, top-6, gated shared expert), identical on every rank; each
    rank routes its own tokens, runs them through the expert-parallel layer holding its eighth,
    quarter or half of the experts (ExpertParallel.moe, the shared expert on the side stream) and
    through the single-GPU layer over the whole bank (moe_folded), and compares.  The expert-
    parallel layer adds the ranks' f32 partials in rank order, the single-GPU one the slots in k
    order, so a row may differ in the last bf16 bit; the line reports how many rows are
    bit-identical and the largest difference in units of the output's last place."""
    import torch.distributed as dist

    world, rank, _ = dist_env()
    E, D, I, k = 64, 512, 256, 6
    El = E // world
    gen = torch.Generator(device="cuda")
    gen.manual_seed(2024)  # the same full bank, router and shared expert on every rank

    def proj(experts, i_f, o_f):
        tr = torch.randint(-32768, 32768, (experts, i_f // 16, o_f // 16, 32), dtype=torch.int16, device="cuda",
                           generator=gen)
        su = (torch.randint(0, 2, (experts, i_f), device="cuda", generator=gen).half() * 2 - 1) * 0.05
        sv = torch.randint(0, 2, (experts, o_f), device="cuda", generator=gen).half() * 2 - 1
        return sx.Proj(tr, su, sv)

    full = sx.Bank(proj(E, D, I), proj(E, D, I), proj(E, I, D))
    shared = sx.Bank(proj(1, D, I), proj(1, D, I), proj(1, I, D))
    local = sx.Bank(*[sx.Proj(p.trellis[rank * El:(rank + 1) * El], p.suh[rank * El:(rank + 1) * El],
                              p.svh[rank * El:(rank + 1) * El]) for p in (full.gate, full.up, full.down)])
    wr = (torch.randn((D, E), device="cuda", generator=gen) * 0.05).to(torch.bfloat16)
    wg = (torch.randn((D, 1), device="cuda", generator=gen) * 0.05).to(torch.bfloat16)
    dec = sx.Decode(sx.Codebook.MCG, 16)
    xg = torch.Generator(device="cuda")
    xg.manual_seed(3000 + rank)
    ep = sx.ExpertParallel.from_process_group()
    rows = same = 0
    worst = 0.0  # max |got - want| over max |want| of the case
    try:
        for T, cap in ((1, 1), (5, 8), (37, 40)):
            x = torch.randn((T, D), device="cuda", generator=xg).to(torch.bfloat16)
            inds, scores, _ = sx.router_topk_gate(x @ wr, k)
            gate = x @ wg
            got = ep.moe(x, local, E, inds, scores, dec, rows_cap=cap, shared_gate=gate, shared_bank=shared)
            want = sx.moe_folded(x, full, shared, inds, scores, dec, shared_gate=gate)
            torch.cuda.synchronize()
            same += int((got == want).all(dim=1).sum())
            rows += T
            diff = float((got.float() - want.float()).abs().max() / want.float().abs().max().clamp_min(1e-30))
            worst = max(worst, diff)
    finally:
        torch.cuda.synchronize()
        ep.destroy()
    t = torch.tensor([float(rows), float(same), worst], device="cuda")
    mx = t.clone()
    dist.all_reduce(t, op=dist.ReduceOp.SUM)
    dist.all_reduce(mx, op=dist.ReduceOp.MAX)
    assert sx.device_error() == 0
    return {"n": world, "rows": int(t[0]), "bit_identical_rows": int(t[1]), "max_abs_diff_over_max": float(mx[2]),
            "within_last_bf16_bit": float(mx[2]) <= 2.0 ** -7,
            "transport": "peer (NVLink)",
            "case": "64 experts 512/256 K2 top-6 + gated shared expert; 1, 5, 37 tokens per rank; "
                    "rank-order vs k-order f32 sums, so a row may differ in its last bf16 bit"}


def ep_efficiency(sx, _lib, torch, args, stream, sptr, hbm_peak, tf_peak, out):
    """The expert-parallel layer's scaling at N > 1, measured in this run: every rank also runs the
    one-GPU layer over the whole 512-expert bank (a replica, the same kernels as the N = 1 bench),
    and eff(N) = tokens/s at N / (N x tokens/s of one GPU), weak (T tokens per rank against T on
    one GPU) and at an equal total (64 decode tokens split over the ranks; 8192 prefill tokens split
    over the ranks, measured here against 8192 on one GPU)."""
    world, _, _ = dist_env()
    one = moe_bench(sx, _lib, torch, args, stream, sptr, hbm_peak, single=True)
    pre1 = prefill_bench(sx, torch, args, stream, tf_peak, single=True)
    strong = prefill_bench(sx, torch, args, stream, tf_peak, T=8192 // world)
    ep, ep_pre = out["moe"], out["moe_prefill"]
    res = {"ranks": world, "one_gpu": {f"T{T}_tokens_per_s": one[f"T{T}"]["tokens_per_s"] for T in (1, 8, 64)}}
    res["one_gpu"]["prefill_8192_tokens_per_s"] = pre1["tokens_per_s"]
    res["decode_weak_eff"] = {f"T{T}": round(ep[f"T{T}"]["tokens_per_s"] / (world * one[f"T{T}"]["tokens_per_s"]), 4)
                              for T in (1, 8, 64)}
    t_eq = 64 // world
    res["decode_equal_total_64_eff"] = round(ep[f"T{t_eq}"]["tokens_per_s"] / (world * one["T64"]["tokens_per_s"]), 4)
    res["prefill_weak_eff"] = round(ep_pre["tokens_per_s"] / (world * pre1["tokens_per_s"]), 4)
    res["prefill_equal_total_8192"] = {"tokens_per_rank": strong["tokens_per_rank"],
                                       "tokens_per_s": strong["tokens_per_s"], "ms_per_layer": strong["ms_per_layer"],
                                       "eff": round(strong["tokens_per_s"] / (world * pre1["tokens_per_s"]), 4)}
    return res


def qwen_shared(sx, torch, gen, D, I):
    """The configs[2] layer's shared expert (one SwiGLU expert of intermediate I, K2 n32, replicated
    on every rank) and its bf16 gate vector [D, 1]: the layer adds sigmoid(x . wg) * shared(x)
    (moeWithGatedShared)."""
    parts = []
    for (i_f, o_f) in ((D, I), (D, I), (I, D)):
        tr = torch.randint(-32768, 32768, (1, i_f // 16, o_f // 16, 32), dtype=torch.int16, device="cuda", generator=gen)
        su = (torch.randint(0, 2, (1, i_f), device="cuda", generator=gen).half() * 2 - 1) * 0.05
        sv = torch.randint(0, 2, (1, o_f), device="cuda", generator=gen).half() * 2 - 1
        parts.append(sx.Proj(tr, su, sv))
    wg = (torch.randn((D, 1), device="cuda", generator=gen) * 0.02).to(torch.bfloat16)
    return sx.Bank(*parts), wg


def moe_bench(sx, _lib, torch, args, stream, sptr, hbm_peak, single=False):
    """hidden 2048, 512 experts of 512, top-10, K2 (n32) MCG random banks,
    softmax router over fp32 logits from a bf16 2048x512 matrix, one sigmoid-gated shared expert of
    512; tokens/s of router + shared expert + routed experts for T tokens per rank.  One GPU: sx_moe over the whole bank.  N GPUs: expert parallel
    (sx_ep_moe), rank g holding experts [g*512/N, (g+1)*512/N), every rank routing its own T tokens
    (weak scaling: N*T tokens per step); tokens/s = N*T over the slowest rank's layer time.  Each
    measurement replays a CUDA graph of layers over a ring of distinct bank copies (> 2x L2)."""
    import torch.distributed as dist

    world, rank, _ = dist_env()
    if single:  # every rank its own one-GPU layer over the whole bank: the efficiency reference
        world, rank = 1, 0
    E, D, I, k = 512, 2048, 512, 10
    El = E // world
    bank_bytes = El * 3 * (D * I * 32 // 128 + 2 * (D + I))
    copies = max(2, -(-2 * L2_BYTES // bank_bytes))
    gen = torch.Generator(device="cuda")
    gen.manual_seed(1000 + rank)
    banks = []
    for c in range(copies):
        parts = []
        for (i_f, o_f) in ((D, I), (D, I), (I, D)):
            tr = torch.randint(-32768, 32768, (El, i_f // 16, o_f // 16, 32), dtype=torch.int16, device="cuda",
                               generator=gen)
            su = (torch.randint(0, 2, (El, i_f), device="cuda", generator=gen).half() * 2 - 1) * 0.05
            sv = torch.randint(0, 2, (El, o_f), device="cuda", generator=gen).half() * 2 - 1
            parts.append(sx.Proj(tr, su, sv))
        banks.append(sx.Bank(*parts))
    dec = sx.Decode(sx.Codebook.MCG, 16)
    ep = sx.ExpertParallel.from_process_group() if world > 1 else None
    res = {"experts_per_rank": El, "ranks": world, "copies": copies, "scaling": "weak (T tokens per rank)"}
    rgen = torch.Generator(device="cuda")
    rgen.manual_seed(7)  # the router and the shared expert are replicated: same weights on every rank
    wr = (torch.randn((D, E), device="cuda", generator=rgen) * 0.02).to(torch.bfloat16)
    shared, wg = qwen_shared(sx, torch, rgen, D, I)
    # T tokens per rank; at N > 1 also 64 / N per rank: the 64-token step split over the ranks
    # (equal total tokens per step: the strong-scaling point of the expert-parallel layer)
    Ts = [1, 8, 64] + ([64 // world] if world > 1 and 64 // world not in (1, 8, 64) else [])
    real_world = dist_env()[0]
    for T in Ts:
        x = torch.randn((T, D), device="cuda", generator=gen).to(torch.bfloat16)

        def layer(c):
            # bf16 logits straight into the router; at one token the router launch also computes
            # the shared expert's gate logit (the reference's softmax_gate, rows == 1 only)
            if T == 1:
                inds, scores, gate = sx.router_topk_gate(x @ wr, k, gate=(x, wg))
            else:
                inds, scores, _ = sx.router_topk_gate(x @ wr, k)
                gate = x @ wg
            if ep is None:  # the shared expert rides the routed launches
                return sx.moe_folded(x, banks[c % copies], shared, inds, scores, dec, shared_gate=gate)
            # expert parallel: the shared expert runs on the side stream during the exchange
            return ep.moe(x, banks[c % copies], E, inds, scores, dec, rows_cap=T, shared_gate=gate, shared_bank=shared)

        for i in range(max(3, args.warmup)):
            layer(i)
        torch.cuda.synchronize()
        reps = 2 * copies
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=stream):
            for i in range(reps):
                layer(i)
        g.replay()
        torch.cuda.synchronize()
        if real_world > 1:
            dist.barrier()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        rounds = max(3, args.steps)
        e0.record(stream)
        for _ in range(rounds):
            g.replay()
        e1.record(stream)
        torch.cuda.synchronize()
        ms = e0.elapsed_time(e1) / (rounds * reps)
        if real_world > 1:  # the slowest rank (with `single`, the slowest replica)
            tt = torch.tensor([ms], device="cuda")
            dist.all_reduce(tt, op=dist.ReduceOp.MAX)
            ms = float(tt.item())
        del g
        phases = None
        if ep is not None:  # one layer in a graph with CUDA events at the expert-parallel call's phases
            ep.phase_timing(True)
            layer(0)
            torch.cuda.synchronize()
            g1 = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g1, stream=stream):
                layer(0)
            for _ in range(3):
                g1.replay()
            phases = ep.phase_ms()
            torch.cuda.synchronize()
            del g1
            ep.phase_timing(False)
            pt = torch.tensor([phases[n] for n in ep.PHASES], device="cuda")
            dist.all_reduce(pt, op=dist.ReduceOp.MAX)
            phases = {n: round(float(v), 4) for n, v in zip(ep.PHASES, pt)}
        inds, _ = sx.router_topk((x @ wr).float(), k)
        active = int(torch.unique(inds).numel())
        # algorithmic HBM bytes of the layer on each rank: the experts it owns that any rank's
        # tokens touch, the shared expert, the router matrix and gate vector, x and y
        all_inds = inds.to(torch.int32).contiguous()
        if world > 1:
            gathered = torch.empty((world * T, k), dtype=torch.int32, device="cuda")
            dist.all_gather_into_tensor(gathered, all_inds)
            all_inds = gathered
        touched = torch.unique(all_inds)
        owned = int(((touched >= rank * El) & (touched < (rank + 1) * El)).sum())
        expert_b = 3 * (D * I * 32 // 128 + 2 * (D + I))
        rank_bytes = owned * expert_b + expert_b + D * E * 2 + D * 2 + 2 * T * D * 2
        tot = torch.tensor([float(rank_bytes)], device="cuda")
        if world > 1:
            dist.all_reduce(tot)
        gbs = float(tot.item()) / (ms * 1e-3) / 1e9
        res[f"T{T}"] = {"tokens_per_s": round(world * T / (ms * 1e-3), 1), "ms_per_layer": round(ms, 4),
                        "tokens_per_rank": T, "active_experts_rank0_tokens": active,
                        "alg_bytes_all_ranks": int(tot.item()), "gbs": round(gbs, 1),
                        "hbm_frac_of_measured": round(gbs / (world * hbm_peak), 4)}
        if phases:
            res[f"T{T}"]["ep_phases_ms_max_over_ranks_graph"] = phases
    if world > 1:
        res["equal_total_64_tokens"] = f"T{64 // world}"
    if ep is not None:
        torch.cuda.synchronize()
        ep.destroy()
    return res


def prefill_bench(sx, torch, args, stream, tf_peak, T=8192, single=False):
    """the configs[2] layer in prefill, 8192 tokens of bf16 N(0,1) hidden
    states per rank, routing skewed by a Zipf(1.1) bias log(r_e^-1.1 / sum) over a seeded rank
    permutation added to the logits; router + gated shared expert + routed experts through the
    tensor-core path.  One GPU: sx_moe over the whole bank.  N GPUs: expert parallel (sx_ep_moe,
    rows_cap = 8192), rank g holding experts [g*512/N, (g+1)*512/N) and routing its own 8192 tokens
    (weak scaling); the Zipf bias is the same on every rank, so the hot experts' owners carry more
    rows.  Roofline: tensor, F = 2*T*k*3*H*I + 2*T*3*H*I + 2*T*H*E flops per rank (routed GEMMs,
    shared expert, router) over the measured dense bf16 peak; weights are decoded inside the GEMMs."""
    import torch.distributed as dist

    world, rank, _ = dist_env()
    real_world = world
    if single:  # every rank its own one-GPU layer over the whole bank: the efficiency reference
        world, rank = 1, 0
    E, D, I, k = 512, 2048, 512, 10
    El = E // world
    gen = torch.Generator(device="cuda")
    gen.manual_seed(77 + rank)
    parts = []
    for (i_f, o_f) in ((D, I), (D, I), (I, D)):
        tr = torch.randint(-32768, 32768, (El, i_f // 16, o_f // 16, 32), dtype=torch.int16, device="cuda", generator=gen)
        su = (torch.randint(0, 2, (El, i_f), device="cuda", generator=gen).half() * 2 - 1) * 0.05
        sv = torch.randint(0, 2, (El, o_f), device="cuda", generator=gen).half() * 2 - 1
        parts.append(sx.Proj(tr, su, sv))
    bank = sx.Bank(*parts)
    dec = sx.Decode(sx.Codebook.MCG, 16)
    rgen = torch.Generator(device="cuda")
    rgen.manual_seed(78)  # router and shared expert: replicated
    wr = (torch.randn((D, E), device="cuda", generator=rgen) * 0.02).to(torch.bfloat16)
    shared, wg = qwen_shared(sx, torch, rgen, D, I)
    ranks = torch.randperm(E, generator=torch.Generator().manual_seed(5)).float() + 1.0
    zb = (ranks ** -1.1)
    bias = torch.log(zb / zb.sum()).cuda()
    x = torch.randn((T, D), device="cuda", generator=gen).to(torch.bfloat16)
    L = sx._lib.load()
    ep = sx.ExpertParallel.from_process_group() if world > 1 else None
    if ep is None:
        d = dec.c()
        ws = torch.empty(L.sx_moe_folded_workspace_bytes(ctypes.byref(bank.c()), ctypes.byref(shared.c()), ctypes.byref(d),
                                                         None, T, k), dtype=torch.uint8, device="cuda")
    else:
        ws = torch.empty(ep.workspace_bytes(bank, T, k, shared_bank=shared), dtype=torch.uint8, device="cuda")

    def layer():
        logits = (x @ wr).float() + bias
        inds, scores, _ = sx.router_topk_gate(logits, k)
        gate = x @ wg
        if ep is None:
            return sx.moe_folded(x, bank, shared, inds, scores, dec, shared_gate=gate, workspace=ws)
        return ep.moe(x, bank, E, inds, scores, dec, rows_cap=T, shared_gate=gate, workspace=ws, shared_bank=shared)

    for _ in range(max(3, args.warmup)):
        layer()
    torch.cuda.synchronize()
    if real_world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    reps = max(3, args.steps)
    e0.record(stream)
    for _ in range(reps):
        layer()
    e1.record(stream)
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / reps
    phases = None
    if ep is not None:  # one more layer with CUDA events at the expert-parallel call's phases
        ep.phase_timing(True)
        layer()
        ph = ep.phase_ms()
        ep.phase_timing(False)
        pt = torch.tensor([ph[n] for n in ep.PHASES], device="cuda")
        dist.all_reduce(pt, op=dist.ReduceOp.MAX)
        phases = {n: round(float(v), 4) for n, v in zip(ep.PHASES, pt)}
    if real_world > 1:
        tt = torch.tensor([ms], device="cuda")
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        ms = float(tt.item())
    flops = world * (2.0 * T * k * 3 * D * I + 2.0 * T * 3 * D * I + 2.0 * T * D * E)
    inds, _ = sx.router_topk((x @ wr).float() + bias, k)
    counts = torch.bincount(inds.flatten().long(), minlength=E)
    res = {"tokens": world * T, "tokens_per_rank": T, "ranks": world, "tokens_per_s": round(world * T / (ms * 1e-3), 1),
           "ms_per_layer": round(ms, 3), "tflops": round(flops / (ms * 1e-3) / 1e12, 1),
           "tensor_frac_of_measured": round(flops / (ms * 1e-3) / 1e12 / (world * tf_peak), 4),
           "max_rows_per_expert_rank0_tokens": int(counts.max()), "active_experts": int((counts > 0).sum())}
    if phases:
        res["ep_phases_ms_max_over_ranks"] = phases
    if ep is not None:
        torch.cuda.synchronize()
        ep.destroy()
    del ws
    torch.cuda.empty_cache()
    return res


def deepseek_bench(sx, torch, args, stream, tf_peak):
    """a DeepSeek-style FFN stack of 16 layers, hidden 7168, 256 routed
    experts of 2048 + one shared expert of 2048, top-8 sigmoid routing with a bias (renormalised,
    x2.5).  Routed experts are STQ SPEC1 (window 15) in two rate groups, K1 (n16, experts 0..63) and
    K2 (n32, experts 64..255): 1.75 bits per weight on average; the group an expert falls in is
    fixed by its id range, which is how a rate-grouped pack orders experts.  The shared expert is K4
    (n64): in the routed call on one GPU (sx_moe_ragged_folded: its own chain launches, no routing
    pass), on the side stream of the expert-parallel call at N > 1.  Each layer: router, shared
    expert + rate-grouped routed layer, residual add.  One GPU: sx_moe_ragged
    over all 256 experts.  N GPUs: expert parallel (sx_ep_moe_ragged), rank g holding experts
    [g*256/N, (g+1)*256/N) as its own rate groups, every rank running the stack on its own T tokens
    (weak scaling); router and shared expert replicated.  Decode batches T = 1, 8, 64 (CUDA graph of
    the 16 layers) and prefill T = 4096.  Random trellis words, sign-only scales (the decode cost
    does not depend on the values); 39 GB of routed weights over the world.  Each layer takes the
    RMS-normed residual stream as its input (torch's rms_norm, in the timed region), so the stack's
    activations and routing stay those of a well-scaled model."""
    import torch.distributed as dist

    world, rank, _ = dist_env()
    H, I, E, k, L = 7168, 2048, 256, 8, 16
    K1 = 64  # experts [0, 64) are K1 (n16), the rest K2 (n32)
    El = E // world
    e0, e1 = rank * El, (rank + 1) * El
    groups = [(b - a, n) for a, b, n in ((e0, min(e1, K1), 16), (max(e0, K1), e1, 32)) if b > a]
    gen = torch.Generator(device="cuda")
    gen.manual_seed(4242 + rank)
    rgen = torch.Generator(device="cuda")
    rgen.manual_seed(4243)  # router and shared expert: replicated

    def proj(g, experts, i_f, o_f, n):
        tr = torch.randint(-32768, 32768, (experts, i_f // 16, o_f // 16, n), dtype=torch.int16, device="cuda",
                           generator=g)
        su = (torch.randint(0, 2, (experts, i_f), device="cuda", generator=g).half() * 2 - 1) * 0.02
        sv = torch.randint(0, 2, (experts, o_f), device="cuda", generator=g).half() * 2 - 1
        return sx.Proj(tr, su, sv)

    layers = []
    for _ in range(L):
        banks = [sx.Bank(proj(gen, e, H, I, n), proj(gen, e, H, I, n), proj(gen, e, I, H, n)) for e, n in groups]
        shared = sx.Bank(proj(rgen, 1, H, I, 64), proj(rgen, 1, H, I, 64), proj(rgen, 1, I, H, 64))
        wr = (torch.randn((H, E), device="cuda", generator=rgen) * 0.02).to(torch.bfloat16)
        bias = torch.randn((E,), device="cuda", generator=rgen) * 0.1
        rb = sx.Ragged.from_banks(banks)
        del banks
        layers.append((rb, shared, wr, bias))
    dec = sx.Decode(sx.Codebook.SPEC1, 15, 1)  # spec1-w15: the table with rows at n = 16..128
    ep = sx.ExpertParallel.from_process_group() if world > 1 else None
    routed_gb = sum(sum(t.numel() * 2 for t in rb.trellis) for rb, _, _, _ in layers) / 1e9
    res = {"layers": L, "ranks": world, "routed_bits_per_weight": 1.75, "routed_gb_rank0": round(routed_gb, 2),
           "scaling": "weak (T tokens per rank)" if world > 1 else "one GPU"}
    Lib = sx._lib.load()
    for T in (1, 8, 64, 4096):
        x0 = torch.randn((T, H), device="cuda", generator=gen).to(torch.bfloat16)
        d = dec.c()
        routed_ws = (ep.workspace_bytes(layers[0][0], T, k, shared_bank=layers[0][1]) if ep is not None else
                     Lib.sx_moe_ragged_folded_workspace_bytes(ctypes.byref(layers[0][0].c()),
                                                              ctypes.byref(layers[0][1].c()), ctypes.byref(d), None, T, k))
        ws = torch.empty(routed_ws, dtype=torch.uint8, device="cuda")

        def stack():
            x = x0
            for rb, shared, wr, bias in layers:
                # the block's input norm (a model's post-attention RMSNorm): without it the residual
                # stream of random-weight SwiGLU layers grows without bound and routes on inf/NaN
                h = torch.nn.functional.rms_norm(x, (H,))
                inds, scores, _ = sx.router_topk_gate(h @ wr, k, mode=sx.RouterMode.SIGMOID_BIAS, bias=bias,
                                                      route_norm=True, route_scale=2.5)
                if ep is None:  # the K4 shared expert in the same call as the K1/K2 routed groups
                    x = x + sx.moe_folded(h, rb, shared, inds, scores, dec, workspace=ws)
                else:  # the shared expert on the side stream while the rows are exchanged
                    x = x + ep.moe(h, rb, E, inds, scores, dec, rows_cap=T, workspace=ws, shared_bank=shared)
            return x

        finite = bool(torch.isfinite(stack()).all())
        stack()
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
        e0_, e1_ = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        rounds = max(2, args.steps)
        if T <= 64:
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=stream):
                stack()
            g.replay()
            torch.cuda.synchronize()
            if world > 1:
                dist.barrier()
            torch.cuda.synchronize()
            e0_.record(stream)
            for _ in range(rounds):
                g.replay()
            e1_.record(stream)
            torch.cuda.synchronize()
            del g
        else:
            e0_.record(stream)
            for _ in range(rounds):
                stack()
            e1_.record(stream)
            torch.cuda.synchronize()
        ms = e0_.elapsed_time(e1_) / rounds
        if world > 1:
            tt = torch.tensor([ms], device="cuda")
            dist.all_reduce(tt, op=dist.ReduceOp.MAX)
            ms = float(tt.item())
        flops = world * 2.0 * T * L * (k + 1) * 3 * H * I
        res[f"T{T}"] = {"tokens_per_s": round(world * T / (ms * 1e-3), 1), "ms_per_stack": round(ms, 3),
                        "tflops": round(flops / (ms * 1e-3) / 1e12, 1), "output_finite": finite}
        if ep is not None and T == 4096:  # the last layer's phases, one eager stack with events on
            ep.phase_timing(True)
            stack()
            ph = ep.phase_ms()
            ep.phase_timing(False)
            pt = torch.tensor([ph[n] for n in ep.PHASES], device="cuda")
            dist.all_reduce(pt, op=dist.ReduceOp.MAX)
            res[f"T{T}"]["ep_phases_ms_last_layer_max_over_ranks"] = {n: round(float(v), 4)
                                                                     for n, v in zip(ep.PHASES, pt)}
        del ws
    assert sx.device_error() == 0
    if ep is not None:
        torch.cuda.synchronize()
        ep.destroy()
    del layers
    torch.cuda.empty_cache()
    return res


def run_profile(args):
    """ncu case: the 4096x14336 K2 (n32) M=1 projection (config 1's rate, the sweep's largest
    shape) over 12 distinct weight copies (176 MB > L2); the tensor-core projection of
    --profile-shape at K2 over --profile-rows rows (weight copies past twice L2); the prefill layer;
    or the bench's MoE decode layer at --profile-tokens tokens (8 by default)."""
    import torch

    import sushi_b200 as sx

    torch.cuda.set_device(0)
    dec = sx.Decode(sx.Codebook.MCG, 16)
    if args.profile == "prefill":
        class A:  # the prefill layer as in the bench, warmup + steps layers
            warmup, steps = args.warmup, args.steps
        prefill_bench(sx, torch, A, torch.cuda.current_stream(), 1618.5)
        torch.cuda.synchronize()
        assert sx.device_error() == 0
        print("profile case done", flush=True)
        return
    if args.profile == "gemm":
        out_f, in_f = (int(v) for v in args.profile_shape.split("x"))
        n, rows = 32, args.profile_rows
        copies = max(4, -(-2 * L2_BYTES // (in_f * out_f * n // 128)))  # weights past L2 between launches
        tr = torch.randint(-32768, 32768, (copies, in_f // 16, out_f // 16, n), dtype=torch.int16, device="cuda")
        su = (torch.randint(0, 2, (copies, in_f), device="cuda").half() * 2 - 1) * 0.05
        sv = torch.randint(0, 2, (copies, out_f), device="cuda").half() * 2 - 1
        projs = [sx.Proj(tr[c], su[c], sv[c]) for c in range(copies)]
        x = torch.randn((rows, in_f), device="cuda").to(torch.bfloat16)
        for i in range(args.warmup + args.steps):
            sx.linear_gemm(x, projs[i % copies], dec)
        torch.cuda.synchronize()
        assert sx.device_error() == 0
        print("profile case done", flush=True)
        return
    if args.profile == "gemv":
        in_f, out_f, n, copies = 14336, 4096, 32, 12
        tr = torch.randint(-32768, 32768, (copies, in_f // 16, out_f // 16, n), dtype=torch.int16, device="cuda")
        su = (torch.randint(0, 2, (copies, in_f), device="cuda").half() * 2 - 1) * 0.05
        sv = torch.randint(0, 2, (copies, out_f), device="cuda").half() * 2 - 1
        projs = [sx.Proj(tr[c], su[c], sv[c]) for c in range(copies)]
        x = torch.randn((1, in_f), device="cuda").to(torch.bfloat16)
        for i in range(args.warmup + args.steps):
            sx.linear(x, projs[i % copies], dec)
    else:
        # the bench's configs[2] layer (moe_bench's `layer`), eagerly: router logits, the router
        # (with the shared expert's gate logit at one token), the routed experts with the gated
        # shared expert folded in
        E, D, I, k, T = 512, 2048, 512, 10, args.profile_tokens
        parts = []
        for (i_f, o_f) in ((D, I), (D, I), (I, D)):
            tr = torch.randint(-32768, 32768, (E, i_f // 16, o_f // 16, 32), dtype=torch.int16, device="cuda")
            su = (torch.randint(0, 2, (E, i_f), device="cuda").half() * 2 - 1) * 0.05
            sv = torch.randint(0, 2, (E, o_f), device="cuda").half() * 2 - 1
            parts.append(sx.Proj(tr, su, sv))
        bank = sx.Bank(*parts)
        gen = torch.Generator(device="cuda")
        gen.manual_seed(7)
        wr = (torch.randn((D, E), device="cuda", generator=gen) * 0.02).to(torch.bfloat16)
        shared, wg = qwen_shared(sx, torch, gen, D, I)
        x = torch.randn((T, D), device="cuda").to(torch.bfloat16)
        for i in range(args.warmup + args.steps):
            if T == 1:
                inds, scores, gate = sx.router_topk_gate(x @ wr, k, gate=(x, wg))
            else:
                inds, scores, _ = sx.router_topk_gate(x @ wr, k)
                gate = x @ wg
            sx.moe_folded(x, bank, shared, inds, scores, dec, shared_gate=gate)
    torch.cuda.synchronize()
    assert sx.device_error() == 0
    print("profile case done", flush=True)


def cpu_moe_layer(orc, synth, T, threads):
    """The reference's CPU path for one configs[2] decode layer of T tokens: routing per
    moeRoutingChain (softmax, top-10, renormalised; src/moe_router.zig:16-65) over f32 logits,
    then per (token, slot) the SwiGLU expert of f32_truth.Dense.run (src/exl3/f32_truth.zig:85)
    with every projection through format.project (decode + matmul, src/exl3/expert_exl3.zig:546),
    plus the sigmoid-gated shared expert.  Returns seconds per layer."""
    E, D, I, k, n = 512, 2048, 512, 10, 32
    rng = np.random.default_rng(31)
    wr = (rng.standard_normal((D, E)) * 0.02).astype(np.float32)
    wg = (rng.standard_normal(D) * 0.02).astype(np.float32)
    x = synth.activations(32, T, D)
    banks = {}

    def expert(e):
        if e not in banks:
            banks[e] = [tuple(a[0] for a in synth.random_bank(7000 + 3 * e + p, 1, i_f, o_f, n))
                        for p, (i_f, o_f) in enumerate(((D, I), (D, I), (I, D)))]
        return banks[e]

    def swiglu(e, xr):
        (gt, gs, gv), (ut, us, uv), (dt, ds, dv) = expert(e)
        g = orc.project(xr, gt, gs, gv, D, I, n, orc.CB_MCG, 16, threads=threads)[0]
        u = orc.project(xr, ut, us, uv, D, I, n, orc.CB_MCG, 16, threads=threads)[0]
        act = (g / (1.0 + np.exp(-g)) * u).astype(np.float32)
        return orc.project(act, dt, ds, dv, I, D, n, orc.CB_MCG, 16, threads=threads)[0]

    def layer():
        logits = x @ wr
        y = np.zeros((T, D), np.float32)
        for r in range(T):
            ii, ww = orc.router_truth(logits[r:r + 1], k)
            for e, w in zip(ii[0], ww[0]):
                y[r] += np.float32(w) * swiglu(int(e), x[r])
            y[r] += swiglu(-1, x[r]) / np.float32(1.0 + np.exp(-float(x[r] @ wg)))
        return y

    layer()  # warm: decodes nothing ahead, but builds the touched experts' packs
    reps = 3
    t0 = time.perf_counter()
    for _ in range(reps):
        layer()
    return (time.perf_counter() - t0) / reps


def cpu_baseline():
    """The reference's CPU decode + matmul timed on this host: the headline projection with every
    host thread and with one, and the configs[2] MoE decode layer at 1 and 8 tokens."""
    from oracle import oracle as orc
    from oracle import synth

    model, cores = host_cpu()
    orc.set_num_threads(cores)
    in_f, out_f, n = 14336, 4096, 32
    tr, su, sv = synth.random_bank(5, 1, in_f, out_f, n)
    x = synth.activations(5, 1, in_f)
    orc.project(x, tr[0], su[0], sv[0], in_f, out_f, n, orc.CB_MCG, 16)
    t0 = time.perf_counter()
    reps = 3
    for _ in range(reps):
        orc.project(x, tr[0], su[0], sv[0], in_f, out_f, n, orc.CB_MCG, 16)
    dt = (time.perf_counter() - t0) / reps
    t0 = time.perf_counter()
    orc.project_single_thread(x, tr[0], su[0], sv[0], in_f, out_f, n, orc.CB_MCG, 16)
    dt1 = time.perf_counter() - t0
    b = alg_bytes(in_f, out_f, n, 1)
    moe = {}
    for T in (1, 8):
        sec = cpu_moe_layer(orc, synth, T, cores)
        moe[f"T{T}"] = {"tokens_per_s": round(T / sec, 2), "ms_per_layer": round(sec * 1e3, 2)}
    return {"value": round(b / dt / 1e9, 3), "unit": UNIT, "cores": orc.num_threads(), "kind": "port",
            "cpu_model": model, "single_thread_gbs": round(b / dt1 / 1e9, 4),
            "sample": "4096x14336 K2 M=1 projection x3 on every host thread, x1 on one (format.project restated "
                      "in C++, OpenMP over output tiles)",
            "moe_decode_layer": dict(moe, workload="configs[2] layer, routed top-10 + gated shared expert, "
                                                   "every projection through format.project on every host thread")}


if __name__ == "__main__":
    main()
