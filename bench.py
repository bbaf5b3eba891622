#!/usr/bin/env python
"""Benchmark of the fused sequence-mixing hot path on B200 (one JSON line).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--config linear|mingru]

Default workload: BASELINE configs[1] -- the diagonal linear-RNN scan
h_t = a_t h_{t-1} + b_t, forward + backward, bf16 io / f32 state,
batch 8 x seq 4096 x hidden 2048 per GPU (weak scaling: rank r owns batch
rows [8r, 8r+8) of a global batch of 8N, no collective on the data path).
A step = one forward + one backward pass over the shard; tokens = batch*seq.

--impl ours       our kernels (libedifice_b200.so); device-timed with CUDA
                  events, max over ranks; plus e2e through the public API with
                  host buffers, roofline of the dominant kernel, CPU baseline.
--impl reference  the reference algorithm on the host CPU (the oracle port of
                  Edifice's Nx fallbacks, f32, OpenMP over all host cores);
                  rank 0 only.

Under torchrun every rank joins an NCCL group used only for the barrier and
the max-over-ranks reduction of the elapsed time.
"""
import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--config", choices=["linear", "mingru"], default="linear")
    ap.add_argument("--e2e-steps", type=int, default=10)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    return ap.parse_args()


def dist_env():
    return (int(os.environ.get("RANK", "0")), int(os.environ.get("WORLD_SIZE", "1")),
            int(os.environ.get("LOCAL_RANK", "0")))


# ------------------------------------------------------------------ clocks
class ClockSampler:
    """nvidia-smi clocks/throttle sampler for the timed region (100 ms period)."""
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index):
        self.gpu = gpu_index
        self.rows = []
        self.proc = None
        self.thread = None

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "--query-gpu=" + self.FIELDS, "--format=csv,noheader,nounits",
                 "-i", str(self.gpu), "-lms", "100"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except (OSError, ValueError):
            self.proc = None
            return
        self.thread = threading.Thread(target=self._read, daemon=True)
        self.thread.start()

    def _read(self):
        for line in self.proc.stdout:
            self.rows.append((time.time(), [x.strip() for x in line.split(",")]))

    def stop(self):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
            if self.thread:
                self.thread.join(timeout=2)

    def summary(self, t0, t1):
        if not self.rows:
            return None
        inside = [r for t, r in self.rows if t0 <= t <= t1]
        used = inside if inside else [r for _, r in self.rows]
        sm = [float(r[1]) for r in used if r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in used if r[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in used for i in range(4)
                          if len(r) > 5 + i and r[5 + i].lower().startswith("active")})
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": max(mx) if mx else None, "reasons": reasons,
                "samples": len(inside), "window": "timed" if inside else "whole run"}


def measured_peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), "measured (MEASURED_PEAKS.json hbm_gbs)"
    return 6650.0, "fallback (6.65 TB/s pool measurement)"


def ncu_traffic(kernel_key):
    """Per-launch DRAM bytes of a kernel from the committed ncu summary, if any."""
    p = os.path.join(ROOT, "profiles", "ncu_traffic.json")
    if not os.path.exists(p):
        return None
    with open(p) as f:
        d = json.load(f)
    e = d.get(kernel_key)
    return None if e is None else e.get("traffic_bytes_per_launch")


# ------------------------------------------------------------- CPU baseline
def cpu_scan_step(cfg, a, b, dy, prec="f32"):
    import oracle as O
    if cfg.mingru:
        h = O.mingru_fwd(a, b, prec=prec)
        O.mingru_bwd(a, b, None, h, dy, prec=prec)
    else:
        h = O.linear_scan_fwd(a, b, prec=prec)
        O.linear_scan_bwd(a, None, h, dy, prec=prec)


def cpu_sample(cfg, rows, seed=0):
    import numpy as np
    rng = np.random.default_rng(seed)
    shp = (rows, cfg.seq_len, cfg.hidden)
    a = (1 / (1 + np.exp(-rng.standard_normal(shp, dtype=np.float32)))).astype(np.float32)
    b = rng.standard_normal(shp, dtype=np.float32)
    dy = rng.standard_normal(shp, dtype=np.float32)
    return a, b, dy


def cpu_threads():
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1


def time_cpu_baseline(cfg, budget_s=15.0):
    """Oracle f32 port, all host threads, on `rows` batch rows of the config;
    repeats until ~budget_s of CPU work.  Returns the cpu_baseline object."""
    import oracle as O
    n = cpu_threads()
    O.set_threads(n)
    rows = cfg.batch
    a, b, dy = cpu_sample(cfg, rows)
    cpu_scan_step(cfg, a, b, dy)  # warm
    t0 = time.perf_counter()
    reps = 0
    while True:
        cpu_scan_step(cfg, a, b, dy)
        reps += 1
        el = time.perf_counter() - t0
        if el >= budget_s or reps >= 200:
            break
    tok_s = reps * rows * cfg.seq_len / el
    return {"value": tok_s, "unit": "tokens/s", "cores": n, "kind": "port",
            "sample": "%d x fwd+bwd of the full %d-row config (%s), %.1f s of CPU work, "
                      "oracle f32 port of the Nx fallbacks (fused_scan.ex:4429-4444, 884-916)"
                      % (reps, rows, cfg.name, el)}


# ------------------------------------------------------------------ ours
def run_ours(args, cfg):
    import torch
    import torch.distributed as dist
    from edifice_b200 import fused_scan as fs
    from edifice_b200 import shard, device_errors

    rank, world, local = dist_env()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        import datetime
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=dev)

    units = shard.plan_units(cfg.units, rank, world)
    a, b, dy = shard.scan_inputs(cfg, units, dev)
    fwd = fs.mingru_scan if cfg.mingru else fs.linear_scan
    bwd_fn = (lambda a_, h_, dy_: fs.mingru_backward(a_, b, None, h_, dy_)) if cfg.mingru else \
        (lambda a_, h_, dy_: fs.linear_scan_backward(a_, None, h_, dy_))

    def step(ev=None):
        if ev is not None:
            ev[0].record()
        h = fwd(a, b)
        if ev is not None:
            ev[1].record()
        g = bwd_fn(a, h, dy)
        if ev is not None:
            ev[2].record()
        return h, g

    for _ in range(max(3, args.warmup)):
        step()
    torch.cuda.synchronize()
    K = args.steps
    evs = [[torch.cuda.Event(enable_timing=True) for _ in range(3)] for _ in range(K)]
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)

    sampler = ClockSampler(local)
    sampler.start()
    time.sleep(0.3)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    t_wall0 = time.time()
    start.record()
    for i in range(K):
        step(evs[i])
    end.record()
    torch.cuda.synchronize()
    t_wall1 = time.time()
    if world > 1:
        dist.barrier()
    sampler.stop()
    elapsed = start.elapsed_time(end)  # ms
    fwd_ms = statistics.mean(e[0].elapsed_time(e[1]) for e in evs)
    bwd_ms = statistics.mean(e[1].elapsed_time(e[2]) for e in evs)
    if world > 1:
        t = torch.tensor([elapsed, fwd_ms, bwd_ms], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        elapsed, fwd_ms, bwd_ms = t.tolist()
    errs = device_errors()

    # ---- e2e through the public API with host buffers
    e2e = None
    if args.e2e_steps > 0:
        pin = [x.cpu().pin_memory() for x in (a, b, dy)]
        dev_in = [torch.empty_like(x) for x in (a, b, dy)]
        outs_host = None

        def e2e_step():
            nonlocal outs_host
            for d_, h_ in zip(dev_in, pin):
                d_.copy_(h_, non_blocking=True)
            h = fwd(dev_in[0], dev_in[1])
            if cfg.mingru:
                g = fs.mingru_backward(dev_in[0], dev_in[1], None, h, dev_in[2])
            else:
                g = fs.linear_scan_backward(dev_in[0], None, h, dev_in[2])
            res = (h,) + tuple(g)
            if outs_host is None:
                outs_host = [torch.empty(r.shape, dtype=r.dtype, pin_memory=True) for r in res]
            for o_, r_ in zip(outs_host, res):
                o_.copy_(r_, non_blocking=True)
            return res

        e2e_step()
        e2e_step()
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        s2, e2 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s2.record()
        for _ in range(args.e2e_steps):
            e2e_step()
        e2.record()
        torch.cuda.synchronize()
        el2 = s2.elapsed_time(e2)
        if world > 1:
            t = torch.tensor([el2], device=dev, dtype=torch.float64)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            el2 = t.item()
        h2d = sum(x.numel() * x.element_size() for x in pin)
        d2h = sum(x.numel() * x.element_size() for x in outs_host)
        e2e = {"value": world * cfg.tokens * args.e2e_steps / (el2 / 1000.0), "unit": "tokens/s",
               "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
               "ms_per_step": el2 / args.e2e_steps, "steps": args.e2e_steps,
               "api": "edifice_b200.fused_scan (%s + backward)" %
                      ("mingru_scan" if cfg.mingru else "linear_scan")}

    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    if rank != 0:
        return

    peak, peak_src = measured_peaks()
    kern_bytes = {"fwd": cfg.bytes_fwd(), "bwd": cfg.bytes_bwd()}
    kern_ms = {"fwd": fwd_ms, "bwd": bwd_ms}
    dom = max(kern_ms, key=kern_ms.get)
    achieved = kern_bytes[dom] / (kern_ms[dom] / 1000.0) / 1e9
    kname = "%s_%s" % ("mingru" if cfg.mingru else "linear_scan", dom)
    traffic = ncu_traffic(kname)
    roof = {"bound": "hbm", "kernel": kname, "achieved": round(achieved, 1),
            "peak": peak, "unit": "GB/s", "frac": round(achieved / peak, 4),
            "peak_source": peak_src,
            "algorithmic_bytes_per_launch": kern_bytes[dom],
            "traffic": traffic}
    per_kernel = {k: {"ms": round(kern_ms[k], 4),
                      "GB/s": round(kern_bytes[k] / (kern_ms[k] / 1000.0) / 1e9, 1),
                      "frac_of_peak": round(kern_bytes[k] / (kern_ms[k] / 1000.0) / 1e9 / peak, 4)}
                  for k in kern_ms}
    cpu = None
    if world == 1 and not args.no_cpu_baseline:
        cpu = time_cpu_baseline(cfg)
    ms_step = elapsed / K
    value = world * cfg.tokens * K / (elapsed / 1000.0)
    line = {
        "metric": "scan/delta/attn fwd+bwd tokens/s",
        "value": value, "unit": "tokens/s", "n_gpus": world, "steps": K,
        "warmup": max(3, args.warmup), "ms_per_step": ms_step, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
        "config": {"workload": "%s fwd+bwd (BASELINE configs[1]%s)" %
                               (cfg.name, ", MinGRU form" if cfg.mingru else ""),
                   "batch_per_gpu": cfg.batch, "global_batch": cfg.batch * world,
                   "seq_len": cfg.seq_len, "hidden": cfg.hidden,
                   "parallelism": "dp%d (batch-row shards, no collective)" % world,
                   "l2": "inputs larger than L2 (%.2f GB touched per step > 126 MB)"
                         % ((kern_bytes["fwd"] + kern_bytes["bwd"]) / 1e9)},
        "roofline": roof, "kernels": per_kernel, "cpu_baseline": cpu, "e2e": e2e,
        "gpu_launches": 2 * K,
        "clocks": sampler.summary(t_wall0, t_wall1),
        "device_errors": errs,
    }
    print(json.dumps(line), flush=True)


# --------------------------------------------------------------- reference
def run_reference(args, cfg):
    rank, world, _ = dist_env()
    if rank != 0:
        return
    import oracle as O
    n = cpu_threads()
    O.set_threads(n)
    # size the per-step sample so W+K steps fit in ~150 s
    rows = cfg.batch
    a, b, dy = cpu_sample(cfg, rows)
    t0 = time.perf_counter()
    cpu_scan_step(cfg, a, b, dy)
    one = time.perf_counter() - t0
    total = (args.steps + args.warmup) * one
    if total > 150.0:
        frac = 150.0 / total
        hs = max(64, int(cfg.hidden * frac) // 64 * 64)
        a, b, dy = a[:1, :, :hs].copy(), b[:1, :, :hs].copy(), dy[:1, :, :hs].copy()
        rows, sample = 1, "1 batch row x %d of %d channels" % (hs, cfg.hidden)
        tok_per_step = cfg.seq_len * hs / cfg.hidden
    else:
        sample = "the full %d-row config" % rows
        tok_per_step = rows * cfg.seq_len
    for _ in range(args.warmup):
        cpu_scan_step(cfg, a, b, dy)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        cpu_scan_step(cfg, a, b, dy)
    el = time.perf_counter() - t0
    value = tok_per_step * args.steps / el
    line = {
        "impl": "reference",
        "metric": "scan/delta/attn fwd+bwd tokens/s", "value": value, "unit": "tokens/s",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": el * 1000.0 / args.steps, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": "%s fwd+bwd (BASELINE configs[1])" % cfg.name,
                   "batch_per_gpu": cfg.batch, "seq_len": cfg.seq_len, "hidden": cfg.hidden},
        "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": n, "kind": "port",
                         "sample": sample + "; tokens scaled by the sampled fraction; oracle "
                                   "f32 restatement of the Nx fallbacks (the reference's Nx/EXLA "
                                   "host path itself needs Erlang/Elixir, absent here)"},
        "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def main():
    args = parse()
    from edifice_b200.shard import ScanConfig
    cfg = ScanConfig(name="mingru_cfg1", mingru=True) if args.config == "mingru" else ScanConfig()
    if args.impl == "reference":
        run_reference(args, cfg)
    else:
        run_ours(args, cfg)


if __name__ == "__main__":
    main()
