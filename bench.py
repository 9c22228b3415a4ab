"""Benchmark of the B200 sampler on the heterogeneous continuous-batch
workload: batch 256 x vocab 128256 fp32 logits per step, per-row temperature,
top-k, top-p and repetition / presence / frequency penalties over a 512-token
history (the reference's serial per-sequence sampling loop,
src/inference.rs:112-138 -> src/decoder.rs:35-100, batched).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

One process per GPU (torchrun for N > 1). Batch rows are independent, so each
rank samples its own 256-row batch with no collective on the data path
(weak scaling); the time is the max over ranks of the device-timed region.
Prints one JSON line on rank 0.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "rust-llm_b200"))
sys.path.insert(0, os.path.join(ROOT, "oracle"))

B, V, H = 256, 128256, 512
METRIC = "sampled tokens/s at batch 256 x vocab 128256 fp32"
UNIT = "tokens/s"
POOL = 8  # distinct step buffers cycled through (8 x 131 MB > L2)


def algorithmic_bytes(b=B, v=V, h=H):
    # logits + history + hist_len + params + uniforms + token + prob + status
    return b * v * 4 + b * h * 4 + b * 4 + b * 24 + b * 4 + b * 4 + b * 4 + b * 4


def measured_peak():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            return float(json.load(f)["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


def committed_traffic():
    try:
        with open(os.path.join(ROOT, "profiles", "traffic.json")) as f:
            return json.load(f)
    except Exception:
        return {}


class ClockSampler:
    """nvidia-smi clock / throttle sampling during the timed region."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index):
        self.idx = gpu_index
        self.proc = None

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.idx), f"--query-gpu={self.Q}", "--format=csv,noheader,nounits",
                 "-lms", "100"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except Exception:
            self.proc = None

    def stop(self):
        if self.proc is None:
            return None
        time.sleep(0.25)
        self.proc.terminate()
        try:
            out, _ = self.proc.communicate(timeout=5)
        except Exception:
            self.proc.kill()
            return None
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in out.strip().splitlines():
            f = [x.strip() for x in line.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx = float(f[2])
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        if not sm:
            return None
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm)}


def make_params(step, rng_seed=2000):
    import workloads

    r = np.random.Generator(np.random.PCG64(rng_seed + step))
    from rlsampler import ROW_PARAMS_DTYPE

    p = np.zeros(B, ROW_PARAMS_DTYPE)
    p["temperature"] = r.uniform(0.5, 1.5, B)
    p["top_k"] = r.choice(np.array([0, 20, 50, 100]), B)
    p["top_p"] = r.uniform(0.8, 1.0, B)
    p["repeat_penalty"] = r.uniform(1.0, 1.3, B)
    p["presence_penalty"] = r.uniform(0.0, 0.5, B)
    p["frequency_penalty"] = r.uniform(0.0, 0.5, B)
    hist = r.integers(0, V, (B, H)).astype(np.int32)
    u = workloads.uniforms(2, step, B)
    return p, hist, u


def cpu_baseline(max_seconds=10.0, max_steps=400, distinct=2):
    """The CPU restatement of the sampler (oracle/, a port: the Rust
    reference cannot be built here) on this host's cores, over a bounded
    sample of config-2 steps (about max_seconds of timed sampling, cycling
    over `distinct` generated step batches)."""
    import oracle
    import workloads

    nthreads = os.cpu_count() or 1
    batches = [workloads.config2(i) for i in range(distinct)]
    hl = np.full(B, H, np.int32)
    rows = 0
    elapsed = 0.0
    steps = 0
    while steps < max_steps and elapsed < max_seconds:
        batch = batches[steps % distinct]
        t0 = time.perf_counter()
        oracle.spec_sample_batch(batch.logits, batch.hist, hl, None, batch.params, batch.uniforms,
                                 nthreads=nthreads)
        elapsed += time.perf_counter() - t0
        rows += B
        steps += 1
    return {"value": rows / elapsed, "unit": UNIT, "cores": nthreads, "kind": "port",
            "sample": f"{steps} steps x {B} rows x {V} vocab of the same workload ({distinct} distinct step "
                      f"batches cycled), {nthreads} threads, {elapsed:.1f} s of sampling"}


def run_reference(args, rank, world):
    line = {"impl": "reference", "metric": METRIC, "unit": UNIT, "higher_is_better": True}
    if rank != 0:
        return
    import oracle
    import workloads

    nthreads = os.cpu_count() or 1
    batch = workloads.config2(0)
    hl = np.full(B, H, np.int32)
    # each step samples a bounded slice of the 256-row batch (full V)
    rows_per_step = max(8, min(B, 4 * nthreads))
    sl = slice(0, rows_per_step)
    for _ in range(args.warmup):
        oracle.spec_sample_batch(batch.logits[sl], batch.hist[sl], hl[sl], None, batch.params[sl],
                                 batch.uniforms[sl], nthreads=nthreads)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        oracle.spec_sample_batch(batch.logits[sl], batch.hist[sl], hl[sl], None, batch.params[sl],
                                 batch.uniforms[sl], nthreads=nthreads)
    dt = time.perf_counter() - t0
    val = rows_per_step * args.steps / dt
    line.update({
        "value": val, "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": dt / args.steps * 1e3, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic", "config": {"workload": "hetero_batch_b256_v128256_f32", "global_batch": B,
                                        "vocab": V, "history": H, "rows_per_step_timed": rows_per_step},
        "cpu_baseline": {"value": val, "unit": UNIT, "cores": nthreads, "kind": "port",
                         "sample": f"{rows_per_step} of the {B} rows per step, full vocab, {nthreads} threads"},
        "e2e": {"value": val, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    })
    print(json.dumps(line), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--e2e-steps", type=int, default=20)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)

    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))

    if args.impl == "reference":
        return run_reference(args, rank, world)

    import torch
    import torch.distributed as dist

    import rlsampler

    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        import datetime

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=dev)

    s = rlsampler.Sampler(local, max_batch=B, max_vocab=V, max_history=H)
    stream = torch.cuda.current_stream(dev)

    # ---- device-resident pool of step inputs (inputs > L2) ----
    gen = torch.Generator(device=dev)
    prior = (-1.1 * torch.log(torch.arange(V, device=dev, dtype=torch.float64) + 1.0)).float()
    pool = []
    for i in range(POOL):
        gen.manual_seed(1000 * 2 + i + 7919 * rank)
        lg = torch.randn((B, V), generator=gen, device=dev, dtype=torch.float32) * 4.0 + prior
        p, hist, u = make_params(i + 100 * rank)
        pool.append(dict(logits=lg, params=rlsampler.params_tensor(p, dev),
                         hist=torch.from_numpy(hist).to(dev), hl=torch.full((B,), H, dtype=torch.int32, device=dev),
                         u=torch.from_numpy(u).to(dev)))
    out_tok = torch.empty(B, dtype=torch.int32, device=dev)
    out_prob = torch.empty(B, dtype=torch.float32, device=dev)
    row_st = torch.empty(B, dtype=torch.int32, device=dev)

    def step(i):
        d = pool[i % POOL]
        s.sample(d["logits"], d["params"], d["u"], d["hist"], d["hl"], None, out_tok, out_prob, row_st,
                 stream=stream)

    for i in range(args.warmup):
        step(i)
    torch.cuda.synchronize()
    bad = int((row_st != 0).sum().item())

    clk = ClockSampler(local)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    clk.start()
    ev0 = torch.cuda.Event(enable_timing=True)
    ev1 = torch.cuda.Event(enable_timing=True)
    ev0.record(stream)
    for i in range(args.steps):
        step(i)
    ev1.record(stream)
    torch.cuda.synchronize()
    clocks = clk.stop()
    ms = ev0.elapsed_time(ev1)
    if world > 1:
        t = torch.tensor([ms], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
        dist.barrier()
    ms_per_step = ms / args.steps
    value = world * B * args.steps / (ms / 1e3)

    # ---- end to end through the host-buffer entry point (pinned memory) ----
    hp = pool[0]
    h_logits = torch.empty((B, V), dtype=torch.float32, pin_memory=True)
    h_logits.copy_(hp["logits"].cpu())
    p0, hist0, u0 = make_params(0)
    h_params = np.ascontiguousarray(p0)
    h_hist = np.ascontiguousarray(hist0)
    h_hl = np.full(B, H, np.int32)
    h_u = np.ascontiguousarray(u0)
    h_tok = torch.empty(B, dtype=torch.int32, pin_memory=True)
    h_prob = torch.empty(B, dtype=torch.float32, pin_memory=True)
    import ctypes

    cp = lambda a: a.ctypes.data_as(ctypes.c_void_p)
    tp = lambda t: ctypes.c_void_p(t.data_ptr())

    def e2e_step():
        s.sample_host_ptrs(tp(h_logits), B, V, cp(h_params), cp(h_u), tp(h_tok), tp(h_prob), cp(h_hist),
                           cp(h_hl), H, None, 0)

    for _ in range(3):
        e2e_step()
    if world > 1:
        dist.barrier()
    t0 = time.perf_counter()
    for _ in range(args.e2e_steps):
        e2e_step()
    e2e_s = time.perf_counter() - t0
    if world > 1:
        t = torch.tensor([e2e_s], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_s = float(t.item())
    e2e_val = world * B * args.e2e_steps / e2e_s
    h2d = B * V * 4 + B * H * 4 + B * 4 + B * 24 + B * 4
    d2h = B * 4 + B * 4

    if rank == 0:
        peak, peak_kind = measured_peak()
        alg = algorithmic_bytes()
        achieved = alg / (ms_per_step * 1e-3) / 1e9
        traffic = committed_traffic().get("spec_step_f32_config2")
        line = {
            "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms_per_step, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": {"workload": "hetero_batch_b256_v128256_f32", "global_batch": world * B, "per_gpu_batch": B,
                       "vocab": V, "history": H, "parallelism": f"rows{world}",
                       "l2": f"inputs larger than L2: {POOL} distinct {B}x{V} f32 step buffers cycled"},
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                         "frac": achieved / peak, "peak_kind": peak_kind,
                         "kernel": "one step: spec_pipe_kernel (stream) + spec_finish_kernel, timed together",
                         "algorithmic_bytes_per_launch": alg, "traffic": traffic},
            # two of this library's kernels per step: the streaming kernel and the finish kernel
            "gpu_launches": 2 * args.steps,
            "rows_not_ok": bad,
            "e2e": {"value": e2e_val, "unit": UNIT, "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                    "path": "rl_sample_host (pinned host buffers, H2D + kernel + D2H + sync per step)"},
            "clocks": clocks,
        }
        if not args.no_cpu_baseline:
            line["cpu_baseline"] = cpu_baseline()
        print(json.dumps(line), flush=True)
    s.close()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
