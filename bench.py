"""Benchmark of the B200 sampler (rust-llm's logits -> token path,
src/decoder.rs, batched) on the five workloads:

  1  single sequence at the CLI defaults: B 1 x V 32000, top_k 40, top_p 0.9,
     repetition penalty over a 64-token history (microseconds per token)
  2  heterogeneous continuous batch: B 256 x V 128256 f32, per-row T, top_k,
     top_p and penalties over a 512-token history (the headline; tokens/s)
  3  grammar-constrained: B 64 x V 32000 with bit-packed allowed masks
  4  beam step: 16 items x 8 beams x V 151936 (beam extensions/s)
  5  vocabulary shards: B 1024 x V 256000 bf16 split across the ranks,
     merged by one NCCL all-gather (tokens/s, strong scaling)

    python bench.py [--config C] [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

One process per GPU (torchrun for N > 1); rank 0 prints one JSON line. For
configs 1-4 every rank samples its own batch with no collective (weak
scaling); config 5 splits one batch's vocabulary across the ranks. The
default (config 2) line also carries the config-5 step at the same N under
"vocab_shards", so a scaling run measures both.
"""
from __future__ import annotations

import argparse
import ctypes
import datetime
import json
import os
import platform
import statistics
import subprocess
import sys
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "rust-llm_b200"))
sys.path.insert(0, os.path.join(ROOT, "oracle"))

POOL = 8  # distinct step buffers cycled through (inputs larger than L2 for config 2)

CONFIGS = {
    1: dict(workload="single_seq_cli_defaults_b1_v32000", B=1, V=32000, H=64,
            metric="microseconds per sampled token at batch 1 x vocab 32000 (CLI defaults)", unit="us/token",
            higher=False),
    2: dict(workload="hetero_batch_b256_v128256_f32", B=256, V=128256, H=512,
            metric="sampled tokens/s at batch 256 x vocab 128256 fp32", unit="tokens/s", higher=True),
    3: dict(workload="grammar_b64_v32000", B=64, V=32000, H=0,
            metric="sampled tokens/s at batch 64 x vocab 32000 with grammar masks", unit="tokens/s", higher=True),
    4: dict(workload="beam_16x8_v151936", B=128, V=151936, H=0,
            metric="beam extensions/s at 16 items x 8 beams x vocab 151936", unit="beam extensions/s", higher=True),
    5: dict(workload="vocab_shard_b1024_v256000_bf16", B=1024, V=256000, H=256,
            metric="sampled tokens/s at batch 1024 x vocab 256000 bf16, vocabulary split across the GPUs",
            unit="tokens/s", higher=True),
    6: dict(workload="lmhead_sample_b256_h4096_v128256_bf16", B=256, V=128256, H=512, HID=4096,
            metric="sampled tokens/s from final hidden states at batch 256 x hidden 4096 x vocab 128256 "
                   "(bf16 LM head on the tensor cores + the batched sampler)", unit="tokens/s", higher=True),
}


def algorithmic_bytes(cfg, n_ranks=1):
    """Bytes one step must move at least (logits once, history, params,
    masks, outputs), per GPU."""
    c = CONFIGS[cfg]
    B, V, H = c["B"], c["V"], c["H"]
    if cfg == 4:
        return B * V * 4 + B * (4 + 1 + 4) + 16 * 16 * (4 + 4 + 4 + 1)
    if cfg == 5:
        w = -(-V // n_ranks)
        return B * w * 2 + B * H * 4 + B * 4 + B * 24 + B * 4 + B * 12 + (B * 1056 * n_ranks if n_ranks > 1 else 0)
    mask = B * ((V + 31) // 32) * 4 if cfg == 3 else 0
    return B * V * 4 + B * H * 4 + B * 4 + B * 24 + B * 4 + B * 12 + mask


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


def cpu_model():
    try:
        with open("/proc/cpuinfo") as f:
            for line in f:
                if line.startswith("model name"):
                    return line.split(":", 1)[1].strip()
    except Exception:
        pass
    return platform.processor() or "unknown"


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
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": mx, "reasons": sorted(reasons), "samples": len(sm)}


# ---------------------------------------------------------------------------
# Step inputs (seeded, synthetic: the reference publishes no data set)
# ---------------------------------------------------------------------------
def config2_params(step, B, V, H):
    import workloads
    from rlsampler import ROW_PARAMS_DTYPE

    r = np.random.Generator(np.random.PCG64(2000 + step))
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


def make_pool(cfg, dev, rank, n_ranks, count=POOL):
    """`count` device-resident steps of the configuration (this rank's part:
    its own rows for configs 1-4, its own columns of shared rows for 5)."""
    import torch

    import rlsampler
    import workloads

    c = CONFIGS[cfg]
    B, V, H = c["B"], c["V"], c["H"]
    gen = torch.Generator(device=dev)
    pool = []
    for i in range(count):
        gen.manual_seed(1000 * cfg + i + (7919 * rank if cfg != 5 else 0))
        d = {}
        if cfg == 2:
            prior = (-1.1 * torch.log(torch.arange(V, device=dev, dtype=torch.float64) + 1.0)).float()
            d["logits"] = torch.randn((B, V), generator=gen, device=dev, dtype=torch.float32) * 4.0 + prior
            p, hist, u = config2_params(i + 100 * rank, B, V, H)
        elif cfg in (1, 3):
            b = workloads.config1(i + 100 * rank) if cfg == 1 else workloads.config3(i + 100 * rank)
            d["logits"] = torch.from_numpy(b.logits).to(dev)
            p, u = b.params, b.uniforms
            hist = b.hist
            if b.mask is not None:
                d["mask"] = torch.from_numpy(b.mask.view(np.int32)).to(dev)
        elif cfg == 4:
            bb = workloads.config4(i + 100 * rank)
            d["logits"] = torch.from_numpy(bb.logits).to(dev)
            d["scores"] = torch.from_numpy(bb.scores).to(dev)
            d["done"] = torch.from_numpy(bb.done).to(dev)
            d["lens"] = torch.from_numpy(bb.lens).to(dev)
            pool.append(d)
            continue
        else:  # 5: the full rows, bf16; each rank keeps its own columns
            import sharded

            off, w = sharded.shard_bounds(V, n_ranks)[rank] if n_ranks > 1 else (0, V)
            full = (torch.randn((B, V), generator=gen, device=dev, dtype=torch.float32) * 4.0).to(torch.bfloat16)
            d["logits"] = full[:, off:off + w].contiguous()
            del full
            r = np.random.Generator(np.random.PCG64(5000 + i))
            from rlsampler import ROW_PARAMS_DTYPE

            p = np.zeros(B, ROW_PARAMS_DTYPE)
            p["temperature"] = 0.8
            p["top_k"] = 64
            p["top_p"] = 0.95
            p["repeat_penalty"] = 1.2
            hist = r.integers(0, V, (B, H)).astype(np.int32)
            u = workloads.uniforms(5, i, B)
        d["params"] = rlsampler.params_tensor(p, dev)
        d["u"] = torch.from_numpy(np.ascontiguousarray(u)).to(dev)
        if hist is not None:
            d["hist"] = torch.from_numpy(np.ascontiguousarray(hist)).to(dev)
            d["hl"] = torch.full((B,), hist.shape[1], dtype=torch.int32, device=dev)
        pool.append(d)
    return pool


# ---------------------------------------------------------------------------
# CPU legs: the oracle (a C++ restatement of src/decoder.rs; the Rust
# reference cannot be built here) on this host's cores
# ---------------------------------------------------------------------------
def _host_step(d):
    """A pool step's inputs on the host, in the oracle's layout."""
    B = d["logits"].shape[0]
    lg = d["logits"].float().cpu().numpy()
    from rlsampler import ROW_PARAMS_DTYPE

    p = d["params"].cpu().numpy().view(ROW_PARAMS_DTYPE)
    hist = d["hist"].cpu().numpy() if "hist" in d else None
    hl = d["hl"].cpu().numpy() if "hl" in d else None
    mask = d["mask"].cpu().numpy().view(np.uint32) if "mask" in d else None
    return lg, p, d["u"].cpu().numpy(), hist, hl, mask, B


def _oracle_step(step, nthreads):
    import oracle

    lg, p, u, hist, hl, mask, B = step
    tok, prob, bad = oracle.spec_sample_batch(lg, hist, hl, mask, p, u, nthreads=nthreads)
    return tok, prob


def cpu_baseline(cfg, host_steps, gpu_tokens, seconds=5.0):
    """The oracle timed over a bounded sample of the same steps, on one
    core and on all cores; its tokens are compared with the device's for
    the same steps (parity counter)."""
    nall = os.cpu_count() or 1
    unit_per_step = CONFIGS[cfg]["B"]
    out = {}
    parity = None
    for label, nth in (("1core", 1), ("all", nall)):
        elapsed, steps = 0.0, 0
        toks = []
        while elapsed < seconds and steps < 100000:
            st = host_steps[steps % len(host_steps)]
            t0 = time.perf_counter()
            tok, _ = _oracle_step(st, nth)
            elapsed += time.perf_counter() - t0
            if steps < len(host_steps):
                toks.append(tok)
            steps += 1
        v = steps * unit_per_step / elapsed
        out[label] = dict(value=(1e6 / v if cfg == 1 else v), steps=steps, seconds=round(elapsed, 2), threads=nth)
        if parity is None and gpu_tokens is not None:
            n = sum(len(t) for t in toks)
            eq = sum(int((t == g).sum()) for t, g in zip(toks, gpu_tokens))
            parity = {"rows_checked": n, "tokens_equal": eq,
                      "note": "device tokens of timed steps vs the oracle on the same inputs; rows may differ only "
                              "where a draw or cutoff is within 1e-6 of a CDF boundary"}
    c = CONFIGS[cfg]
    line = {"value": out["all"]["value"], "unit": c["unit"], "cores": nall, "kind": "port",
            "cpu_model": cpu_model(), "one_core": out["1core"]["value"], "all_cores": out["all"]["value"],
            "sample": f"{out['all']['steps']} steps of the same workload on {nall} threads "
                      f"({out['all']['seconds']} s) and {out['1core']['steps']} on one thread "
                      f"({out['1core']['seconds']} s), cycling over {len(host_steps)} distinct steps"}
    return line, parity


def run_reference(args, rank, world):
    """--impl reference: the CPU sampler (the oracle port of src/decoder.rs;
    the Rust crate cannot be built here) on this host's cores, on whole
    distinct batches of the same configuration. Rank 0 only."""
    c = CONFIGS[args.config]
    line = {"impl": "reference", "metric": c["metric"], "unit": c["unit"], "higher_is_better": c["higher"]}
    if rank != 0:
        return
    import oracle
    import workloads

    nthreads = os.cpu_count() or 1
    cfg = args.config
    B = c["B"]

    if cfg == 6:
        # hidden states and the random-init weight as bf16 values held in f32
        # (the reference dequantizes its weights to f32, src/model.rs:237)
        r = np.random.Generator(np.random.PCG64(6000))
        HID = c["HID"]

        def bf16_round(a):
            u = a.view(np.uint32)
            return ((u + 0x7FFF + ((u >> 16) & 1)) & 0xFFFF0000).view(np.float32)

        weight = bf16_round(r.standard_normal((c["V"], HID), dtype=np.float32) * np.float32(HID ** -0.5 * 3.0))

    def batch(i):
        if cfg == 6:
            rb = np.random.Generator(np.random.PCG64(6100 + i))
            p, hist, u = config2_params(600 + i, B, c["V"], c["H"])
            return dict(hidden=bf16_round(rb.standard_normal((B, c["HID"]), dtype=np.float32)), params=p, hist=hist,
                        hl=np.full(B, c["H"], np.int32), u=u)
        if cfg == 1:
            b = workloads.config1(i)
        elif cfg == 2:
            b = workloads.config2(i)
        elif cfg == 3:
            b = workloads.config3(i)
        elif cfg == 5:
            b = workloads.config5_rows(i, rows=list(range(0, 1024, 16)))
        else:
            return workloads.config4(i)
        return b

    steps = [batch(i) for i in range(min(args.steps, 4))]

    def run(b):
        if cfg == 6:
            lg = oracle.matmul_vec(b["hidden"], weight, nthreads=nthreads)
            oracle.spec_sample_batch(lg, b["hist"], b["hl"], None, b["params"], b["u"], nthreads=nthreads)
            return B
        if cfg == 4:
            oracle.beam_step(b.logits, b.items, b.beams, b.scores, b.done, b.lens, b.alpha, b.eos, 1, 2 * b.beams)
            return b.items * b.beams
        hl = b.hist_len
        oracle.spec_sample_batch(b.logits, b.hist, hl, b.mask, b.params, b.uniforms, nthreads=nthreads)
        return b.logits.shape[0]

    for i in range(min(args.warmup, 3)):
        run(steps[i % len(steps)])
    # whole steps until K are done or the time budget runs out (the line
    # reports the steps actually timed)
    units, done = 0, 0
    t0 = time.perf_counter()
    while done < args.steps:
        units += run(steps[done % len(steps)])
        done += 1
        if time.perf_counter() - t0 > args.ref_seconds:
            break
    dt = time.perf_counter() - t0
    v = units / dt
    value = 1e6 / v if cfg == 1 else v
    rows = (steps[0].items * steps[0].beams) if cfg == 4 else (B if cfg == 6 else steps[0].logits.shape[0])
    line.update({
        "value": value, "n_gpus": args.gpus, "steps": done, "steps_requested": args.steps, "warmup": args.warmup,
        "ms_per_step": dt / done * 1e3, "scaling": "weak" if cfg != 5 else "strong", "vs_baseline": None,
        "dtype": "bf16" if cfg in (5, 6) else "f32", "data": "synthetic",
        "config": {"workload": c["workload"], "rows_per_step": rows, "vocab": c["V"],
                   "distinct_steps": len(steps), "same_config": cfg != 5},
        "cpu_baseline": {"value": value, "unit": c["unit"], "cores": nthreads, "kind": "port", "cpu_model": cpu_model(),
                         "sample": f"{done} steps of {rows} rows (whole batches, {len(steps)} distinct), "
                                   f"{nthreads} threads, {dt:.1f} s"},
        "e2e": {"value": value, "unit": c["unit"], "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    })
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------------------
# Device legs
# ---------------------------------------------------------------------------
def timed_loop(step_fn, steps, warmup, stream, world, dev):
    import torch
    import torch.distributed as dist

    for i in range(warmup):
        step_fn(i)
    torch.cuda.synchronize()
    clk = ClockSampler(dev.index)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    clk.start()
    ev0 = torch.cuda.Event(enable_timing=True)
    ev1 = torch.cuda.Event(enable_timing=True)
    ev0.record(stream)
    for i in range(steps):
        step_fn(i)
    ev1.record(stream)
    torch.cuda.synchronize()
    clocks = clk.stop()
    ms = ev0.elapsed_time(ev1)
    if world > 1:
        t = torch.tensor([ms], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
        dist.barrier()
    return ms / steps, clocks


def shard_step_line(steps, warmup, dev, rank, world, stream):
    """The config-5 step (vocabulary split across the ranks, one NCCL
    all-gather inside rl_sample_sharded) at this N: returned on rank 0."""
    import torch

    import rlsampler
    import sharded

    c = CONFIGS[5]
    B, V = c["B"], c["V"]
    pool = make_pool(5, dev, rank, world, count=2)
    tok = torch.empty(B, dtype=torch.int32, device=dev)
    prob = torch.empty(B, dtype=torch.float32, device=dev)
    st = torch.empty(B, dtype=torch.int32, device=dev)
    if world > 1:
        ss = sharded.ShardedSampler(V, max_batch=B, device=dev, max_history=c["H"])
        fn = lambda i: ss.sample(pool[i % 2]["logits"], pool[i % 2]["params"], pool[i % 2]["u"], pool[i % 2]["hist"],
                                 pool[i % 2]["hl"], out_tok=tok, out_prob=prob, row_status=st, stream=stream)
    else:
        ss = rlsampler.Sampler(dev.index, max_batch=B, max_vocab=V, max_history=c["H"])
        fn = lambda i: ss.sample(pool[i % 2]["logits"], pool[i % 2]["params"], pool[i % 2]["u"], pool[i % 2]["hist"],
                                 pool[i % 2]["hl"], None, tok, prob, st, stream=stream)
    ms, _ = timed_loop(fn, steps, warmup, stream, world, dev)
    bad = int((st != 0).sum().item())
    ss.close()
    return {"metric": c["metric"], "value": B * steps / (ms * steps / 1e3), "unit": c["unit"], "ms_per_step": ms,
            "ranks": world, "scaling": "strong", "dtype": "bf16", "rows_not_ok": bad,
            "exchange": "one ncclAllGather of 1056 B per row and rank inside rl_sample_sharded" if world > 1
            else "one piece (rl_sample_batch)",
            "algorithmic_bytes_per_gpu": algorithmic_bytes(5, world)}


def gbnf_line(s, dev, stream, steps=30):
    """Config 3 with a real grammar: 64 sequences constrained by the JSON
    grammar (GBNF) over a 32,000-token synthetic vocabulary. A step: the
    allowed rows on the host (rl_gbnf_mask_batch, all host threads), their
    copy to the device, the masked batched sampler, the tokens back, and each
    token accepted into its sequence's state (a finished sequence restarts)."""
    import statistics

    import torch

    import grammar
    import rlsampler
    import workloads

    toks = workloads.json_vocab(32000)
    V = len(toks)
    eos = V - 1
    g = grammar.Gbnf(workloads.GBNF_JSON, toks, eos_id=eos)
    B = 64
    rng = np.random.default_rng(33)
    states = [g.new_state() for _ in range(B)]
    p = np.zeros(B, rlsampler.ROW_PARAMS_DTYPE)
    p["temperature"] = 0.8
    p["top_k"] = 50
    p["top_p"] = 0.95
    p["repeat_penalty"] = 1.0
    pd = rlsampler.params_tensor(p, dev)
    gen = torch.Generator(device=dev)
    gen.manual_seed(3300)
    logits = [torch.randn((B, V), generator=gen, device=dev) * 3.0 for _ in range(4)]
    u = torch.from_numpy(rng.random((steps + 3, B)).astype(np.float32)).to(dev)
    hmask = torch.empty((B, g.words), dtype=torch.int32, pin_memory=True)
    hrows = hmask.numpy().view(np.uint32)
    dmask = torch.empty((B, g.words), dtype=torch.int32, device=dev)
    tok = torch.empty(B, dtype=torch.int32, device=dev)
    prob = torch.empty(B, dtype=torch.float32, device=dev)
    st = torch.empty(B, dtype=torch.int32, device=dev)
    htok = torch.empty(B, dtype=torch.int32, pin_memory=True)
    nthreads = os.cpu_count() or 1
    t_mask, t_dev, t_acc, allowed, finished = [], [], [], [], 0
    for i in range(steps + 3):
        t0 = time.perf_counter()
        _, n = g.mask_batch(states, out=hrows, nthreads=nthreads)
        t1 = time.perf_counter()
        dmask.copy_(hmask, non_blocking=True)
        s.sample(logits[i % 4], pd, u[i], None, None, dmask, tok, prob, st, stream=stream)
        htok.copy_(tok, non_blocking=True)
        stream.synchronize()
        t2 = time.perf_counter()
        toks_np = htok.numpy()
        g.accept_batch(states, toks_np, nthreads=nthreads)
        for b in np.flatnonzero(toks_np == eos).tolist():
            states[b] = g.new_state()
            finished += 1
        t3 = time.perf_counter()
        if i >= 3:
            t_mask.append(t1 - t0)
            t_dev.append(t2 - t1)
            t_acc.append(t3 - t2)
            allowed += n.tolist()
    step = statistics.median([a + b + c for a, b, c in zip(t_mask, t_dev, t_acc)])
    return {"value": B / step, "unit": "tokens/s", "ms_per_step": step * 1e3,
            "mask_ms": statistics.median(t_mask) * 1e3, "device_ms": statistics.median(t_dev) * 1e3,
            "accept_ms": statistics.median(t_acc) * 1e3, "host_threads": nthreads,
            "allowed_tokens_median": int(statistics.median(allowed)), "allowed_tokens_max": int(max(allowed)),
            "documents_finished": finished, "batch": B, "vocab": V, "steps": steps,
            "path": "rl_gbnf_mask_batch (host) -> mask H2D -> rl_sample_batch with masks -> tokens D2H -> "
                    "rl_gbnf_accept_batch; medians over the steps"}


def lmhead_line(args, dev, rank, world, stream):
    """Config 6: hidden states -> tokens. The LM head (src/model.rs:236-262)
    as one tcgen05 GEMM (rl_lmhead_sample: bf16 weight [V, 4096] resident in
    HBM, f32 logits into the handle's staging buffer) and the batched sampler
    on config-2 sampling parameters; plus the fused greedy path (no logits
    written) and single-row decode."""
    import torch

    import rlsampler

    c = CONFIGS[6]
    B, V, H, HID = c["B"], c["V"], c["H"], c["HID"]
    gen = torch.Generator(device=dev)
    gen.manual_seed(6000 + 7919 * rank)
    weight = (torch.randn((V, HID), generator=gen, device=dev) * HID ** -0.5 * 3.0).to(torch.bfloat16)
    pool = []
    for i in range(POOL):
        d = {"hidden": torch.randn((B, HID), generator=gen, device=dev).to(torch.bfloat16)}
        p, hist, u = config2_params(600 + i + 100 * rank, B, V, H)
        d["params"] = rlsampler.params_tensor(p, dev)
        d["u"] = torch.from_numpy(np.ascontiguousarray(u)).to(dev)
        d["hist"] = torch.from_numpy(np.ascontiguousarray(hist)).to(dev)
        d["hl"] = torch.full((B,), H, dtype=torch.int32, device=dev)
        pool.append(d)
    s = rlsampler.Sampler(dev.index, max_batch=B, max_vocab=V, max_history=H)
    tok = torch.empty(B, dtype=torch.int32, device=dev)
    prob = torch.empty(B, dtype=torch.float32, device=dev)
    st = torch.empty(B, dtype=torch.int32, device=dev)

    def step(i):
        d = pool[i % POOL]
        s.lmhead_sample(d["hidden"], weight, d["params"], d["u"], d["hist"], d["hl"], tok, prob, st, stream=stream)

    ms, clocks = timed_loop(step, args.steps, args.warmup, stream, world, dev)
    bad = int((st != 0).sum().item())

    def ev_loop(fn, n, warm=3):
        for i in range(warm):
            fn(i)
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for i in range(n):
            fn(i)
        e1.record(stream)
        torch.cuda.synchronize()
        return e0.elapsed_time(e1) / n

    logits = torch.empty((B, V), dtype=torch.float32, device=dev)
    gemm_ms = ev_loop(lambda i: s.lmhead_logits(pool[i % POOL]["hidden"], weight, out=logits, stream=stream), 20)
    greedy_ms = ev_loop(lambda i: s.lmhead_greedy(pool[i % POOL]["hidden"], weight, stream=stream), 20)
    h1 = pool[0]["hidden"][:1]
    decode_ms = ev_loop(lambda i: s.lmhead_greedy(h1, weight, stream=stream), 20)
    flops = 2.0 * B * HID * V
    w_bytes = V * HID * 2
    if rank != 0:
        s.close()
        return None
    peaks = {}
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            peaks = json.load(f)
    except Exception:
        pass
    tf_peak = float(peaks.get("bf16_tflops", 1590.0))
    hbm_peak = float(peaks.get("hbm_gbs", 6650.0))
    achieved = flops / (gemm_ms * 1e-3) / 1e12
    traffic = committed_traffic().get("lmhead_kernel_b256_h4096_v128256")

    # end to end through the C ABI: pinned host hidden states in, tokens out
    # (the weight is resident, as in a serving engine)
    hh = torch.empty((B, HID), dtype=torch.bfloat16, pin_memory=True)
    hh.copy_(pool[0]["hidden"].cpu())
    htok = torch.empty(B, dtype=torch.int32, pin_memory=True)
    dh = torch.empty((B, HID), dtype=torch.bfloat16, device=dev)
    d0 = pool[0]

    def e2e_step():
        dh.copy_(hh, non_blocking=True)
        s.lmhead_sample(dh, weight, d0["params"], d0["u"], d0["hist"], d0["hl"], tok, prob, st, stream=stream)
        htok.copy_(tok, non_blocking=True)
        stream.synchronize()

    for _ in range(3):
        e2e_step()
    t0 = time.perf_counter()
    ne = max(args.e2e_steps, 10)
    for _ in range(ne):
        e2e_step()
    e2e_s = (time.perf_counter() - t0) / ne
    hbm_bytes = w_bytes + B * HID * 2 + B * V * 4
    line = {
        "metric": c["metric"], "value": world * B / (ms / 1e3), "unit": c["unit"], "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "bf16", "data": "synthetic (seeded hidden states, random-init bf16 weight)",
        "config": {"workload": c["workload"], "global_batch": B * world, "per_gpu_batch": B, "hidden": HID, "vocab": V,
                   "history": H, "parallelism": f"rows{world}",
                   "l2": "the 1.05 GB weight (larger than L2) streams from HBM every step"},
        "roofline": {"bound": "tensor", "achieved": achieved, "peak": tf_peak, "unit": "TFLOP/s",
                     "frac": achieved / tf_peak, "peak_kind": "measured (burst)" if peaks else "fallback",
                     "kernel": "lmhead_kernel (tcgen05 GEMM, logits written in f32), CUDA events around 20 launches",
                     "kernel_ms": gemm_ms, "flops_per_launch": flops,
                     "hbm_view": {"bytes": hbm_bytes, "gbs": hbm_bytes / (gemm_ms * 1e-3) / 1e9, "peak": hbm_peak},
                     "traffic": traffic,
                     "traffic_source": "profiles/traffic.json (ncu dram__bytes of one launch)" if traffic else None},
        "kernel_ms": {"lmhead_kernel": gemm_ms, "sampler (step - GEMM)": ms - gemm_ms},
        "greedy_fused": {"value": B / (greedy_ms / 1e3), "unit": "tokens/s", "ms_per_step": greedy_ms,
                         "path": "rl_lmhead_greedy: argmax in the GEMM epilogue, logits never written"},
        "decode_b1": {"us_per_token": decode_ms * 1e3, "weight_gbs": w_bytes / (decode_ms * 1e-3) / 1e9,
                      "frac_of_hbm_peak": w_bytes / (decode_ms * 1e-3) / 1e9 / hbm_peak,
                      "path": "rl_lmhead_greedy at B=1 (weight-streaming GEMV on the tensor cores)"},
        "gpu_launches": 4 * args.steps,
        "rows_not_ok": bad,
        "e2e": {"value": B / e2e_s, "unit": "tokens/s", "h2d_bytes_per_step": B * HID * 2, "d2h_bytes_per_step": B * 4,
                "ms_per_step": e2e_s * 1e3,
                "path": "pinned hidden states -> device, rl_lmhead_sample, tokens -> pinned host, sync per step"},
        "clocks": clocks,
    }
    if not args.no_cpu_baseline and world == 1:
        import oracle
        from rlsampler import ROW_PARAMS_DTYPE

        x = pool[0]["hidden"].float().cpu().numpy()
        w = weight.float().cpu().numpy()
        s.lmhead_logits(pool[0]["hidden"], weight, out=logits, stream=stream)
        torch.cuda.synchronize()
        lg_dev = logits.cpu().numpy()
        p0 = pool[0]["params"].cpu().numpy().view(ROW_PARAMS_DTYPE)
        hist0, hl0, u0 = pool[0]["hist"].cpu().numpy(), pool[0]["hl"].cpu().numpy(), pool[0]["u"].cpu().numpy()
        out = {}
        nall = os.cpu_count() or 1
        ref = None
        for label, nth, rows in (("1core", 1, 2), ("all", nall, nall)):
            rows = min(rows, B)
            t0 = time.perf_counter()
            lg = oracle.matmul_vec(x[:rows], w, nthreads=nth)
            oracle.spec_sample_batch(lg, hist0[:rows], hl0[:rows], None, p0[:rows], u0[:rows], nthreads=nth)
            dt = time.perf_counter() - t0
            out[label] = {"value": rows / dt, "rows": rows, "seconds": dt, "threads": nth}
            ref = lg
        n = ref.shape[0]
        bound = HID * 2.0 ** -21 * (np.abs(x[:n]).astype(np.float64) @ np.abs(w).astype(np.float64).T)
        err = np.abs(lg_dev[:n].astype(np.float64) - ref.astype(np.float64))
        dtok, _, _ = oracle.spec_sample_batch(lg_dev[:n], hist0[:n], hl0[:n], None, p0[:n], u0[:n], nthreads=nall)
        s.lmhead_sample(pool[0]["hidden"], weight, pool[0]["params"], pool[0]["u"], pool[0]["hist"], pool[0]["hl"],
                        tok, prob, st, stream=stream)
        torch.cuda.synchronize()
        line["cpu_baseline"] = {"value": out["1core"]["value"], "unit": "tokens/s", "cores": 1, "kind": "port",
                                "all_cores": out["all"], "cpu_model": cpu_model(),
                                "sample": f"{out['1core']['rows']} rows (matmul_vec + spec sampler, one thread); "
                                          f"{out['all']['rows']} rows on {nall} threads"}
        line["parity_sample"] = {"rows": int(n), "logits_max_abs_err_vs_oracle": float(err.max()),
                                 "logits_within_f32_sum_bound": bool((err <= bound).all()),
                                 "tokens_equal_oracle_sampler_on_device_logits":
                                     int((tok.cpu().numpy()[:n] == dtok).sum())}
    s.close()
    return line


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--config", type=int, default=2, choices=[1, 2, 3, 4, 5, 6])
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=None)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--e2e-steps", type=int, default=20)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-shards", action="store_true", help="config 2: leave out the config-5 step")
    ap.add_argument("--ref-seconds", type=float, default=120.0, help="--impl reference: time budget of the loop")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)
    if args.steps is None:
        args.steps = {1: 2000, 2: 200, 3: 500, 4: 200, 5: 50, 6: 100}[args.config]

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
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
    cfg = args.config
    c = CONFIGS[cfg]
    B, V, H = c["B"], c["V"], c["H"]
    stream = torch.cuda.current_stream(dev)
    if cfg == 6:
        line = lmhead_line(args, dev, rank, world, stream)
        if rank == 0:
            print(json.dumps(line), flush=True)
        if world > 1:
            dist.barrier()
            dist.destroy_process_group()
        return
    pool = make_pool(cfg, dev, rank, world) if cfg != 5 else None

    out_tok = torch.empty(B, dtype=torch.int32, device=dev)
    out_prob = torch.empty(B, dtype=torch.float32, device=dev)
    row_st = torch.empty(B, dtype=torch.int32, device=dev)
    kernel_ms = None
    launches_per_step = 2
    s = None
    if cfg in (1, 2, 3):
        s = rlsampler.Sampler(local, max_batch=B, max_vocab=V, max_history=max(H, 1))

        def step(i):
            d = pool[i % POOL]
            s.sample(d["logits"], d["params"], d["u"], d.get("hist"), d.get("hl"), d.get("mask"), out_tok, out_prob,
                     row_st, stream=stream)

        ms, clocks = timed_loop(step, args.steps, args.warmup, stream, world, dev)
        # per-kernel device times over a few extra (untimed) steps
        s.set_debug(rlsampler.RL_DEBUG_TIMING)
        per = []
        for i in range(8):
            step(i)
            per.append(s.kernel_times())
        s.set_debug(0)
        kernel_ms = [float(np.mean([p[k] for p in per])) for k in range(len(per[0]))]
        launches_per_step = len(kernel_ms)  # short rows: one kernel; long rows: streaming + finish
        units = B
    elif cfg == 4:
        s = rlsampler.Sampler(local, max_batch=B, max_vocab=V, max_history=1)
        launches_per_step = 4  # params fill, streaming, finish, beam combine

        def step(i):
            d = pool[i % POOL]
            s.beam_step(d["logits"], 16, 8, d["scores"], d["done"], d["lens"], 1.0, 2, 1, 16, stream=stream)

        ms, clocks = timed_loop(step, args.steps, args.warmup, stream, world, dev)
        units = 128
        row_st.zero_()
    else:
        line5 = shard_step_line(args.steps, args.warmup, dev, rank, world, stream)
        ms, clocks, units = line5["ms_per_step"], None, B
        launches_per_step = 3 if world > 1 else 2
    bad = int((row_st != 0).sum().item()) if cfg != 5 else line5["rows_not_ok"]
    value_units_per_s = (world if cfg != 5 else 1) * units / (ms / 1e3)

    # ---- end to end through the host-buffer entry point (pinned memory) ----
    e2e = None
    if cfg in (2, 3):
        d = pool[0]
        h_logits = torch.empty((B, V), dtype=torch.float32, pin_memory=True)
        h_logits.copy_(d["logits"].cpu())
        h_params = d["params"].cpu().numpy().copy()
        h_u = d["u"].cpu().numpy().copy()
        h_hist = d["hist"].cpu().numpy().copy() if "hist" in d else None
        h_hl = d["hl"].cpu().numpy().copy() if "hl" in d else None
        h_mask = d["mask"].cpu().numpy().copy() if "mask" in d else None
        h_tok = torch.empty(B, dtype=torch.int32, pin_memory=True)
        h_prob = torch.empty(B, dtype=torch.float32, pin_memory=True)
        cp = lambda a: a.ctypes.data_as(ctypes.c_void_p) if a is not None else None
        tp = lambda t: ctypes.c_void_p(t.data_ptr())

        # the call's arguments bound once (the same pinned buffers every step)
        host_args = (s.h, tp(h_logits), B, V, cp(h_hist), cp(h_hl), H, cp(h_mask),
                     h_mask.shape[1] if h_mask is not None else 0, cp(h_params), cp(h_u), tp(h_tok), tp(h_prob))
        host_call = rlsampler.lib().rl_sample_host

        def e2e_step():
            rlsampler.check(host_call(*host_args), "rl_sample_host")

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
        h2d = B * V * 4 + (B * H * 4 + B * 4 if H else 0) + B * 24 + B * 4 + (h_mask.nbytes if h_mask is not None else 0)
        copy_ms = (B * V * 4) / 40e9 * 1e3
        e2e = {"value": world * B * args.e2e_steps / e2e_s, "unit": "tokens/s", "h2d_bytes_per_step": h2d,
               "d2h_bytes_per_step": B * 8, "ms_per_step": e2e_s / args.e2e_steps * 1e3,
               "device_ms_per_step": ms,
               "path": "rl_sample_host (pinned host buffers, H2D + kernels + D2H + sync per step)"}
    elif cfg == 1:
        # one host call per token through the host-buffer entry point
        d = pool[0]
        h = {k: (d[k].cpu().numpy().copy() if k != "logits" else None) for k in ("params", "u", "hist", "hl")}
        h_logits = torch.empty((1, V), dtype=torch.float32, pin_memory=True)
        h_logits.copy_(d["logits"].cpu())
        h_tok = torch.empty(1, dtype=torch.int32, pin_memory=True)
        h_prob = torch.empty(1, dtype=torch.float32, pin_memory=True)
        cp = lambda a: a.ctypes.data_as(ctypes.c_void_p)
        tp = lambda t: ctypes.c_void_p(t.data_ptr())
        # the call's arguments bound once (the same buffers every token)
        host_args = (s.h, tp(h_logits), 1, V, cp(h["hist"]), cp(h["hl"]), H, None, 0, cp(h["params"]), cp(h["u"]),
                     tp(h_tok), tp(h_prob))
        host_call = rlsampler.lib().rl_sample_host
        fn = lambda: rlsampler.check(host_call(*host_args), "rl_sample_host")
        for _ in range(10):
            fn()
        t0 = time.perf_counter()
        n = 500
        for _ in range(n):
            fn()
        e2e_us = (time.perf_counter() - t0) / n * 1e6
        e2e = {"value": e2e_us, "unit": "us/token", "h2d_bytes_per_step": V * 4 + H * 4 + 4 + 24 + 4,
               "d2h_bytes_per_step": 8, "path": "rl_sample_host, one call per token (host logits in, token out)"}

    gbnf = gbnf_line(s, dev, stream) if cfg == 3 and world == 1 else None

    shards = None
    if cfg == 2 and not args.no_shards:
        shards = shard_step_line(20, 3, dev, rank, world, stream)

    if rank == 0:
        peak, peak_kind = measured_peak()
        alg = algorithmic_bytes(cfg, world)
        step_gbs = alg / (ms * 1e-3) / 1e9
        if kernel_ms:
            dom_ms = kernel_ms[0]
            achieved = alg / (dom_ms * 1e-3) / 1e9
            kern = ("spec_pipe_kernel (the streaming kernel: reads every logit once), CUDA events around it"
                    if len(kernel_ms) > 1 else
                    "small_rows_kernel (one CTA per row, the row in shared memory), CUDA events around it")
        else:
            dom_ms = ms
            achieved = step_gbs
            kern = "the whole step (its kernels timed together)"
        # config 1 samples one token per step and rank: microseconds per token
        value = ms * 1e3 if cfg == 1 else value_units_per_s
        traffic = {2: committed_traffic().get("spec_pipe_kernel_f32_config2"),
                   1: committed_traffic().get("small_rows_kernel_f32_config1"),
                   }.get(cfg)
        line = {
            "metric": c["metric"], "value": value, "unit": c["unit"], "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": c["higher"],
            "scaling": "strong" if cfg == 5 else "weak", "vs_baseline": None, "dtype": "bf16" if cfg == 5 else "f32",
            "data": "synthetic (seeded; the reference publishes no data set)",
            "config": {"workload": c["workload"], "global_batch": B * (world if cfg != 5 else 1), "per_gpu_batch": B,
                       "vocab": V, "history": H, "parallelism": (f"vocab{world}" if cfg == 5 else f"rows{world}"),
                       "l2": ("inputs larger than L2: 8 distinct 256x128256 f32 step buffers cycled" if cfg == 2 else
                              f"{POOL} distinct step buffers cycled (a step's inputs fit in L2)")},
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak,
                         "peak_kind": peak_kind, "kernel": kern, "algorithmic_bytes_per_launch": alg,
                         "kernel_ms": dom_ms, "step_gbs": step_gbs, "step_frac": step_gbs / peak, "traffic": traffic,
                         "traffic_source": "profiles/traffic.json (ncu dram__bytes of one launch of the kernel above)" if traffic else None},
            "kernel_ms": (({"spec_pipe_kernel": kernel_ms[0], "spec_finish_kernel": kernel_ms[1]}
                           if len(kernel_ms) > 1 else {"small_rows_kernel": kernel_ms[0]}) if kernel_ms else None),
            "gpu_launches": launches_per_step * args.steps,
            "rows_not_ok": bad,
            "e2e": e2e,
            "clocks": clocks,
        }
        if shards:
            line["vocab_shards"] = shards
        if gbnf:
            line["gbnf_json"] = gbnf
        if not args.no_cpu_baseline and world == 1 and cfg != 5:
            if cfg == 4:
                import oracle

                steps_h = [pool[i] for i in range(2)]
                t0 = time.perf_counter()
                n = 0
                while time.perf_counter() - t0 < 5.0:
                    d = steps_h[n % 2]
                    lg = d["logits"].cpu().numpy()
                    oracle.beam_step(lg, 16, 8, d["scores"].cpu().numpy(), d["done"].cpu().numpy(),
                                     d["lens"].cpu().numpy(), 1.0, 2, 1, 16)
                    n += 1
                dt = time.perf_counter() - t0
                line["cpu_baseline"] = {"value": n * 128 / dt, "unit": c["unit"], "cores": 1, "kind": "port",
                                        "cpu_model": cpu_model(), "sample": f"{n} beam steps, one thread, {dt:.1f} s"}
            else:
                host_steps = [_host_step(pool[i]) for i in range(2)]
                # the device's tokens for the same two steps
                gtoks = []
                for i in range(2):
                    d = pool[i]
                    s.sample(d["logits"], d["params"], d["u"], d.get("hist"), d.get("hl"), d.get("mask"), out_tok,
                             out_prob, row_st, stream=stream)
                    torch.cuda.synchronize()
                    gtoks.append(out_tok.cpu().numpy().copy())
                cb, parity = cpu_baseline(cfg, host_steps, gtoks)
                line["cpu_baseline"] = cb
                line["parity_sample"] = parity
        print(json.dumps(line), flush=True)
    if s is not None:
        s.close()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
