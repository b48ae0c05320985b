#!/usr/bin/env python
"""MoE-layer tokens/s on B200 for DiskMule's routed-expert path.

Default workload (N=1): the Qwen3.5-shaped MoE block of the benchmark table
(hidden 2048, 512 experts, top-10, intermediate 512, Q4_K gate/up, Q6_K down,
shared expert with a sigmoid gate), prefill of T=512 tokens per step. Weights
(1.06 GB) exceed the 126 MB L2, so every step streams them from HBM. Decode (T=1)
is reported beside it. One JSON line on rank 0.

  python bench.py [--gpus N --steps K --warmup W] [--impl reference]

`--impl reference` times the CPU restatement of the reference path (the oracle)
on this host's cores over a bounded token sample per step. Under torchrun each
rank runs an independent replica on its own GPU (the GGUF block does not shard);
the timed region is bracketed by barriers and the max over ranks is reported.
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
sys.path.insert(0, ROOT)


def parse_args():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=600)  # ~0.3 s timed: the clock sampler sees it
    p.add_argument("--warmup", type=int, default=5)
    p.add_argument("--impl", default="ours", choices=["ours", "reference"])
    p.add_argument("--config", default="qwen35")
    p.add_argument("--tokens", type=int, default=512)
    p.add_argument("--decode-steps", type=int, default=200)
    p.add_argument("--cpu-seconds", type=float, default=10.0)
    p.add_argument("--ep", action="store_true",
                   help="expert parallelism over the ranks (config 4: --config glm52 --tokens 8192 "
                        "tokens in total, split over the GPUs)")
    p.add_argument("--stack", action="store_true",
                   help="out-of-core decode (config 5): a stack of GLM-5.2 layers with experts in "
                        "pinned host memory and --slots HBM slots per layer; --steps decode steps")
    p.add_argument("--layers", type=int, default=8)
    p.add_argument("--slots", type=int, default=8)
    p.add_argument("--vocab", type=int, default=32768)
    p.add_argument("--pool-experts", type=int, default=0,
                   help="distinct expert blobs in host memory (0: every expert, if host memory "
                        "allows)")
    p.add_argument("--check-steps", type=int, default=16,
                   help="decode steps replayed on the CPU oracle (token parity, CPU baseline)")
    return p.parse_args()


CLOCK_QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
               "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
               "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
REASONS = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]


class ClockSampler:
    """nvidia-smi sampled every 200 ms while the timed region runs. Only one process
    samples (`active`): several nvidia-smi pollers slow the driver calls of paths that
    synchronise with the host every step. Entering waits `settle` seconds, so the timed
    region starts after nvidia-smi's own start-up."""

    def __init__(self, index: int, active: bool = True, settle: float = 1.5):
        self.index = index
        self.proc = None
        self.active = active
        self.settle = settle

    def __enter__(self):
        if not self.active:
            return self
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={CLOCK_QUERY}", "--format=csv,noheader,nounits",
                 "-lms", "200", "-i", str(self.index)],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
        if self.proc is not None and self.settle > 0:
            time.sleep(self.settle)
        return self

    def __exit__(self, *exc):
        self.out = ""
        if self.proc is not None:
            time.sleep(0.25)
            self.proc.terminate()
            try:
                self.out, _ = self.proc.communicate(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
                self.out, _ = self.proc.communicate()

    def summary(self):
        sm, mx, reasons = [], [], set()
        for line in (self.out or "").splitlines():
            f = [c.strip() for c in line.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx.append(float(f[2]))
            except ValueError:
                continue
            for name, flag in zip(REASONS, f[5:9]):
                if flag.lower().startswith("active"):
                    reasons.add(name)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": max(mx),
                "reasons": sorted(reasons), "samples": len(sm)}


def measured_peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        with open(path) as f:
            d = json.load(f)
        return d.get("hbm_gbs", 6650.0), "measured"
    return 6650.0, "fallback"


def measured_tensor_peak():
    """Dense bf16/fp16 TFLOP/s (burst: the stage is timed inside a short forward)."""
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        with open(path) as f:
            d = json.load(f)
        if "bf16_tflops" in d:
            return d["bf16_tflops"], "measured"
    return 1590.0, "fallback"


FORMAT_NAMES = {0: "F32", 1: "F16", 6: "Q5_0", 8: "Q8_0", 12: "Q4_K", 14: "Q6_K", 30: "BF16"}


def choose_roofline(kernel, flops, nbytes, ms, hbm, tensor, traffic):
    """Roofline of one stage: the tensor peak when its FLOP per byte is above the ridge
    (peak FLOP/s / peak bytes/s), else HBM. hbm = (GB/s, source), tensor = (TFLOP/s, source)."""
    (peak, peak_src), (tpeak, tpeak_src) = hbm, tensor
    intensity = flops / nbytes
    if intensity > tpeak * 1e12 / (peak * 1e9):
        achieved = flops / (ms / 1e3) / 1e12
        r = {"bound": "tensor", "achieved": achieved, "peak": tpeak, "unit": "TFLOP/s",
             "frac": achieved / tpeak, "traffic": traffic, "kernel": kernel,
             "algorithmic_flops": flops, "algorithmic_bytes": nbytes, "peak_source": tpeak_src,
             "note": "fp16 MMAs on hi + lo activation halves: the tensor pipe does twice "
                     "the algorithmic FLOPs"}
    else:
        achieved = nbytes / (ms / 1e3) / 1e9
        r = {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
             "frac": achieved / peak, "traffic": traffic, "kernel": kernel,
             "algorithmic_bytes": nbytes, "peak_source": peak_src}
    r["flop_per_byte"] = round(intensity, 1)
    return r


def stage_flops(sl, T):
    """Algorithmic FLOPs (2 per multiply-add) of the expert stages."""
    cfg = sl.cfg
    H, I, k = cfg["hidden"], cfg["intermediate"], cfg["top_k"]
    P = T * k + (T if cfg.get("shared") else 0)
    return {"expert_up": 2.0 * P * 2 * I * H, "expert_down": 2.0 * P * I * H}


def ncu_traffic(kernel: str, workload: str):
    """DRAM bytes per launch of `kernel` from the committed ncu summary, if any."""
    path = os.path.join(ROOT, "profiles", "ncu_traffic.json")
    if not os.path.exists(path):
        return None
    with open(path) as f:
        d = json.load(f)
    return d.get(f"{kernel}@{workload}")


# ---------------------------------------------------------------------------
# reference arm: the CPU restatement of the reference path (the oracle)
# ---------------------------------------------------------------------------

def cpu_tokens_per_second(cfg_name: str, seconds: float, threads: int, seed: int = 1,
                          sample: int | None = None):
    from diskmule_b200.synthetic import CONFIGS, SyntheticLayer, input_spec, layer_specs, vectors
    from oracle import oracle as O
    cfg = dict(CONFIGS[cfg_name])
    sl = SyntheticLayer(cfg_name, cfg, seed, None, layer_specs(cfg, seed), vectors(cfg, seed))
    w = sl.host_weights()
    fn = {"gemma4": O.gemma_moe, "qwen35": O.qwen_moe, "glm52": O.glm_moe}[cfg["family"]]
    n = sample or max(threads, 8)
    spec = input_spec(cfg, n, 21)
    raw = spec.host()
    x = raw.view(np.float32).reshape(n, -1)
    fn(w, x[:1], threads=threads)  # touch the weights once
    done, t0 = 0, time.perf_counter()
    while True:
        rc, _, _, _ = fn(w, x, threads=threads)
        assert rc == O.OK
        done += n
        el = time.perf_counter() - t0
        if el >= seconds:
            break
    return done / el, n, el


def run_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    threads = os.cpu_count() or 1
    per_step = []
    sample = max(threads, 8)
    for i in range(args.warmup + args.steps):
        tps, n, el = cpu_tokens_per_second(args.config, 0.0, threads, sample=sample)
        if i >= args.warmup:
            per_step.append(n / tps)
    total_tokens = sample * args.steps
    secs = sum(per_step)
    value = total_tokens / secs
    line = {
        "impl": "reference", "metric": f"MoE-layer tokens/s ({args.config}, CPU reference path)",
        "value": value, "unit": "tokens/s", "n_gpus": args.gpus, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": 1e3 * secs / args.steps, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": f"{args.config} MoE block, {sample}-token sample per step",
                   "parallelism": "cpu"},
        "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": threads, "kind": "port",
                         "sample": f"{sample} tokens per step of the {args.config} block "
                                   "(tokens are independent in the reference)"},
        "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    emit(line)


# ---------------------------------------------------------------------------
# our arm
# ---------------------------------------------------------------------------

def stage_bytes(sl, T, counts):
    """Algorithmic bytes per stage (weights once per distinct expert touched)."""
    cfg = sl.cfg
    H, I, E, k = cfg["hidden"], cfg["intermediate"], cfg["experts"], cfg["top_k"]
    sp = sl.specs
    active = int((counts > 0).sum())
    shared = 1 if cfg.get("shared") else 0
    P = T * k + shared * T
    xb = 2 if cfg["family"] == "glm52" else 4
    up_w = sp["gate"].expert_bytes + (sp["up"].expert_bytes if "up" in sp else 0)
    up = (active + shared) * up_w + T * H * xb + P * I * 4
    down = (active + shared) * sp["down"].expert_bytes + P * I * 4 + P * H * 4
    router = sp["router"].nbytes + T * H * xb + T * (E + 1) * 4
    return {"expert_up": up, "expert_down": down, "router": router}


def run_ours(args):
    import torch
    import torch.distributed as dist

    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    if world > 1:
        import datetime
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))

    def barrier():
        if world > 1:
            dist.barrier()

    def max_over_ranks(v):
        if world == 1:
            return v
        t = torch.tensor([v], dtype=torch.float64, device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    from diskmule_b200 import _native as N
    from diskmule_b200.moe import CudaContext
    from diskmule_b200.synthetic import build_layer, input_spec

    ctx = CudaContext(local)
    sl = build_layer(ctx, args.config, seed=1)
    cfg = sl.cfg
    T, H, k = args.tokens, cfg["hidden"], cfg["top_k"]
    xdt = torch.bfloat16 if cfg["family"] == "glm52" else torch.float32
    x = torch.empty((T, H), dtype=xdt, device="cuda")
    y = torch.empty((T, H), dtype=torch.float32, device="cuda")
    xs = input_spec(cfg, T, 21 + rank)
    xs.device_fill(x.data_ptr())
    ctx.synchronize()
    stream = torch.cuda.current_stream()
    sptr = stream.cuda_stream

    def step(tokens, xp, yp):
        sl.layer.forward(xp, yp, tokens, stream=sptr)

    # ---- prefill: the headline value ----
    for _ in range(args.warmup):
        step(T, x.data_ptr(), y.data_ptr())
    torch.cuda.synchronize()
    launches = sl.layer.last_launch_count()
    barrier()
    torch.cuda.synchronize()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local, active=rank == 0) as clk:
        barrier()  # rank 0 entered after the sampler settled
        torch.cuda.synchronize()
        start.record(stream)
        for _ in range(args.steps):
            step(T, x.data_ptr(), y.data_ptr())
        end.record(stream)
        torch.cuda.synchronize()
    barrier()
    ms = max_over_ranks(start.elapsed_time(end))
    value = world * T * args.steps / (ms / 1e3)

    # ---- per-stage times (same workload, profiled pass) for the roofline ----
    counts, _, _, _ = sl.layer.last_dispatch(T)
    sl.layer.set_profiling(True)
    totals = {}
    n_prof = min(args.steps, 50)
    for _ in range(n_prof):
        step(T, x.data_ptr(), y.data_ptr())
        for name, t in sl.layer.stage_times().items():
            totals[name] = totals.get(name, 0.0) + t
    sl.layer.set_profiling(False)
    avg = {n: v / n_prof for n, v in totals.items()}
    nbytes = stage_bytes(sl, T, counts)
    weight_gb = sum(sl.specs[n].expert_bytes for n in ("gate", "up", "down") if n in sl.specs) * \
        (cfg["experts"] + (1 if cfg.get("shared") else 0)) / 1e9
    dominant = max(("expert_up", "expert_down"), key=lambda n: avg[n])
    peak, peak_src = measured_peaks()
    tpeak, tpeak_src = measured_tensor_peak()
    nflops = stage_flops(sl, T)
    workload = f"{args.config}-T{T}"
    traffic = ncu_traffic(dominant, workload)
    roofline = choose_roofline(dominant, nflops[dominant], nbytes[dominant], avg[dominant],
                               (peak, peak_src), (tpeak, tpeak_src), traffic)
    roofline["stage_ms"] = {n: round(v, 4) for n, v in avg.items()}

    # ---- decode (T=1) ----
    # Distinct tokens, and L2 flushed (a 256 MB write) before every timed token, so each
    # token's router and expert weights come from HBM; tokens are timed one by one with
    # events on the launching stream and the flushes stay outside the timed spans.
    n_dec = 12  # forward() keeps up to 16 CUDA graphs keyed by buffers
    x1 = torch.empty((n_dec, H), dtype=xdt, device="cuda")
    input_spec(cfg, n_dec, 33 + rank).device_fill(x1.data_ptr())
    y1 = torch.empty((n_dec, H), dtype=torch.float32, device="cuda")
    flush = torch.empty(256 << 20, dtype=torch.uint8, device="cuda")
    xrow = x1.element_size() * H
    ctx.synchronize()

    def dec(i):
        j = i % n_dec
        step(1, x1.data_ptr() + j * xrow, y1.data_ptr() + j * H * 4)

    for i in range(args.warmup):
        dec(i)
    barrier()
    torch.cuda.synchronize()
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
          for _ in range(args.decode_steps)]
    for i in range(args.decode_steps):
        flush.fill_(i & 0xFF)
        ev[i][0].record(stream)
        dec(i)
        ev[i][1].record(stream)
    torch.cuda.synchronize()
    barrier()
    dms = max_over_ranks(sum(a.elapsed_time(b) for a, b in ev))
    decode_tps = world * args.decode_steps / (dms / 1e3)
    dec(0)
    c1, _, _, _ = sl.layer.last_dispatch(1)
    b1 = stage_bytes(sl, 1, c1)
    dec_bytes = b1["expert_up"] + b1["expert_down"] + b1["router"]
    sl.layer.set_profiling(True)
    dtot = {}
    for i in range(20):
        flush.fill_(i & 0xFF)
        dec(i)
        for name, t in sl.layer.stage_times().items():
            dtot[name] = dtot.get(name, 0.0) + t
    sl.layer.set_profiling(False)
    del flush
    dstage = {n: round(1e3 * v / 20, 2) for n, v in dtot.items()}
    up_bw = b1["expert_up"] / (dstage["expert_up"] * 1e-6) / 1e9 if dstage.get("expert_up") else 0
    dn_bw = b1["expert_down"] / (dstage["expert_down"] * 1e-6) / 1e9 if dstage.get("expert_down") else 0
    decode = {"tokens_per_s": decode_tps, "us_per_token": 1e3 * dms / args.decode_steps,
              "algorithmic_bytes_per_token": dec_bytes,
              "hbm_frac": dec_bytes / (dms / args.decode_steps / 1e3) / 1e9 / peak,
              "stage_us": dstage,
              "expert_up_hbm_frac": up_bw / peak, "expert_down_hbm_frac": dn_bw / peak}

    # ---- end to end through the public host API (pinned host buffers) ----
    xh = torch.empty((T, H), dtype=xdt, pin_memory=True)
    xh.copy_(x.cpu())
    xnp = xh.view(torch.int16).numpy() if xdt == torch.bfloat16 else xh.numpy()
    # page-locked outputs, as a host that keeps its buffers would pass
    out = (torch.empty((T, H), dtype=torch.float32, pin_memory=True).numpy(),
           torch.empty((T, k), dtype=torch.int32, pin_memory=True).numpy().view(np.uint32),
           torch.empty((T, k), dtype=torch.float32, pin_memory=True).numpy())
    for _ in range(2):
        sl.layer.forward_host(xnp, out=out)
    barrier()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        sl.layer.forward_host(xnp, out=out)
    el = max_over_ranks(time.perf_counter() - t0)
    e2e = {"value": world * T * args.steps / el, "unit": "tokens/s",
           "h2d_bytes_per_step": int(T * H * (2 if xdt == torch.bfloat16 else 4)),
           "d2h_bytes_per_step": int(T * H * 4 + T * k * 8)}

    line = None
    if rank == 0:
        cpu = None
        if world == 1:
            threads = os.cpu_count() or 1
            tps, n, secs = cpu_tokens_per_second(args.config, args.cpu_seconds, threads)
            cpu = {"value": tps, "unit": "tokens/s", "cores": threads, "kind": "port",
                   "sample": f"{n}-token batches of the {args.config} block for {secs:.1f} s"}
        line = {
            "metric": f"MoE-layer tokens/s ({args.config} prefill T={T})",
            "value": value, "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms / args.steps, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": {"workload": f"{args.config} MoE block, prefill T={T} per GPU",
                       "tokens_per_step": T, "hidden": H, "experts": cfg["experts"],
                       "top_k": k, "intermediate": cfg["intermediate"],
                       "formats": f"{FORMAT_NAMES.get(cfg['gate_type'], cfg['gate_type'])} gate/up, "
                                  f"{FORMAT_NAMES.get(cfg['down_type'], cfg['down_type'])} down",
                       "parallelism": f"replicas x{world}",
                       "l2": f"expert weights ({weight_gb:.2f} GB) larger than L2; no flush needed"},
            "roofline": roofline, "decode": decode, "e2e": e2e,
            "gpu_launches": launches * args.steps,
            "clocks": clk.summary(),
            "cpu_baseline": cpu,
        }
        emit(line)
    sl.close()
    ctx.close()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


# ---------------------------------------------------------------------------
# expert parallelism (config 4)
# ---------------------------------------------------------------------------

def cpu_glm_sample_tokens_per_second(cfg_name: str, sample: int, threads: int, seed: int = 1):
    """The oracle GLM block on `sample` tokens, with host weights for the experts those
    tokens select only (the full pool is tens of GB)."""
    from diskmule_b200 import _native as N
    from diskmule_b200.synthetic import CONFIGS, SyntheticLayer, input_spec, layer_specs, vectors
    from oracle import oracle as O
    cfg = dict(CONFIGS[cfg_name])
    specs = layer_specs(cfg, seed)
    sl = SyntheticLayer(cfg_name, cfg, seed, None, specs, vectors(cfg, seed))
    raw = input_spec(cfg, sample, 21).host()
    x = (raw.view(np.uint16).reshape(sample, -1).astype(np.uint32) << 16).view(np.float32)
    router = specs["router"].host()
    bias = specs["bias"].host().view(np.float32)
    chosen = set()
    for t in range(sample):
        _, lg = O.glm_matvec(N.BF16, cfg["experts"], cfg["hidden"], router, x[t], threads)
        _, idx, _ = O.glm_select(lg, bias, cfg["top_k"], cfg["n_groups"], cfg["topk_groups"],
                                 cfg["normalize"])
        chosen.update(int(i) for i in idx)
    w = sl.host_weights(sorted(chosen))
    t0 = time.perf_counter()
    rc, _, _, _ = O.glm_moe(w, x, threads=threads)
    assert rc == O.OK
    return sample / (time.perf_counter() - t0)


def run_ep(args):
    import datetime
    import torch
    import torch.distributed as dist

    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    if "MASTER_ADDR" not in os.environ:  # a single process: a one-rank group
        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ.setdefault("MASTER_PORT", "29533")
    dist.init_process_group("nccl", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=120),
                            device_id=torch.device("cuda", local))

    def max_over_ranks(v):
        t = torch.tensor([v], dtype=torch.float64, device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    from diskmule_b200.ep import ExpertParallel, cuda_backend_for
    from diskmule_b200.moe import CudaContext
    from diskmule_b200.synthetic import CONFIGS, build_layer, input_spec

    cfg = dict(CONFIGS[args.config])
    E, H, I, k = cfg["experts"], cfg["hidden"], cfg["intermediate"], cfg["top_k"]
    per = E // world
    T_total = args.tokens
    T = T_total // world
    ctx = CudaContext(local)
    sl = build_layer(ctx, args.config, seed=1, expert_range=(rank * per, per))
    xdt = torch.bfloat16 if cfg["family"] == "glm52" else torch.float32
    x = torch.empty((T, H), dtype=xdt, device="cuda")
    input_spec(cfg, T, 21 + rank).device_fill(x.data_ptr())
    ctx.synchronize()
    backend = cuda_backend_for(sl)
    ep = ExpertParallel(backend, E, k)
    stream = torch.cuda.current_stream()

    for _ in range(args.warmup):
        y = ep.forward(x)
    torch.cuda.synchronize()
    dist.barrier()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local, active=rank == 0) as clk:
        dist.barrier()  # rank 0 entered after the sampler settled
        torch.cuda.synchronize()
        start.record(stream)
        for _ in range(args.steps):
            y = ep.forward(x)
        end.record(stream)
        torch.cuda.synchronize()
    dist.barrier()
    ms = max_over_ranks(start.elapsed_time(end))
    value = T_total * args.steps / (ms / 1e3)
    # launches of one step (route + received rows + shared rows + combine)
    launches = 0
    T_probe = T
    ep.forward(x)
    launches = sl.layer.last_launch_count()  # combine; the others are counted below
    routed = backend.route(x)
    launches += sl.layer.last_launch_count()
    ids = torch.zeros((T_probe,), dtype=torch.int32, device="cuda")
    backend.expert_rows(x if cfg["family"] != "gemma4" else routed.expert_in, ids)
    launches += 2 * sl.layer.last_launch_count()

    # e2e: host input copied in and output copied back every step
    xh = torch.empty((T, H), dtype=xdt, pin_memory=True)
    xh.copy_(x.cpu())
    yh = torch.empty((T, H), dtype=torch.float32, pin_memory=True)
    torch.cuda.synchronize()
    dist.barrier()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        xd = xh.to("cuda", non_blocking=True)
        yh.copy_(ep.forward(xd), non_blocking=True)
        torch.cuda.synchronize()
    el = max_over_ranks(time.perf_counter() - t0)

    # tensor roofline: useful FLOPs per GPU per step / time
    shared = 1 if cfg.get("shared") else 0
    flops = T * (k + shared) * 3 * 2 * H * I
    peaks = {}
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        with open(path) as f:
            peaks = json.load(f)
    peak = peaks.get("bf16_tflops_sustained") or peaks.get("bf16_tflops") or 1590.0
    achieved = flops / (ms / args.steps / 1e3) / 1e12
    if rank == 0:
        cpu = None
        if world == 1 and cfg["family"] == "glm52":
            threads = os.cpu_count() or 1
            sample = 8
            cpu = {"value": cpu_glm_sample_tokens_per_second(args.config, sample, threads),
                   "unit": "tokens/s", "cores": threads, "kind": "port",
                   "sample": f"{sample} tokens of the {args.config} block (host weights of the "
                             "experts they select)"}
        line = {
            "metric": f"MoE-layer tokens/s ({args.config} prefill T={T_total}, expert parallel)",
            "value": value, "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms / args.steps, "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
            "config": {"workload": f"{args.config} MoE block, prefill T={T_total} split over "
                                   f"{world} GPU(s), experts sharded {per} per GPU",
                       "parallelism": f"ep{world}", "tokens_per_gpu": T,
                       "l2": "weights larger than L2; no flush needed"},
            "roofline": {"bound": "tensor", "achieved": achieved, "peak": peak,
                         "unit": "TFLOP/s", "frac": achieved / peak, "traffic": None,
                         "kernel": "whole EP step", "algorithmic_flops_per_gpu": flops},
            "e2e": {"value": T_total * args.steps / el, "unit": "tokens/s",
                    "h2d_bytes_per_step": int(T * H * (2 if xdt == torch.bfloat16 else 4)),
                    "d2h_bytes_per_step": int(T * H * 4)},
            "gpu_launches": launches * args.steps,
            "clocks": clk.summary(),
            "cpu_baseline": cpu,
        }
        emit(line)
    sl.close()
    ctx.close()
    dist.barrier()
    dist.destroy_process_group()


# ---------------------------------------------------------------------------
# configuration 5: out-of-core decode through the expert cache
# ---------------------------------------------------------------------------

def host_memory_free() -> int:
    """Bytes this process may still take: MemAvailable, capped by the cgroup limit."""
    avail = None
    try:
        with open("/proc/meminfo") as f:
            for line in f:
                if line.startswith("MemAvailable:"):
                    avail = int(line.split()[1]) * 1024
    except OSError:
        pass
    avail = avail or 0
    for path in ("/sys/fs/cgroup/memory.max", "/sys/fs/cgroup/memory/memory.limit_in_bytes"):
        try:
            raw = open(path).read().strip()
        except OSError:
            continue
        if raw != "max" and raw.isdigit():
            limit = int(raw)
            used = 0
            for upath in ("/sys/fs/cgroup/memory.current",
                          "/sys/fs/cgroup/memory/memory.usage_in_bytes"):
                try:
                    used = int(open(upath).read().strip())
                    break
                except (OSError, ValueError):
                    continue
            avail = min(avail, max(0, limit - used))
        break
    return avail


def pinned_h2d_gbs(ctx, pool_ptr: int, nbytes: int, reps: int = 3) -> float:
    """Pinned host -> HBM copy bandwidth of this box (the PCIe roofline)."""
    import torch
    dst = torch.empty(nbytes, dtype=torch.uint8, device="cuda")
    src = torch.from_numpy(np.ctypeslib.as_array((np.ctypeslib.ctypes.c_uint8 * nbytes)
                                                 .from_address(pool_ptr)))
    best = 0.0
    for _ in range(reps):
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        dst.copy_(src, non_blocking=True)
        b.record()
        torch.cuda.synchronize()
        best = max(best, nbytes / (a.elapsed_time(b) / 1e3) / 1e9)
    del dst
    return best


def run_stack(args):
    import torch
    from diskmule_b200.moe import CudaContext
    from diskmule_b200.stack import GlmStack, OracleStack
    from diskmule_b200.synthetic import CONFIGS

    cfg = CONFIGS["glm52"]
    E, H, I, k = cfg["experts"], cfg["hidden"], cfg["intermediate"], cfg["top_k"]
    expert_bytes = 3 * H * I * 2
    full = args.layers * E
    if args.pool_experts:
        pool = min(args.pool_experts, full)
    else:
        # leave 64 GB and half of the rest of host memory to everything else
        usable = max(0, host_memory_free() - (64 << 30)) // 2
        pool = max(1, min(full, usable // expert_bytes))
    torch.cuda.set_device(0)
    ctx = CudaContext(0)
    t0 = time.perf_counter()
    st = GlmStack(ctx, "glm52", layers=args.layers, slots=args.slots, vocab=args.vocab,
                  pool_experts=pool)
    setup_s = time.perf_counter() - t0
    peak_h2d = pinned_h2d_gbs(ctx, st.pool.pointer, min(st.pool.length, 1 << 30))
    first = 1
    # greedy tokens on the GPU; the first steps replayed on the oracle below
    warm = st.decode(first, args.warmup)
    s0 = st.cache.stats()
    stream = torch.cuda.current_stream()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(0, settle=2.0) as clk:
        a.record(stream)
        tokens = st.decode(warm[-1] if warm else first, args.steps)
        b.record(stream)
        torch.cuda.synchronize()
    ms = a.elapsed_time(b)
    s1 = st.cache.stats()
    d = {key: s1[key] - s0[key] for key in ("hits", "misses", "evictions", "h2d_bytes",
                                             "io_wait_ns", "fills")}
    value = args.steps / (ms / 1e3)
    launches = sum(layer.last_launch_count() for layer in st.layers) + 2 + args.layers + 1

    # e2e: every step's token comes from the host and goes back to it
    tok_h = np.array([tokens[-1]], np.int32)
    import ctypes as C
    from diskmule_b200 import _native as N
    ring = st.token_ring
    torch.cuda.synchronize()
    t1 = time.perf_counter()
    e2e_steps = max(1, min(args.steps, 32))
    for _ in range(e2e_steps):
        N.check(N.lib().dm_buffer_write(ring.handle, 0, tok_h.ctypes.data_as(C.c_void_p), 4))
        st.step(ring.device_pointer, ring.device_pointer + 4)
        N.check(N.lib().dm_buffer_read(ring.handle, 4, tok_h.ctypes.data_as(C.c_void_p), 4))
    e2e = e2e_steps / (time.perf_counter() - t1)

    # oracle replay of the first steps from the same first token
    threads = os.cpu_count() or 1
    ref = OracleStack(st, threads=threads)
    check_n = min(args.check_steps, len(warm) + len(tokens))
    t2 = time.perf_counter()
    ref_tokens = ref.decode(first, check_n)
    cpu_s = time.perf_counter() - t2
    ours = (warm + tokens)[:check_n]

    achieved = d["h2d_bytes"] / (ms / 1e3) / 1e9
    hbm_bytes_step = args.layers * (k + 1) * expert_bytes
    line = {
        "metric": "MoE decode tokens/s (GLM-5.2 stack, experts out of core)",
        "value": value, "unit": "tokens/s", "n_gpus": 1, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms / args.steps, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
        "config": {"workload": f"{args.layers} GLM-5.2 sparse layers, {args.slots} HBM slots per "
                               f"layer, greedy batch-1 decode, vocab {args.vocab}",
                   "host_pool_gb": st.pool.length / 1e9, "pool_experts": pool,
                   "experts_total": full, "setup_s": setup_s,
                   "l2": "weights larger than L2; every miss copies 75.5 MB"},
        "roofline": {"bound": "pcie-h2d", "achieved": achieved, "peak": peak_h2d, "unit": "GB/s",
                     "frac": achieved / peak_h2d if peak_h2d else None, "traffic": None,
                     "peak_source": "pinned host->HBM copy measured in this run",
                     "hbm_expert_bytes_per_step": hbm_bytes_step},
        "cache": {"hits": d["hits"], "misses": d["misses"], "evictions": d["evictions"],
                  "misses_per_step": d["misses"] / args.steps,
                  "fill_device_s": d["io_wait_ns"] / 1e9, "h2d_bytes": d["h2d_bytes"]},
        "e2e": {"value": e2e, "unit": "tokens/s", "h2d_bytes_per_step": 4,
                "d2h_bytes_per_step": 4},
        "gpu_launches": launches * args.steps,
        "clocks": clk.summary(),
        "greedy_tokens_match_oracle": ours == ref_tokens,
        "checked_steps": check_n, "tokens_head": (warm + tokens)[:16],
        "status": st.status_bits(),
        "cpu_baseline": {"value": check_n / cpu_s, "unit": "tokens/s", "cores": threads,
                         "kind": "port",
                         "sample": f"{check_n} greedy steps of the same stack on the oracle "
                                   "(experts read from the host pool)"},
    }
    emit(line)
    st.close()
    ctx.close()


_RESULT_OUT = None


def emit(line: dict) -> None:
    """Print the one JSON result line on the process's original standard output."""
    print(json.dumps(line), file=_RESULT_OUT or sys.stdout, flush=True)


def main():
    global _RESULT_OUT
    # Libraries write banners to standard output from C (NCCL prints its version when a
    # communicator starts): keep the original stdout for the result line alone and send
    # everything else written to file descriptor 1 to stderr.
    sys.stdout.flush()
    _RESULT_OUT = os.fdopen(os.dup(1), "w")
    os.dup2(2, 1)
    args = parse_args()
    if args.impl == "reference":
        run_reference(args)
    elif args.ep:
        run_ep(args)
    elif args.stack:
        run_stack(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
