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


DEFAULT_TOKENS = {"glm52": 8192, "qwen35": 512, "gemma4": 4096}


def parse_args():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=None,
                   help="timed steps (default: 100 for glm52, 600 for the GGUF blocks)")
    p.add_argument("--warmup", type=int, default=5)
    p.add_argument("--impl", default="ours", choices=["ours", "reference"])
    p.add_argument("--config", default="glm52",
                   help="glm52 (configuration 4, expert parallel over the ranks; the default), "
                        "qwen35 or gemma4 (GGUF blocks, one replica per rank)")
    p.add_argument("--tokens", type=int, default=None,
                   help="tokens per step (default 8192 for glm52 in total over the ranks, "
                        "512 for qwen35 and 4096 for gemma4 per rank)")
    p.add_argument("--decode-steps", type=int, default=200)
    p.add_argument("--cpu-seconds", type=float, default=10.0)
    p.add_argument("--sample", type=int, default=4,
                   help="tokens per step of the CPU reference arm and of the parity check")
    p.add_argument("--profile-pass", type=int, default=0, metavar="R",
                   help="untimed: R forwards of --config/--tokens on one GPU with CUDA graphs "
                        "off, so every kernel is its own launch (the command profiled by ncu)")
    p.add_argument("--uniform", action="store_true",
                   help="gemma4: no Zipf(1.1) router bias (configuration 1's plain routing; "
                        "the default is configuration 3's skewed routing)")
    p.add_argument("--no-extras", action="store_true",
                   help="skip the GGUF-block and decode figures reported beside the headline")
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
    a = p.parse_args()
    if a.tokens is None:
        a.tokens = DEFAULT_TOKENS.get(a.config, 512)
    if a.steps is None:
        a.steps = 256 if a.stack else (100 if a.config == "glm52" else 600)
    return a


def metric_name(config: str, tokens: int) -> str:
    """The metric string, the same for both arms and every GPU count."""
    return f"MoE-layer tokens/s ({config} prefill T={tokens})"


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


def measured_tensor_peak(sustained: bool = False):
    """Dense bf16/fp16 TFLOP/s: the burst figure for a stage timed inside a short forward,
    the sustained one (a seconds-long GEMM loop under the power cap) for a long step."""
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        with open(path) as f:
            d = json.load(f)
        key = "bf16_tflops_sustained" if sustained else "bf16_tflops"
        if key in d:
            return d[key], "measured" + (" (sustained)" if sustained else " (burst)")
    return (1400.0, "fallback (sustained)") if sustained else (1590.0, "fallback (burst)")


FORMAT_NAMES = {0: "F32", 1: "F16", 6: "Q5_0", 8: "Q8_0", 12: "Q4_K", 14: "Q6_K", 30: "BF16"}
KERNEL_NAMES = {"gguf": {"expert_up": "tc_expert_kernel (gate/up)",
                         "expert_down": "tc_expert_kernel (down)"},
                "bf16": {"expert_up": "tc_bf16_kernel (gate/up)",
                         "expert_down": "tc_bf16_kernel (down)"}}


def choose_roofline(kernel, flops, nbytes, ms, hbm, tensor, traffic, note=None):
    """Roofline of one stage: the tensor peak when its FLOP per byte is above the ridge
    (peak FLOP/s / peak bytes/s), else HBM. hbm = (GB/s, source), tensor = (TFLOP/s, source)."""
    (peak, peak_src), (tpeak, tpeak_src) = hbm, tensor
    intensity = flops / nbytes
    if intensity > tpeak * 1e12 / (peak * 1e9):
        achieved = flops / (ms / 1e3) / 1e12
        r = {"bound": "tensor", "achieved": achieved, "peak": tpeak, "unit": "TFLOP/s",
             "frac": achieved / tpeak, "traffic": traffic, "kernel": kernel,
             "algorithmic_flops": flops, "algorithmic_bytes": nbytes, "peak_source": tpeak_src}
        if note:
            r["note"] = note
    else:
        achieved = nbytes / (ms / 1e3) / 1e9
        r = {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
             "frac": achieved / peak, "traffic": traffic, "kernel": kernel,
             "algorithmic_bytes": nbytes, "peak_source": peak_src}
    r["flop_per_byte"] = round(intensity, 1)
    r["kernel_ms"] = round(ms, 4)
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
# the CPU restatement of the reference path (the oracle): reference arm, CPU baseline
# and parity checker. The reference arm generates its inputs with the oracle library's
# copy of the seeded generator, so it never loads the CUDA library.
# ---------------------------------------------------------------------------

def glm_sample(cfg_name: str, x32: np.ndarray, threads: int, fill=None, seed: int = 1):
    """Oracle GLM block over the token rows x32 [n, H] (f32 values of bf16 rows), with
    host weights for the experts those tokens select only (the whole pool is tens of GB).
    Returns (seconds of the block call, y, idx, w)."""
    from diskmule_b200.synthetic import CONFIGS, SyntheticLayer, layer_specs, vectors
    from oracle import oracle as O
    cfg = dict(CONFIGS[cfg_name])
    specs = layer_specs(cfg, seed)
    sl = SyntheticLayer(cfg_name, cfg, seed, None, specs, vectors(cfg, seed))
    router = specs["router"].host(fill=fill)
    bias = specs["bias"].host(fill=fill).view(np.float32)
    chosen = set()
    for t in range(x32.shape[0]):
        _, lg = O.glm_matvec(O.BF16, cfg["experts"], cfg["hidden"], router, x32[t], threads)
        _, idx, _ = O.glm_select(lg, bias, cfg["top_k"], cfg["n_groups"], cfg["topk_groups"],
                                 cfg["normalize"])
        chosen.update(int(i) for i in idx)
    w = sl.host_weights(sorted(chosen), fill=fill)
    t0 = time.perf_counter()
    rc, y, idx, wt = O.glm_moe(w, x32, threads=threads)
    el = time.perf_counter() - t0
    assert rc == O.OK
    return el, y, idx, wt


def gguf_sample(cfg_name: str, x32: np.ndarray, threads: int, fill=None, seed: int = 1,
                logit_bias=None):
    """Oracle GGUF block (Qwen / Gemma) over x32 [n, H] with whole host weights."""
    from diskmule_b200.synthetic import CONFIGS, SyntheticLayer, layer_specs, vectors
    from oracle import oracle as O
    cfg = dict(CONFIGS[cfg_name])
    sl = SyntheticLayer(cfg_name, cfg, seed, None, layer_specs(cfg, seed), vectors(cfg, seed))
    sl.logit_bias = logit_bias
    w = sl.host_weights(fill=fill)
    fn = {"gemma4": O.gemma_moe, "qwen35": O.qwen_moe}[cfg["family"]]
    fn(w, x32[:1], threads=threads)  # touch the weights once
    t0 = time.perf_counter()
    rc, y, idx, wt = fn(w, x32, threads=threads)
    el = time.perf_counter() - t0
    assert rc == O.OK
    return el, y, idx, wt


def x32_rows(cfg: dict, rows: np.ndarray) -> np.ndarray:
    """f32 values of token rows (bf16 bits for GLM, f32 otherwise)."""
    if cfg["family"] == "glm52":
        return (rows.view(np.uint16).astype(np.uint32) << 16).view(np.float32)
    return rows.view(np.float32)


def run_reference(args):
    """The reference arm: the oracle on the host cores, on a bounded token sample per step
    of the same workload (tokens are independent in the reference, which runs one token
    at a time: src/glm52/cpu.rs:462-524, src/gemma4/cpu.rs:358-378)."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    from diskmule_b200.synthetic import CONFIGS, input_spec
    from oracle import oracle as O
    threads = os.cpu_count() or 1
    cfg = CONFIGS[args.config]
    n = args.sample if cfg["family"] == "glm52" else max(args.sample, 16)
    # the first n rows of the step's input (row t of a seeded input is the same for any T)
    x32 = x32_rows(cfg, input_spec(cfg, n, 21).host(fill=O.synth_fill)).reshape(n, -1)
    per_step = []
    if cfg["family"] == "glm52":
        from diskmule_b200.synthetic import SyntheticLayer, layer_specs, vectors
        # weights once (the same sample every step), then the block call timed per step
        sl = SyntheticLayer(args.config, dict(cfg), 1, None, layer_specs(dict(cfg), 1),
                            vectors(dict(cfg), 1))
        el, _, idx, _ = glm_sample(args.config, x32, threads, fill=O.synth_fill)
        w = sl.host_weights(sorted(set(idx.ravel().tolist())), fill=O.synth_fill)
        for i in range(args.warmup + args.steps):
            t0 = time.perf_counter()
            rc, _, _, _ = O.glm_moe(w, x32, threads=threads)
            assert rc == O.OK
            if i >= args.warmup:
                per_step.append(time.perf_counter() - t0)
    else:
        from diskmule_b200.synthetic import SyntheticLayer, layer_specs, vectors
        sl = SyntheticLayer(args.config, dict(cfg), 1, None, layer_specs(dict(cfg), 1),
                            vectors(dict(cfg), 1))
        w = sl.host_weights(fill=O.synth_fill)
        fn = {"gemma4": O.gemma_moe, "qwen35": O.qwen_moe}[cfg["family"]]
        for i in range(args.warmup + args.steps):
            t0 = time.perf_counter()
            rc, _, _, _ = fn(w, x32, threads=threads)
            assert rc == O.OK
            if i >= args.warmup:
                per_step.append(time.perf_counter() - t0)
    secs = sum(per_step)
    value = n * args.steps / secs
    sample = (f"{n} tokens per step of the {args.config} block (the first {n} rows of the "
              "step's input; tokens are independent in the reference)")
    line = {
        "impl": "reference", "metric": metric_name(args.config, args.tokens),
        "value": value, "unit": "tokens/s", "n_gpus": args.gpus, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": 1e3 * secs / args.steps, "higher_is_better": True,
        "scaling": "strong" if cfg["family"] == "glm52" else "weak", "vs_baseline": None,
        "dtype": "bf16" if cfg["family"] == "glm52" else "f32", "data": "synthetic",
        "config": {"workload": f"{args.config} MoE block, CPU oracle on a {n}-token sample "
                               "per step", "parallelism": f"cpu ({threads} threads)"},
        "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": threads, "kind": "port",
                         "sample": sample},
        "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    emit(line)


def parity_summary(cfg, y, idx, w, y_ref, idx_ref, w_ref):
    """The north-star bar on a token sample: indices and order bit-exact, selection weights
    within 2e-7, outputs within 1e-3 relative L2."""
    num = np.linalg.norm((y - y_ref).astype(np.float64), axis=-1)
    den = np.linalg.norm(y_ref.astype(np.float64), axis=-1)
    tok = num / np.maximum(den, 1e-30)
    layer = float(np.linalg.norm((y - y_ref).astype(np.float64)) /
                  np.linalg.norm(y_ref.astype(np.float64)))
    same = bool(np.array_equal(idx, idx_ref))
    wmax = float(np.max(np.abs(w - w_ref)))
    return {"tokens": int(y.shape[0]), "indices_equal": same, "weights_max_abs": wmax,
            "rel_l2": layer, "rel_l2_token_max": float(tok.max()),
            "pass": same and wmax <= 2e-7 and layer <= 1e-3}


# ---------------------------------------------------------------------------
# our arm: shared measurement helpers
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


def profile_stages(layer, step, n):
    """Average per-stage device times (ms) over n profiled forwards (CUDA events recorded
    by the library on the launching stream at every stage boundary)."""
    layer.set_profiling(True)
    totals = {}
    for _ in range(n):
        step()
        for name, t in layer.stage_times().items():
            totals[name] = totals.get(name, 0.0) + t
    layer.set_profiling(False)
    return {name: v / n for name, v in totals.items()}


def block_roofline(sl, T, avg, workload, sustained):
    """Roofline of the dominant expert stage from the profiled stage times."""
    counts, _, _, _ = sl.layer.last_dispatch(T)
    nbytes = stage_bytes(sl, T, counts)
    nflops = stage_flops(sl, T)
    dominant = max(("expert_up", "expert_down"), key=lambda n: avg[n])
    hbm = measured_peaks()
    tensor = measured_tensor_peak(sustained)
    bf16 = sl.cfg["gate_type"] == 30
    # the library's tensor-core plans: hi + lo activation halves up to 24 tokens per expert
    # on average, single fp16 rows above (DISKMULE_CUDA_TC_SPLIT=0 / =all override)
    per_expert = T * sl.cfg["top_k"] / sl.cfg["experts"]
    split_env = os.environ.get("DISKMULE_CUDA_TC_SPLIT", "")
    split = split_env == "all" or (per_expert <= 24 and split_env not in ("0", "false"))
    note = None if bf16 else (
        "fp16 MMAs on hi + lo activation halves: the tensor pipe does twice the algorithmic "
        "FLOPs" if split else
        "fp16 MMAs on single fp16 activation rows, each scaled by a power of two")
    r = choose_roofline(dominant, nflops[dominant], nbytes[dominant], avg[dominant], hbm,
                        tensor, ncu_traffic(dominant, workload), note)
    r["kernel"] = KERNEL_NAMES["bf16" if bf16 else "gguf"][dominant]
    r["stage_ms"] = {n: round(v, 4) for n, v in avg.items()}
    return r


def decode_block(sl, steps, warmup, rank, seed=33):
    """Decode (T = 1): distinct tokens, L2 flushed (a 256 MB write) before every timed
    token, so each token's router and expert weights come from HBM; tokens are timed one
    by one with events on the launching stream and the flushes stay outside the spans."""
    import torch
    cfg = sl.cfg
    H = cfg["hidden"]
    xdt = torch.bfloat16 if cfg["family"] == "glm52" else torch.float32
    from diskmule_b200.synthetic import input_spec
    n_dec = 12  # forward() keeps up to 16 CUDA graphs keyed by buffers
    x1 = torch.empty((n_dec, H), dtype=xdt, device="cuda")
    input_spec(cfg, n_dec, seed + rank).device_fill(x1.data_ptr())
    y1 = torch.empty((n_dec, H), dtype=torch.float32, device="cuda")
    flush = torch.empty(256 << 20, dtype=torch.uint8, device="cuda")
    xrow = x1.element_size() * H
    stream = torch.cuda.current_stream()
    sptr = stream.cuda_stream
    torch.cuda.synchronize()

    def dec(i):
        j = i % n_dec
        sl.layer.forward(x1.data_ptr() + j * xrow, y1.data_ptr() + j * H * 4, 1, stream=sptr)

    for i in range(warmup):
        dec(i)
    torch.cuda.synchronize()
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
          for _ in range(steps)]
    for i in range(steps):
        flush.fill_(i & 0xFF)
        ev[i][0].record(stream)
        dec(i)
        ev[i][1].record(stream)
    torch.cuda.synchronize()
    dms = sum(a.elapsed_time(b) for a, b in ev)
    dec(0)
    torch.cuda.synchronize()
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
    peak, _ = measured_peaks()
    dstage = {n: round(1e3 * v / 20, 2) for n, v in dtot.items()}
    up_bw = b1["expert_up"] / (dstage["expert_up"] * 1e-6) / 1e9 if dstage.get("expert_up") else 0
    dn_bw = (b1["expert_down"] / (dstage["expert_down"] * 1e-6) / 1e9
             if dstage.get("expert_down") else 0)
    return {"tokens_per_s": steps / (dms / 1e3), "us_per_token": 1e3 * dms / steps,
            "algorithmic_bytes_per_token": dec_bytes,
            "hbm_frac": dec_bytes / (dms / steps / 1e3) / 1e9 / peak,
            "stage_us": dstage,
            "expert_up_hbm_frac": up_bw / peak, "expert_down_hbm_frac": dn_bw / peak}


def prefill_block(sl, T, steps, warmup, rank, seed=21):
    """Prefill of T tokens on one GPU through dm_moe_forward: value, stage roofline."""
    import torch
    from diskmule_b200.synthetic import input_spec
    cfg = sl.cfg
    H = cfg["hidden"]
    xdt = torch.bfloat16 if cfg["family"] == "glm52" else torch.float32
    x = torch.empty((T, H), dtype=xdt, device="cuda")
    y = torch.empty((T, H), dtype=torch.float32, device="cuda")
    input_spec(cfg, T, seed + rank).device_fill(x.data_ptr())
    stream = torch.cuda.current_stream()
    sptr = stream.cuda_stream

    def step():
        sl.layer.forward(x.data_ptr(), y.data_ptr(), T, stream=sptr)

    for _ in range(warmup):
        step()
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record(stream)
    for _ in range(steps):
        step()
    b.record(stream)
    torch.cuda.synchronize()
    ms = a.elapsed_time(b) / steps
    avg = profile_stages(sl.layer, step, min(steps, 20))
    r = block_roofline(sl, T, avg, f"{sl.name}-T{T}", sustained=False)
    return {"tokens_per_s": T / (ms / 1e3), "ms_per_step": ms, "tokens": T, "roofline": r}


# ---------------------------------------------------------------------------
# GGUF blocks (configurations 1-3): one replica per rank
# ---------------------------------------------------------------------------

def run_gguf(args):
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

    from diskmule_b200.moe import CudaContext
    from diskmule_b200.synthetic import build_layer, input_spec, zipf_bias

    ctx = CudaContext(local)
    bias = zipf_bias(128, 1.1, 5) if args.config == "gemma4" and not args.uniform else None
    sl = build_layer(ctx, args.config, seed=1, logit_bias=bias)
    cfg = sl.cfg
    T, H, k = args.tokens, cfg["hidden"], cfg["top_k"]
    xdt = torch.float32
    x = torch.empty((T, H), dtype=xdt, device="cuda")
    y = torch.empty((T, H), dtype=torch.float32, device="cuda")
    sel_i = torch.empty((T, k), dtype=torch.int32, device="cuda")
    sel_w = torch.empty((T, k), dtype=torch.float32, device="cuda")
    xs = input_spec(cfg, T, 21 + rank)
    xs.device_fill(x.data_ptr())
    ctx.synchronize()
    stream = torch.cuda.current_stream()
    sptr = stream.cuda_stream

    def step():
        sl.layer.forward(x.data_ptr(), y.data_ptr(), T, sel_i.data_ptr(), sel_w.data_ptr(),
                         stream=sptr)

    for _ in range(args.warmup):
        step()
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
            step()
        end.record(stream)
        torch.cuda.synchronize()
    barrier()
    ms = max_over_ranks(start.elapsed_time(end))
    value = world * T * args.steps / (ms / 1e3)
    avg = profile_stages(sl.layer, step, min(args.steps, 50))
    roofline = block_roofline(sl, T, avg, f"{args.config}-T{T}", sustained=False)
    weight_gb = sum(sl.specs[n].expert_bytes for n in ("gate", "up", "down") if n in sl.specs) * \
        (cfg["experts"] + (1 if cfg.get("shared") else 0)) / 1e9
    barrier()
    decode = decode_block(sl, args.decode_steps, args.warmup, rank)

    # e2e through the public host API: pipelined batches (page-locked host buffers)
    xh = torch.empty((T, H), dtype=xdt, pin_memory=True)
    xh.copy_(x.cpu())
    nb = 8
    xs_h = [xh.numpy()] * nb
    ys_h = [torch.empty((T, H), dtype=torch.float32, pin_memory=True).numpy() for _ in range(2)]
    ys_h = [ys_h[i & 1] for i in range(nb)]
    sl.layer.forward_host_batches(xs_h[:2], ys_h[:2])
    barrier()
    reps = max(1, args.steps // nb)
    t0 = time.perf_counter()
    for _ in range(reps):
        sl.layer.forward_host_batches(xs_h, ys_h)
    el = max_over_ranks(time.perf_counter() - t0)
    e2e = {"value": world * T * nb * reps / el, "unit": "tokens/s",
           "h2d_bytes_per_step": int(T * H * 4), "d2h_bytes_per_step": int(T * H * 4),
           "api": f"dm_moe_forward_host_batches, {nb} batches per call"}

    if rank == 0:
        cpu = None
        parity = None
        if world == 1:
            threads = os.cpu_count() or 1
            n = max(args.sample, 16)
            x32 = x32_rows(cfg, xs.host()[: n * H * 4]).reshape(n, H)
            el_c, y_ref, i_ref, w_ref = gguf_sample(args.config, x32, threads, logit_bias=bias)
            step()
            torch.cuda.synchronize()
            # the first n tokens of the benchmarked T-token forward
            parity = parity_summary(cfg, y[:n].cpu().numpy(),
                                    sel_i[:n].cpu().numpy().view(np.uint32),
                                    sel_w[:n].cpu().numpy(), y_ref, i_ref, w_ref)
            cpu = {"value": n / el_c, "unit": "tokens/s", "cores": threads, "kind": "port",
                   "sample": f"{n} tokens of the {args.config} block in one oracle call"}
        line = {
            "metric": metric_name(args.config, T),
            "value": value, "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms / args.steps, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": {"workload": f"{args.config} MoE block, prefill T={T} per GPU"
                                   + (", Zipf(1.1)-biased routing" if bias is not None else ""),
                       "tokens_per_step": T, "hidden": H, "experts": cfg["experts"],
                       "top_k": k, "intermediate": cfg["intermediate"],
                       "formats": f"{FORMAT_NAMES.get(cfg['gate_type'], cfg['gate_type'])} gate/up, "
                                  f"{FORMAT_NAMES.get(cfg['down_type'], cfg['down_type'])} down",
                       "parallelism": f"replicas x{world}",
                       "l2": f"expert weights ({weight_gb:.2f} GB) larger than L2; no flush needed"},
            "roofline": roofline, "decode": decode, "e2e": e2e, "parity": parity,
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
# configuration 4 (the headline): GLM-5.2 bf16 layer, T = 8192, expert parallel
# ---------------------------------------------------------------------------

def run_glm(args):
    import datetime
    import torch
    import torch.distributed as dist

    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    if world > 1:
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

    from diskmule_b200.ep import PeerExpertParallel
    from diskmule_b200.moe import CudaContext
    from diskmule_b200.synthetic import CONFIGS, build_layer, input_spec

    cfg = dict(CONFIGS[args.config])
    E, H, I, k = cfg["experts"], cfg["hidden"], cfg["intermediate"], cfg["top_k"]
    if E % world or args.tokens % world:
        raise SystemExit(f"{E} experts / {args.tokens} tokens do not split over {world} GPUs")
    per = E // world
    T_total = args.tokens
    T = T_total // world
    ctx = CudaContext(local)
    # one GPU holds every expert; with several, rank g holds [g*per, (g+1)*per)
    sl = build_layer(ctx, args.config, seed=1,
                     expert_range=None if world == 1 else (rank * per, per))
    x = torch.empty((T, H), dtype=torch.bfloat16, device="cuda")
    xs = input_spec(cfg, T, 21 + rank)
    xs.device_fill(x.data_ptr())
    ctx.synchronize()
    stream = torch.cuda.current_stream()
    sptr = stream.cuda_stream
    if world == 1:
        y = torch.empty((T, H), dtype=torch.float32, device="cuda")
        sel_i = torch.empty((T, k), dtype=torch.int32, device="cuda")
        sel_w = torch.empty((T, k), dtype=torch.float32, device="cuda")

        def step():
            sl.layer.forward(x.data_ptr(), y.data_ptr(), T, sel_i.data_ptr(), sel_w.data_ptr(),
                             stream=sptr)
            return y
    else:
        # token rows and expert outputs travel as stores into the peers' memory
        ep = PeerExpertParallel(sl.layer, rank, world, T)
        ep.connect_ipc()
        y = torch.empty((T, H), dtype=torch.float32, device="cuda")
        sel_i = torch.empty((T, k), dtype=torch.int32, device="cuda")
        sel_w = torch.empty((T, k), dtype=torch.float32, device="cuda")

        def step():
            return ep.forward(x, y, sel_i, sel_w, stream=sptr)

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    barrier()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local, active=rank == 0) as clk:
        barrier()  # rank 0 entered after the sampler settled
        torch.cuda.synchronize()
        start.record(stream)
        for _ in range(args.steps):
            yy = step()
        end.record(stream)
        torch.cuda.synchronize()
    barrier()
    ms = max_over_ranks(start.elapsed_time(end))
    value = T_total * args.steps / (ms / 1e3)

    # kernels of one step, and the dominant kernel's event-timed duration
    if world == 1:
        launches = sl.layer.last_launch_count()
        avg = profile_stages(sl.layer, step, min(args.steps, 20))
        roofline = block_roofline(sl, T, avg, f"{args.config}-T{T}", sustained=True)
    else:
        ep.status()
        launches = ep.last_launch_count()
        stage = ep_profile(ep, x, y, n=min(args.steps, 20))
        roofline = ep_roofline(sl, stage, T_total * k // world + T)
    barrier()

    # e2e: every step's input comes from page-locked host memory and its output returns
    xh = torch.empty((T, H), dtype=torch.bfloat16, pin_memory=True)
    xh.copy_(x.cpu())
    nb = 8  # batches per call: the copy of a call's first input and last output stay exposed
    if world == 1:
        xs_h = [xh.view(torch.int16).numpy()] * nb
        yb = [torch.empty((T, H), dtype=torch.float32, pin_memory=True).numpy() for _ in range(2)]
        ys_h = [yb[i & 1] for i in range(nb)]
        sl.layer.forward_host_batches(xs_h[:2], ys_h[:2])
        reps = max(1, args.steps // nb)
        t0 = time.perf_counter()
        for _ in range(reps):
            sl.layer.forward_host_batches(xs_h, ys_h)
        el = time.perf_counter() - t0
        e2e_steps = reps * nb
        api = f"dm_moe_forward_host_batches, {nb} batches per call"
    else:
        yh = [torch.empty((T, H), dtype=torch.float32, pin_memory=True) for _ in range(2)]
        e2e_steps = max(4, min(args.steps, 40))
        host_stream(lambda xd, yd: ep.forward(xd, yd), xh, yh, 2, H)
        barrier()
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        host_stream(lambda xd, yd: ep.forward(xd, yd), xh, yh, e2e_steps, H)
        el = time.perf_counter() - t0
        ep.status()
        api = ("PeerExpertParallel.forward, input and output copies of neighbouring steps on "
               "side streams")
    el = max_over_ranks(el)
    e2e = {"value": T_total * e2e_steps / el, "unit": "tokens/s",
           "h2d_bytes_per_step": int(T_total * H * 2), "d2h_bytes_per_step": int(T_total * H * 4),
           "api": api}

    # parity of a seeded sample of rank 0's tokens against the oracle (after timing)
    parity = cpu = None
    n = args.sample
    if rank == 0:
        yy = step()
        torch.cuda.synchronize()
        idx_d, w_d = sel_i[:n].cpu().numpy().view(np.uint32), sel_w[:n].cpu().numpy()
        y_d = yy[:n].float().cpu().numpy()
        threads = os.cpu_count() or 1
        x32 = x32_rows(cfg, xs.host()[: n * H * 2]).reshape(n, H)
        el_c, y_ref, i_ref, w_ref = glm_sample(args.config, x32, threads)
        parity = parity_summary(cfg, y_d, idx_d, w_d, y_ref, i_ref, w_ref)
        if world == 1:
            cpu = {"value": n / el_c, "unit": "tokens/s", "cores": threads, "kind": "port",
                   "sample": f"{n} tokens of the {args.config} block in one oracle call (host "
                             "weights of the experts they select)"}
    barrier()
    if world > 1:
        barrier()  # no rank unmaps its peers' regions while another still stores into them
        ep.close()
        barrier()

    extras = None
    if world == 1 and not args.no_extras:
        extras = {"glm52_decode_T1": decode_block(sl, args.decode_steps, args.warmup, rank)}
    sl.close()
    if world == 1 and not args.no_extras:
        from diskmule_b200.synthetic import zipf_bias
        for name, T_x, bias in (("qwen35", 512, None), ("gemma4", 4096, zipf_bias(128, 1.1, 5))):
            s2 = build_layer(ctx, name, seed=1, logit_bias=bias)
            pre = prefill_block(s2, T_x, max(20, args.steps), args.warmup, rank)
            dec = decode_block(s2, args.decode_steps, args.warmup, rank)
            key = f"{name}_prefill_T{T_x}" + ("_zipf" if bias is not None else "")
            extras[key] = pre
            extras[f"{name}_decode_T1"] = dec
            s2.close()

    if rank == 0:
        line = {
            "metric": metric_name(args.config, T_total),
            "value": value, "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms / args.steps, "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
            "config": {"workload": f"{args.config} MoE layer (configuration 4), prefill "
                                   f"T={T_total} in total"
                                   + (f", split over {world} GPUs, experts sharded {per} per GPU"
                                      if world > 1 else " on one GPU holding every expert"),
                       "parallelism": f"ep{world}", "tokens_per_gpu": T, "hidden": H,
                       "experts": E, "top_k": k, "intermediate": I,
                       "formats": "BF16 router, gate/up, down, shared expert; f32 accumulate",
                       "l2": "expert weights (19.3 GB) larger than L2; no flush needed"},
            "roofline": roofline, "e2e": e2e, "parity": parity,
            "gpu_launches": launches * args.steps,
            "clocks": clk.summary(),
            "cpu_baseline": cpu,
            "extras": extras,
        }
        emit(line)
    ctx.close()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def ep_profile(ep, x, y, n):
    """Average device time (ms) of the three phases of an expert-parallel forward
    (events on the launching stream): dispatch (router, top-k, row stores to the peers),
    experts (wait for every rank's rows, local GEMMs, output stores), combine (wait for
    every rank's outputs, weighted combine)."""
    import torch
    stream = torch.cuda.current_stream()
    tot = {"dispatch": 0.0, "experts": 0.0, "combine": 0.0}
    for _ in range(n):
        ev = [torch.cuda.Event(enable_timing=True) for _ in range(4)]
        ev[0].record(stream)
        ep.dispatch(x)
        ev[1].record(stream)
        ep.experts()
        ev[2].record(stream)
        ep.combine(y)
        ev[3].record(stream)
        torch.cuda.synchronize()
        for i, name in enumerate(("dispatch", "experts", "combine")):
            tot[name] += ev[i].elapsed_time(ev[i + 1])
    return {name: v / n for name, v in tot.items()}


def host_stream(forward, x_host, y_host, steps, hidden):
    """`steps` forwards of the page-locked rows x_host: the input copy of step i+1 runs
    on a side stream while step i computes, and the output copy of step i on another."""
    import torch
    cs = torch.cuda.current_stream()
    s_in, s_out = torch.cuda.Stream(), torch.cuda.Stream()
    T = x_host.shape[0]
    xb = [torch.empty_like(x_host, device="cuda") for _ in range(2)]
    yb = [torch.empty((T, hidden), dtype=torch.float32, device="cuda") for _ in range(2)]
    ready = [torch.cuda.Event() for _ in range(2)]
    used = [torch.cuda.Event() for _ in range(2)]     # forward i finished reading xb / writing yb
    copied = [torch.cuda.Event() for _ in range(2)]   # output copy of step i finished
    with torch.cuda.stream(s_in):
        xb[0].copy_(x_host, non_blocking=True)
        ready[0].record(s_in)
    for i in range(steps):
        j = i & 1
        if i + 1 < steps:
            with torch.cuda.stream(s_in):
                if i >= 1:
                    s_in.wait_event(used[1 - j])
                xb[1 - j].copy_(x_host, non_blocking=True)
                ready[1 - j].record(s_in)
        cs.wait_event(ready[j])
        if i >= 2:
            cs.wait_event(copied[j])
        forward(xb[j], yb[j])
        used[j].record(cs)
        s_out.wait_event(used[j])
        with torch.cuda.stream(s_out):
            y_host[i % len(y_host)].copy_(yb[j], non_blocking=True)
            copied[j].record(s_out)
    torch.cuda.synchronize()


def ep_roofline(sl, stage, rows):
    """Roofline of the local expert GEMMs inside an expert-parallel step: useful FLOPs of
    the rows this rank's experts run (`rows`: the expected T*k/world routed rows plus the
    shared expert's T) ÷ the experts phase's event-timed duration (which also holds the
    wait for the peers' rows and the output stores), against the sustained bf16 peak."""
    cfg = sl.cfg
    H, I = cfg["hidden"], cfg["intermediate"]
    flops = 2.0 * rows * 3 * H * I
    ms = stage["experts"]
    tpeak, src = measured_tensor_peak(True)
    achieved = flops / (ms / 1e3) / 1e12
    return {"bound": "tensor", "achieved": achieved, "peak": tpeak, "unit": "TFLOP/s",
            "frac": achieved / tpeak, "traffic": None,
            "kernel": "tc_bf16_kernel (local experts, experts phase)",
            "algorithmic_flops": flops, "peak_source": src, "kernel_ms": round(ms, 4),
            "stage_ms": {n: round(v, 4) for n, v in stage.items()}}


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
    from diskmule_b200.stack import GlmStack
    from oracle.stack import OracleStack
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


def run_profile_pass(args):
    """R forwards of one block (one GPU, graphs off) for ncu's launch lists and captures;
    the same kernels as the timed steps. Prints one JSON line."""
    os.environ["DISKMULE_CUDA_GRAPHS"] = "0"
    import torch
    from diskmule_b200.moe import CudaContext
    from diskmule_b200.synthetic import build_layer, input_spec, zipf_bias

    torch.cuda.set_device(0)
    ctx = CudaContext(0)
    bias = zipf_bias(128, 1.1, 5) if args.config == "gemma4" and not args.uniform else None
    sl = build_layer(ctx, args.config, seed=1, logit_bias=bias)
    cfg, T = sl.cfg, args.tokens
    xdt = torch.bfloat16 if cfg["family"] == "glm52" else torch.float32
    x = torch.empty((T, cfg["hidden"]), dtype=xdt, device="cuda")
    y = torch.empty((T, cfg["hidden"]), dtype=torch.float32, device="cuda")
    input_spec(cfg, T, 21).device_fill(x.data_ptr())
    ctx.synchronize()
    stream = torch.cuda.current_stream().cuda_stream
    for _ in range(args.profile_pass):
        sl.layer.forward(x.data_ptr(), y.data_ptr(), T, stream=stream)
    torch.cuda.synchronize()
    emit({"profile_pass": args.profile_pass, "config": args.config, "tokens": T,
          "launches_per_forward": sl.layer.last_launch_count()})
    sl.close()
    ctx.close()


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
    elif args.profile_pass:
        run_profile_pass(args)
    elif args.stack:
        run_stack(args)
    elif args.config == "glm52":
        run_glm(args)
    else:
        run_gguf(args)


if __name__ == "__main__":
    main()
