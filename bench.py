#!/usr/bin/env python3
"""Benchmark of the B200 attention path of the MetalNLLB engine.

Headline workload (one "step"): the decoder self-attention decode sweep of
a batch of sentences resident on each GPU - 4 beams x 16 heads x head_dim 64,
fp32, the KV cache growing from length 1 to 256 with a random beam
permutation applied (by index) before every decode step, exactly the
per-sentence shape of the decode-op configuration, batched over sentences the
way the sentence-batched translation shards them.  Metric: algorithmic HBM
bytes per second of the decode attention (K/V cache reads + q/out + new k/v
+ beam index), summed over GPUs (weak scaling: every GPU holds its own
sentences; no collective on the data path).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Under torchrun each rank drives LOCAL_RANK's GPU; rank 0 prints one JSON line.
"""
from __future__ import annotations

import argparse
import datetime
import json
import os
import statistics
import subprocess
import sys
import threading
import time

REPO = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(REPO, "bare-metal-nllb_b200"))

HEADS, HEAD_DIM, BEAMS = 16, 64, 4
DMODEL = HEADS * HEAD_DIM
ROW_BYTES = HEAD_DIM * 4


def step_bytes_per_sentence(L: int, beams: int = BEAMS) -> int:
    """Algorithmic bytes of one decode step at cache length L (positions
    0..L-1, the last one new): K+V rows 2*beams*heads*L*256 B, q and out
    beams*heads*256 B each, new k and v read, beam index 4 B per beam-position."""
    kv = 2 * beams * HEADS * L * ROW_BYTES
    q_out = 2 * beams * HEADS * ROW_BYTES
    new_kv = 2 * beams * HEADS * ROW_BYTES
    index = 4 * beams * L
    return kv + q_out + new_kv + index


def sweep_bytes_per_sentence(T: int) -> int:
    return sum(step_bytes_per_sentence(L) for L in range(1, T + 1))


def load_peaks():
    p = os.path.join(REPO, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), float(d.get("bf16_tflops", 0)), "measured"
    return 6650.0, 1590.0, "fallback"


class ClockSampler:
    """nvidia-smi clocks and throttle reasons sampled during the timed region."""
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.lines = []

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "100"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
        except (FileNotFoundError, OSError):
            self.proc = None
        return self

    def _read(self):
        for ln in self.proc.stdout:
            self.lines.append(ln.strip())

    def __exit__(self, *exc):
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self):
        sm, mx, reasons = [], None, set()
        names = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")
        for ln in self.lines:
            parts = [x.strip() for x in ln.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                mx = float(parts[2])
            except ValueError:
                continue
            for n, v in zip(names, parts[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": mx, "reasons": [], "samples": 0}
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm)}


def parse_args():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=("ours", "reference"), default="ours")
    ap.add_argument("--sentences", type=int, default=128, help="sentences per GPU")
    ap.add_argument("--max-len", type=int, default=256, help="decode steps per sweep")
    ap.add_argument("--no-ops", action="store_true", help="skip the per-config op measurements")
    ap.add_argument("--cpu-sample-s", type=float, default=10.0)
    return ap.parse_args()


# ---------------------------------------------------------------------------
# CPU reference (oracle/_ref: the reference's own decoder.c attention)
# ---------------------------------------------------------------------------
def host_threads() -> int:
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1


def cpu_reference_rate(target_s: float, T: int):
    """Times the reference's decoder_self_attn_cached sweep (bias-injected
    q/k/v, reorder by copy as main.c does) on all host threads, over a bounded
    number of sentences, and returns (GB/s, cores, sample description, kind)."""
    sys.path.insert(0, os.path.join(REPO, "oracle"))
    import pyoracle as po
    kind = "reference"
    lib = po.ref_lib() if po.ref_available() else None
    if lib is None:
        raise RuntimeError("oracle/_ref/libnllb_ref.so is not built")
    cores = host_threads()
    probe_sent = max(1, cores // BEAMS)
    dt = lib.ref_time_decode_sweep(probe_sent, BEAMS, T, cores, 7)
    per_sent = dt / probe_sent
    n_sent = max(probe_sent, min(256, int(target_s / max(per_sent, 1e-6))))
    dt = lib.ref_time_decode_sweep(n_sent, BEAMS, T, cores, 11)
    gbs = n_sent * sweep_bytes_per_sentence(T) / dt / 1e9
    sample = (f"{n_sent} sentence(s) x {BEAMS} beams x {HEADS} heads, cache 1->{T} with a "
              f"permutation reorder per step, {dt:.1f} s on {cores} threads")
    return gbs, cores, sample, kind, dt


# ---------------------------------------------------------------------------
# our arm
# ---------------------------------------------------------------------------
def run_ours(args, rank, world, local_rank):
    import numpy as np
    import torch
    import torch.distributed as dist
    import nllb_attn as na

    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    S, T = args.sentences, args.max_len
    stream = torch.cuda.Stream(device=dev)
    ctx = na.Context(local_rank, n_layers=1, n_heads=HEADS, max_sentences=S, n_beams=BEAMS,
                     max_tgt=T, max_src=1)
    ctx.set_stream(stream.cuda_stream)

    g = torch.Generator(device=dev)
    g.manual_seed(2 + rank)
    # per-step inputs, N(0,1): [T][S][beams][1024]
    q = torch.randn((T, S, BEAMS, DMODEL), generator=g, device=dev)
    k = torch.randn((T, S, BEAMS, DMODEL), generator=g, device=dev)
    v = torch.randn((T, S, BEAMS, DMODEL), generator=g, device=dev)
    out = torch.empty((T, S, BEAMS, DMODEL), device=dev)
    parents = torch.argsort(torch.rand((T, S, BEAMS), generator=g, device=dev), dim=-1).to(torch.int32)
    torch.cuda.synchronize(dev)

    def sweep():
        for t in range(T):
            ctx.reorder(S, parents[t])
            ctx.decode_self(0, t, S, q[t], k[t], v[t], out[t])

    with torch.cuda.stream(stream):
        for _ in range(args.warmup):
            sweep()
    torch.cuda.synchronize(dev)
    ctx.sync()

    def barrier():
        if world > 1:
            dist.barrier()

    vis = os.environ.get("CUDA_VISIBLE_DEVICES", "")
    smi_index = vis.split(",")[local_rank] if vis else str(local_rank)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier()
    torch.cuda.synchronize(dev)
    with ClockSampler(smi_index) as clk:
        with torch.cuda.stream(stream):
            e0.record(stream)
            for _ in range(args.steps):
                sweep()
            e1.record(stream)
        torch.cuda.synchronize(dev)
    barrier()
    ctx.sync()
    elapsed = e0.elapsed_time(e1) / 1e3
    t_max = torch.tensor([elapsed], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(t_max, op=dist.ReduceOp.MAX)
    t_max = float(t_max.item())

    per_rank_bytes = S * sweep_bytes_per_sentence(T)
    value = world * per_rank_bytes * args.steps / t_max / 1e9  # GB/s
    ms_per_step = t_max / args.steps * 1e3

    # dominant kernel alone: events around every decode launch of one sweep
    dec_ms = 0.0
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(T)]
    with torch.cuda.stream(stream):
        for t in range(T):
            ctx.reorder(S, parents[t])
            evs[t][0].record(stream)
            ctx.decode_self(0, t, S, q[t], k[t], v[t], out[t])
            evs[t][1].record(stream)
    torch.cuda.synchronize(dev)
    dec_ms = sum(a.elapsed_time(b) for a, b in evs)
    kernel_gbs = per_rank_bytes / (dec_ms / 1e3) / 1e9
    hbm_peak, tflops_peak, peak_kind = load_peaks()

    # e2e through the host-buffer C ABI: H2D of q/k/v/parents, D2H of out, every launch
    e2e = None
    n_pool = 8
    qh = torch.empty((n_pool, S, BEAMS, DMODEL), pin_memory=True)
    qh.normal_()
    kh = torch.empty_like(qh).normal_()
    vh = torch.empty_like(qh).normal_()
    oh = torch.empty_like(qh)
    ph = torch.argsort(torch.rand((T, S, BEAMS)), dim=-1).to(torch.int32).contiguous()
    qn, kn, vn, on, pn = qh.numpy(), kh.numpy(), vh.numpy(), oh.numpy(), ph.numpy()
    e2e_steps = max(1, min(args.steps, 2))
    ctx.set_stream(None)

    def host_sweep():
        for t in range(T):
            i = t % n_pool
            ctx.reorder_host(S, pn[t])
            ctx.decode_self_host(0, t, S, qn[i], kn[i], vn[i], on[i])

    host_sweep()  # warm-up (staging buffers)
    barrier()
    t0 = time.perf_counter()
    for _ in range(e2e_steps):
        host_sweep()
    t_e2e = time.perf_counter() - t0
    te = torch.tensor([t_e2e], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(te, op=dist.ReduceOp.MAX)
    t_e2e = float(te.item())
    act_bytes = S * BEAMS * DMODEL * 4
    e2e = {
        "value": round(world * per_rank_bytes * e2e_steps / t_e2e / 1e9, 2),
        "unit": "GB/s",
        "h2d_bytes_per_step": T * (3 * act_bytes + S * BEAMS * 4),
        "d2h_bytes_per_step": T * act_bytes,
        "how": "nllb_attn_reorder_host + nllb_attn_decode_self_host per decode step from pinned host "
               "memory; wall clock, max over ranks",
    }

    result = {
        "value": value, "ms_per_step": ms_per_step, "kernel_gbs": kernel_gbs,
        "dec_ms_per_sweep": dec_ms, "clocks": clk.summary(), "hbm_peak": hbm_peak,
        "peak_kind": peak_kind, "e2e": e2e,
    }
    ops = None
    if not args.no_ops and rank == 0:
        ops = measure_ops(ctx_factory=lambda **kw: na.Context(local_rank, **kw), dev=dev,
                          hbm_peak=hbm_peak)
    ctx.close()
    return result, ops


def measure_ops(ctx_factory, dev, hbm_peak):
    """Single-instance numbers for the op configurations (per launch, L2
    flushed before each launch, CUDA events around the kernel only)."""
    import torch
    flush = torch.empty(256 * 2**20 // 4, dtype=torch.float32, device=dev)
    stream = torch.cuda.Stream(device=dev)
    res = {}

    def timed(fn, n):
        ts = []
        with torch.cuda.stream(stream):
            for i in range(n):
                flush.fill_(float(i))
                a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                a.record(stream)
                fn(i)
                b.record(stream)
                ts.append((a, b))
        torch.cuda.synchronize(dev)
        return [a.elapsed_time(b) * 1e-3 for a, b in ts]

    g = torch.Generator(device=dev)
    g.manual_seed(2)
    # decode op: 1 sentence, cache 1->256, permutation before each step
    T = 256
    c = ctx_factory(n_layers=1, n_heads=HEADS, max_sentences=1, n_beams=BEAMS, max_tgt=T, max_src=1)
    c.set_stream(stream.cuda_stream)
    q, k, v = (torch.randn((T, BEAMS, DMODEL), generator=g, device=dev) for _ in range(3))
    out = torch.empty_like(q)
    par = torch.argsort(torch.rand((T, BEAMS), generator=g, device=dev), dim=-1).to(torch.int32)

    def dec(t):
        c.decode_self(0, t, 1, q[t], k[t], v[t], out[t])

    with torch.cuda.stream(stream):
        for t in range(T):  # warm-up sweep
            c.reorder(1, par[t])
            dec(t)
    c.reset()
    ts = []
    with torch.cuda.stream(stream):
        for t in range(T):
            c.reorder(1, par[t])
            flush.fill_(float(t))
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record(stream)
            dec(t)
            b.record(stream)
            ts.append((a, b))
    torch.cuda.synchronize(dev)
    c.sync()
    tt = [a.elapsed_time(b) * 1e-3 for a, b in ts]
    tot_bytes = sweep_bytes_per_sentence(T)
    res["decode_self_config"] = {
        "shape": "1 sentence x 4 beams x 16 heads x 64, cache 1->256, permutation per step",
        "gbs": round(tot_bytes / sum(tt) / 1e9, 1),
        "us_per_launch_mean": round(sum(tt) / T * 1e6, 2),
        "us_at_len_256": round(tt[-1] * 1e6, 2),
        "gbs_at_len_256": round(step_bytes_per_sentence(256) / tt[-1] / 1e9, 1),
        "frac_of_hbm_peak": round(tot_bytes / sum(tt) / 1e9 / hbm_peak, 4),
        "l2": "flushed (256 MB write) before every launch",
    }
    c.close()

    # cross op: Q [4,16,1,64], memory [16,512,64], 128 steps
    n_src, steps = 512, 128
    c = ctx_factory(n_layers=1, n_heads=HEADS, max_sentences=1, n_beams=BEAMS, max_tgt=4, max_src=n_src)
    c.set_stream(stream.cuda_stream)
    Km, Vm = (torch.randn((HEADS, n_src, HEAD_DIM), generator=g, device=dev) for _ in range(2))
    c.set_memory(0, 0, n_src, Km, Vm, n_src * HEAD_DIM, HEAD_DIM)
    qc = torch.randn((steps, BEAMS, DMODEL), generator=g, device=dev)
    oc = torch.empty_like(qc)
    timed(lambda i: c.cross(0, 1, qc[i], oc[i]), 8)
    tt = timed(lambda i: c.cross(0, 1, qc[i], oc[i]), steps)
    c.sync()
    step_b = 2 * HEADS * n_src * ROW_BYTES + 2 * BEAMS * HEADS * ROW_BYTES
    res["cross_config"] = {
        "shape": "4 beams x 16 heads x 64 over memory [16,512,64], 128 steps",
        "gbs": round(step_b * steps / sum(tt) / 1e9, 1),
        "us_per_launch_mean": round(sum(tt) / steps * 1e6, 2),
        "frac_of_hbm_peak": round(step_b * steps / sum(tt) / 1e9 / hbm_peak, 4),
        "l2": "flushed (256 MB write) before every launch",
    }
    c.close()

    # prefill op: [8,16,128,64], key padding 0-31
    B, S = 8, 128
    c = ctx_factory(n_layers=0, n_heads=HEADS, max_sentences=0, n_beams=BEAMS, max_tgt=0, max_src=0)
    c.set_stream(stream.cuda_stream)
    qp, kp, vp = (torch.randn((B, HEADS, S, HEAD_DIM), generator=g, device=dev) for _ in range(3))
    op = torch.empty_like(qp)
    vl = (S - torch.randint(0, 32, (B,), generator=g, device=dev)).to(torch.int32)
    args = c.prefill_args(qp, kp, vp, op, B, HEADS, S, (HEADS * S * 64, S * 64, 64), vl)
    timed(lambda i: c.prefill(args), 5)
    tt = timed(lambda i: c.prefill(args), 50)
    c.sync()
    flops = 4 * B * HEADS * S * S * HEAD_DIM
    tmed = statistics.median(tt)
    res["prefill_config"] = {
        "shape": "Q,K,V [8,16,128,64], scale 1/8, last 0-31 keys masked",
        "tflops_dense": round(flops / tmed / 1e12, 2),
        "us_median": round(tmed * 1e6, 2),
        "path": "FFMA (fp32 SIMT)",
    }
    c.close()
    return res


def main():
    args = parse_args()
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    T = args.max_len
    workload = (f"decode self-attention over the per-beam KV cache, sentence-batched: "
                f"{args.sentences} sentences/GPU x {BEAMS} beams x {HEADS} heads x {HEAD_DIM}, fp32, "
                f"cache length 1->{T} with a random beam permutation (index reorder) before every step")
    config = {"workload": workload, "sentences_per_gpu": args.sentences, "beams": BEAMS,
              "heads": HEADS, "head_dim": HEAD_DIM, "cache_len": f"1..{T}",
              "step": f"one decode sweep of {T} steps (reorder + attention launch per step)",
              "l2": (f"inputs larger than L2: KV cache {args.sentences * 2 * BEAMS * HEADS * T * ROW_BYTES / 1e9:.2f} "
                     "GB per GPU at full length; no flush inside the sweep"),
              "parallelism": f"sentence-sharded x{args.gpus} (no collective on the data path)"}

    if args.impl == "reference":
        if rank != 0:
            return
        vals = []
        for _ in range(args.warmup):
            cpu_reference_rate(min(3.0, args.cpu_sample_s), T)
        for _ in range(args.steps):
            gbs, cores, sample, kind, dt = cpu_reference_rate(args.cpu_sample_s, T)
            vals.append((gbs, dt))
        value = statistics.median(v for v, _ in vals)
        line = {"metric": "decode-attn HBM GB/s", "value": round(value, 3), "unit": "GB/s",
                "impl": "reference", "n_gpus": args.gpus, "steps": args.steps,
                "warmup": args.warmup, "ms_per_step": round(statistics.median(d for _, d in vals) * 1e3, 1),
                "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
                "data": "synthetic", "config": config,
                "cpu_baseline": {"value": round(value, 3), "unit": "GB/s", "cores": cores,
                                 "kind": kind, "sample": sample},
                "e2e": {"value": round(value, 3), "unit": "GB/s", "h2d_bytes_per_step": 0,
                        "d2h_bytes_per_step": 0}}
        print(json.dumps(line), flush=True)
        return

    import torch
    import torch.distributed as dist
    if world > 1:
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local_rank))
    res, ops = run_ours(args, rank, world, local_rank)
    cpu = None
    if rank == 0 and world == 1:
        try:
            gbs, cores, sample, kind, _ = cpu_reference_rate(args.cpu_sample_s, T)
            cpu = {"value": round(gbs, 3), "unit": "GB/s", "cores": cores, "kind": kind, "sample": sample}
        except Exception as e:  # reported, not fatal
            cpu = {"value": None, "unit": "GB/s", "cores": host_threads(), "kind": "reference",
                   "sample": f"unavailable: {e}"}
    traffic = None
    tf = os.path.join(REPO, "profiles", "decode_self_traffic.json")
    if os.path.exists(tf):
        with open(tf) as f:
            traffic = json.load(f).get("dram_bytes_per_launch_scaled")
    if rank == 0:
        hbm = res["hbm_peak"]
        line = {
            "metric": "decode-attn HBM GB/s", "value": round(res["value"], 1), "unit": "GB/s",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(res["ms_per_step"], 3), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": config,
            "roofline": {"bound": "hbm", "achieved": round(res["kernel_gbs"], 1), "peak": hbm,
                         "unit": "GB/s", "frac": round(res["kernel_gbs"] / hbm, 4),
                         "traffic": traffic,
                         "kernel": "decode_self_kernel<4>",
                         "peak_kind": res["peak_kind"],
                         "how": "algorithmic bytes of one sweep / sum of CUDA-event durations of its "
                                f"{T} decode launches on the launching stream"},
            "cpu_baseline": cpu,
            "e2e": res["e2e"],
            "gpu_launches": 2 * T * args.steps,
            "clocks": res["clocks"],
        }
        if ops:
            line["ops"] = ops
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
