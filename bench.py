#!/usr/bin/env python3
"""Benchmark of the B200 attention path and translation engine of MetalNLLB.

Headline workload (one "step"): the sentence-batched translation -- 1024
sources of U[16,128] tokens (seed 4) translated with beam 4 and at most 128
target tokens on the synthetic NLLB-600M-shaped INT8 model, sharded by
sentence over the N GPUs (an LPT plan, no collective on the data path; total
work fixed: strong scaling).  Metric: translated tokens per second of the
whole job (emitted target tokens, EOS excluded, summed over ranks, divided
by the slowest rank's time).

The line also carries the attention kernels' HBM rates inside that
translation (decode self-attention and cross-attention, % of the measured
peak), the decode-attention sweep of 128 sentences per GPU and the three op
configurations (prefill, decode, cross) at their own sizes.

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
        self.i0, self.i1 = 0, None

    def start(self, ready_timeout: float = 5.0):
        """Start sampling and wait (bounded) for the first sample: nvidia-smi
        needs a few hundred ms before it reports, longer than a short timed
        region; call this before the region's barrier."""
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "50"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
            t_end = time.time() + ready_timeout
            while not self.lines and time.time() < t_end and self.proc.poll() is None:
                time.sleep(0.01)
        except (FileNotFoundError, OSError):
            self.proc = None
        return self

    def mark(self):
        """The timed region starts: later samples are the region's."""
        self.i0 = len(self.lines)

    def stop(self):
        """The timed region has ended: keep one more sample, then stop."""
        if self.proc:
            time.sleep(0.06)
            self.i1 = len(self.lines)
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def _read(self):
        for ln in self.proc.stdout:
            self.lines.append(ln.strip())

    def summary(self):
        sm, mx, reasons = [], None, set()
        names = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")
        for ln in self.lines[self.i0:self.i1]:
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
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=("ours", "reference"), default="ours")
    ap.add_argument("--sentences", type=int, default=128, help="sentences per GPU")
    ap.add_argument("--max-len", type=int, default=256, help="decode steps per sweep")
    ap.add_argument("--no-ops", action="store_true", help="skip the per-config op measurements")
    ap.add_argument("--cpu-sample-s", type=float, default=10.0)
    ap.add_argument("--translate-sentences", type=int, default=1024,
                    help="sentences of the sentence-batched translation")
    ap.add_argument("--no-sweep", action="store_true", help="skip the decode-attention sweep")
    ap.add_argument("--ncu-case", choices=("decode", "decode1", "cross", "cross128", "prefill", "linear", "linear512",
                                           "translate", "topk"),
                    help="run one small fixed case for an ncu capture and exit")
    return ap.parse_args()


# ---------------------------------------------------------------------------
# CPU reference (oracle/_ref: the reference's own decoder.c attention)
# ---------------------------------------------------------------------------
def host_threads() -> int:
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1


_REF_PER_SENT = {}  # (T, cores) -> seconds per sentence of the reference sweep (probe, once)


def cpu_reference_rate(target_s: float, T: int):
    """Times the reference's decoder_self_attn_cached sweep (bias-injected
    q/k/v, reorder by copy as main.c does) on all host threads, over a bounded
    number of sentences sized for about target_s seconds, and returns
    (GB/s, cores, sample description, kind, seconds)."""
    sys.path.insert(0, os.path.join(REPO, "oracle"))
    import pyoracle as po
    kind = "reference"
    lib = po.ref_lib() if po.ref_available() else None
    if lib is None:
        raise RuntimeError("oracle/_ref/libnllb_ref.so is not built")
    cores = host_threads()
    probe_sent = max(1, cores // BEAMS)
    if (T, cores) not in _REF_PER_SENT:
        _REF_PER_SENT[(T, cores)] = lib.ref_time_decode_sweep(probe_sent, BEAMS, T, cores, 7) / probe_sent
    per_sent = _REF_PER_SENT[(T, cores)]
    n_sent = max(probe_sent, min(256, int(target_s / max(per_sent, 1e-6))))
    dt = lib.ref_time_decode_sweep(n_sent, BEAMS, T, cores, 11)
    gbs = n_sent * sweep_bytes_per_sentence(T) / dt / 1e9
    sample = (f"{n_sent} sentence(s) x {BEAMS} beams x {HEADS} heads, cache 1->{T} with a "
              f"permutation reorder per step, {dt:.1f} s on {cores} threads")
    return gbs, cores, sample, kind, dt


# ---------------------------------------------------------------------------
# CPU reference of the headline: the reference program itself
# ---------------------------------------------------------------------------
REF_PROGRAM = os.path.join(REPO, "oracle", "_ref", "pico_nllb_g132")
REF_THREADS = 4  # the reference's NUM_THREADS (tensor.c:25-27): threads per program


def _watch_reference(proc, events):
    """Read the program's stdout and timestamp what the rate needs: the end
    of the encode ("[enc]" line) and each beam-search step (its "[beam] step"
    progress line, main.c:491)."""
    buf = b""
    while True:
        chunk = proc.stdout.read1(4096) if hasattr(proc.stdout, "read1") else proc.stdout.read(1)
        if not chunk:
            break
        buf += chunk
        while True:
            cut = min([i for i in (buf.find(b"\r"), buf.find(b"\n")) if i >= 0], default=-1)
            if cut < 0:
                break
            line, buf = buf[:cut].decode(errors="replace"), buf[cut + 1:]
            now = time.perf_counter()
            if line.startswith("[enc]"):
                events.append(("enc", now, line))
            elif line.startswith("[beam] step"):
                events.append(("step", now, line))
            elif line.startswith("best:"):
                events.append(("best", now, line))


def reference_program_rate(model_path: str, sources, window_s: float, procs: int):
    """The reference engine (its own main.c/loader.c/tensor.c/encoder.c/
    decoder.c compiled from its sources, MAX_GEN_LEN 132) on a bounded sample
    of the translation workload: `procs` programs run at once (each with the
    reference's 4 threads), one source each.  Each program is timed from its
    start to the end of its encode, then over `window_s` seconds of its beam
    search (one target token per hypothesis per step), and stopped there.
    Returns (tokens/s, details): per program, the rate of translating the
    whole sentence at the measured speeds -- max_out tokens (main.c:315-316)
    over encode time + max_out / step rate -- summed over the programs."""
    import re
    if not os.path.exists(REF_PROGRAM):
        raise RuntimeError("oracle/_ref/pico_nllb_g132 is not built")
    runs = []
    for src in sources[:procs]:
        args = [REF_PROGRAM, model_path, "eng_Latn", "fra_Latn"] + [str(t) for t in src[1:-1]]
        p = subprocess.Popen(args, stdout=subprocess.PIPE, stderr=subprocess.DEVNULL)
        ev = []
        th = threading.Thread(target=_watch_reference, args=(p, ev), daemon=True)
        th.start()
        runs.append((p, ev, th, len(src), time.perf_counter()))
    t_end = time.perf_counter() + 600.0
    while time.perf_counter() < t_end:
        ready = True
        for p, ev, _, _, _ in runs:
            enc = [t for k, t, _ in ev if k == "enc"]
            fin = p.poll() is not None
            if not fin and (not enc or time.perf_counter() < enc[0] + window_s):
                ready = False
        if ready:
            break
        time.sleep(0.05)
    total, per = 0.0, []
    for p, ev, th, n_src, t0 in runs:
        if p.poll() is None:
            p.kill()
        p.wait()
        th.join(timeout=5)
        enc = [t for k, t, _ in ev if k == "enc"]
        if not enc:
            raise RuntimeError("the reference program ended before its encode finished")
        steps = [(t, int(re.match(r"\[beam\] step (\d+)", ln).group(1))) for k, t, ln in ev if k == "step"]
        steps = [(t, st) for t, st in steps if t <= enc[0] + window_s]
        if len(steps) < 2:
            raise RuntimeError("the sample window saw fewer than two beam-search steps")
        step_rate = (len(steps) - 1) / (steps[-1][0] - steps[0][0])
        t_enc = enc[0] - t0  # process start, model load and encode
        max_out = min(3 * n_src + 10, 132 - 4)
        rate = max_out / (t_enc + max_out / step_rate)
        total += rate
        per.append({"n_src": n_src, "start_to_encoded_s": round(t_enc, 2), "steps_in_window": len(steps),
                    "step_rate": round(step_rate, 3), "tok_s": round(rate, 3)})
    return total, per


def reference_sample(step: int, procs: int, n_total: int = 1024):
    """Sources of the bounded sample of step `step`: `procs` consecutive
    sentences of the workload, a different group each step."""
    from nllb_attn import synth_model as sm
    srcs = sm.config4_sources(n_total)
    return [srcs[(step * procs + j) % n_total] for j in range(procs)]


# ---------------------------------------------------------------------------
# our arm
# ---------------------------------------------------------------------------
_HOST_CPUS_ALL = None  # the process's CPUs before bind_to_gpu_cpus


def bind_to_gpu_cpus(smi_index: str, pci_id: str = ""):
    """Keep this rank on the CPUs NVML names as closest to its GPU (found by
    PCI bus id, else by index), so that its pinned host buffers and copy
    launches stay on that socket; returns the number of CPUs kept, or None
    where NVML gives nothing usable."""
    try:
        import pynvml
        pynvml.nvmlInit()
        try:
            try:
                h = pynvml.nvmlDeviceGetHandleByPciBusId(pci_id.encode())
            except Exception:
                h = pynvml.nvmlDeviceGetHandleByIndex(int(smi_index))
            masks = pynvml.nvmlDeviceGetCpuAffinity(h, ((os.cpu_count() or 64) + 63) // 64)
        finally:
            pynvml.nvmlShutdown()
        cpus = {w * 64 + b for w, m in enumerate(masks) for b in range(64) if (int(m) >> b) & 1}
        global _HOST_CPUS_ALL
        before = os.sched_getaffinity(0)
        cpus &= before
        if cpus:
            _HOST_CPUS_ALL = before
            os.sched_setaffinity(0, cpus)
            return len(cpus)
    except Exception:
        pass
    return None


def measure_attention_sweep(args, rank, world, local_rank, host_cpus):
    """The decode-attention sweep: every rank's `args.sentences` sentences x
    4 beams x 16 heads x 64, cache 1 -> max_len with a random beam
    permutation (index reorder) before every step; algorithmic HBM bytes per
    second, summed over ranks (weak scaling), the dominant kernel alone, and
    the same sweep through the host-buffer C ABI."""
    import torch
    import torch.distributed as dist
    import nllb_attn as na

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

    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    n_sweeps = 5
    barrier()
    torch.cuda.synchronize(dev)
    with torch.cuda.stream(stream):
        e0.record(stream)
        for _ in range(n_sweeps):
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
    value = world * per_rank_bytes * n_sweeps / t_max / 1e9  # GB/s
    ms_per_step = t_max / n_sweeps * 1e3

    # dominant kernel alone: the same decode launches back to back (no reorder
    # kernels in between; identical bytes), events around the whole sweep
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    n_dec = 3
    with torch.cuda.stream(stream):
        a.record(stream)
        for _ in range(n_dec):
            for t in range(T):
                ctx.decode_self(0, t, S, q[t], k[t], v[t], out[t])
        b.record(stream)
    torch.cuda.synchronize(dev)
    dec_ms = a.elapsed_time(b) / n_dec
    kernel_gbs = per_rank_bytes / (dec_ms / 1e3) / 1e9
    hbm_peak, tflops_peak, peak_kind = load_peaks()

    # e2e through the host-buffer C ABI: H2D of q/k/v/parents, D2H of out, every launch
    e2e = None
    n_pool = 8
    # every host buffer pinned (torch.empty_like would not keep the pinning)
    qh, kh, vh, oh = (torch.empty((n_pool, S, BEAMS, DMODEL), pin_memory=True) for _ in range(4))
    for t_ in (qh, kh, vh):
        t_.normal_()
    ph = torch.empty((T, S, BEAMS), dtype=torch.int32, pin_memory=True)
    ph.copy_(torch.argsort(torch.rand((T, S, BEAMS)), dim=-1).to(torch.int32))
    qn, kn, vn, on, pn = qh.numpy(), kh.numpy(), vh.numpy(), oh.numpy(), ph.numpy()
    e2e_steps = 2
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
    if host_cpus:
        e2e["host_cpus_per_rank"] = host_cpus  # the rank's CPUs: those NVML names for its GPU

    traffic = None
    tf = os.path.join(REPO, "profiles", "decode_self_traffic.json")
    if os.path.exists(tf):
        with open(tf) as f:
            traffic = json.load(f).get("dram_bytes_per_launch_scaled")
    result = {
        "workload": (f"decode self-attention sweep: {S} sentences/GPU x {BEAMS} beams x {HEADS} heads x "
                     f"{HEAD_DIM}, fp32, cache 1->{T} with a random beam permutation (index reorder) before "
                     "every step; inputs resident in HBM (KV cache larger than L2)"),
        "gbs": round(value, 1), "unit": "GB/s", "scaling": "weak", "sweeps": n_sweeps,
        "ms_per_sweep": round(ms_per_step, 3),
        "roofline": {"bound": "hbm", "kernel": "decode_self_kernel<4>", "achieved": round(kernel_gbs, 1),
                     "peak": hbm_peak, "unit": "GB/s", "frac": round(kernel_gbs / hbm_peak, 4),
                     "traffic": traffic, "peak_kind": peak_kind,
                     "how": f"algorithmic bytes of one sweep / duration of its {T} decode launches run back to "
                            "back on the launching stream (CUDA events around 3 sweeps)"},
        "e2e": e2e,
    }
    ops = None
    if not args.no_ops and rank == 0 and world == 1:
        ops = measure_ops(ctx_factory=lambda **kw: na.Context(local_rank, **kw), dev=dev,
                          hbm_peak=hbm_peak)
    ctx.close()
    return result, ops


def graph_seconds(fn, stream, dev, reps=3):
    """Capture fn() (which launches on `stream`) in a CUDA graph and return the
    best of `reps` replays, timed with CUDA events on that stream."""
    import torch
    with torch.cuda.stream(stream):
        fn()
    torch.cuda.synchronize(dev)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        fn()
    best = None
    with torch.cuda.stream(stream):
        graph.replay()
        for _ in range(reps):
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record(stream)
            graph.replay()
            b.record(stream)
            torch.cuda.synchronize(dev)
            t = a.elapsed_time(b) * 1e-3
            best = t if best is None else min(best, t)
    del graph
    return best


def measure_ops(ctx_factory, dev, hbm_peak, tflops_note=""):
    """The three op configurations at their own sizes.  Each is one CUDA graph
    replaying the configuration over R independent instances in rotation, so
    that consecutive launches touch disjoint data and the working set exceeds
    the 126 MB L2 (no flush kernel inside the timed region)."""
    import torch
    stream = torch.cuda.Stream(device=dev)
    g = torch.Generator(device=dev)
    g.manual_seed(2)
    res = {}

    # decode op: 4 beams x 16 heads x 64, cache 1->256, permutation before each step
    T, R = 256, 24
    ctxs = [ctx_factory(n_layers=1, n_heads=HEADS, max_sentences=1, n_beams=BEAMS, max_tgt=T,
                        max_src=1) for _ in range(R)]
    for c in ctxs:
        c.set_stream(stream.cuda_stream)
    q, k, v = (torch.randn((R, T, BEAMS, DMODEL), generator=g, device=dev) for _ in range(3))
    out = torch.empty_like(q)
    par = torch.argsort(torch.rand((R, T, BEAMS), generator=g, device=dev), dim=-1).to(torch.int32)

    def dec_sweep():
        for t in range(T):
            for r, c in enumerate(ctxs):
                c.reorder(1, par[r, t])
                c.decode_self(0, t, 1, q[r, t], k[r, t], v[r, t], out[r, t])

    t_all = graph_seconds(dec_sweep, stream, dev)
    for c in ctxs:
        c.sync()
        c.close()
    tot = R * sweep_bytes_per_sentence(T)
    res["decode_self_config"] = {
        "shape": "1 sentence x 4 beams x 16 heads x 64, cache 1->256, permutation reorder before every step",
        "gbs": round(tot / t_all / 1e9, 1),
        "frac_of_hbm_peak": round(tot / t_all / 1e9 / hbm_peak, 4),
        "us_per_step": round(t_all / (T * R) * 1e6, 2),
        "how": f"CUDA graph of the sweep over {R} independent sentences in rotation "
               f"({R * 2 * BEAMS * HEADS * T * ROW_BYTES / 1e6:.0f} MB of cache > L2); "
               "a step = reorder + decode launch",
    }
    del q, k, v, out

    # cross op: Q [4,16,1,64] over memory [16,512,64], 128 steps
    n_src, steps, R = 512, 128, 32
    ctxs = [ctx_factory(n_layers=1, n_heads=HEADS, max_sentences=1, n_beams=BEAMS, max_tgt=4,
                        max_src=n_src) for _ in range(R)]
    mems = []
    for c in ctxs:
        c.set_stream(stream.cuda_stream)
        Km, Vm = (torch.randn((HEADS, n_src, HEAD_DIM), generator=g, device=dev) for _ in range(2))
        with torch.cuda.stream(stream):
            c.set_memory(0, 0, n_src, Km, Vm, n_src * HEAD_DIM, HEAD_DIM)
        mems.append((Km, Vm))
    qc = torch.randn((R, steps, BEAMS, DMODEL), generator=g, device=dev)
    oc = torch.empty_like(qc)

    def cross_steps():
        for i in range(steps):
            for r, c in enumerate(ctxs):
                c.cross(0, 1, qc[r, i], oc[r, i])

    t_all = graph_seconds(cross_steps, stream, dev)
    for c in ctxs:
        c.sync()
        c.close()
    step_b = 2 * HEADS * n_src * ROW_BYTES + 2 * BEAMS * HEADS * ROW_BYTES
    res["cross_config"] = {
        "shape": "4 beams x 16 heads x 64 over memory [16,512,64], 128 steps",
        "gbs": round(R * steps * step_b / t_all / 1e9, 1),
        "frac_of_hbm_peak": round(R * steps * step_b / t_all / 1e9 / hbm_peak, 4),
        "us_per_step": round(t_all / (steps * R) * 1e6, 2),
        "how": f"CUDA graph of 128 steps over {R} independent memories in rotation "
               f"({R * 2 * HEADS * n_src * ROW_BYTES / 1e6:.0f} MB > L2)",
    }
    del mems, qc, oc

    # prefill op: [8,16,128,64], key padding 0-31
    B, S, R = 8, 128, 16
    c = ctx_factory(n_layers=0, n_heads=HEADS, max_sentences=0, n_beams=BEAMS, max_tgt=0, max_src=0)
    c.set_stream(stream.cuda_stream)
    qp, kp, vp = (torch.randn((R, B, HEADS, S, HEAD_DIM), generator=g, device=dev) for _ in range(3))
    op = torch.empty_like(qp)
    vl = (S - torch.randint(0, 32, (R, B), generator=g, device=dev)).to(torch.int32)
    args = [c.prefill_args(qp[r], kp[r], vp[r], op[r], B, HEADS, S, (HEADS * S * 64, S * 64, 64), vl[r])
            for r in range(R)]

    def prefill_rounds():
        for _ in range(4):
            for a in args:
                c.prefill(a)

    t_all = graph_seconds(prefill_rounds, stream, dev)
    c.sync()
    c.close()
    flops = 4 * B * HEADS * S * S * HEAD_DIM
    per = t_all / (4 * R)
    res["prefill_config"] = {
        "shape": "Q,K,V [8,16,128,64], scale 1/8, last 0-31 keys masked",
        "tflops_dense": round(flops / per / 1e12, 2),
        "us_per_launch": round(per * 1e6, 2),
        "how": f"CUDA graph of 4 rounds over {R} independent inputs ({R * 4 * 16.8:.0f} MB > L2)",
    }
    return res


def _synth_model_path() -> str:
    from nllb_attn import synth_model as sm
    return sm.default_model_path(0)


SYNTH_MODEL = _synth_model_path()


def config4_sources(n: int = 1024, seed: int = 4):
    """Sentence-batched translation workload (nllb_attn.synth_model.config4_sources)."""
    from nllb_attn import synth_model as sm
    return sm.config4_sources(n, seed)


def reference_translate_rate(model_path: str):
    """The reference engine (its own main.c, compiled from its sources) on the
    single-sentence configuration: tokens/s as it reports them (decode time)."""
    import re
    from nllb_attn import synth_model as sm
    exe = os.path.join(REPO, "oracle", "_ref", "pico_nllb_g36")
    if not os.path.exists(exe):
        return None
    src = sm.source_ids(0, 16)
    out = subprocess.run([exe, model_path, "eng_Latn", "fra_Latn"] + [str(t) for t in src[1:-1]],
                         capture_output=True, text=True, timeout=600).stdout
    m = re.search(r"^best: (\d+) tokens, score=[-0-9.]+, enc=(\d+)ms, dec=(\d+)ms, ([0-9.]+) tok/s", out, re.M)
    if not m:
        return None
    n, enc, dec = int(m.group(1)), int(m.group(2)), int(m.group(3))
    return {"tok_s_decode": float(m.group(4)), "tok_s_total": round(n / ((enc + dec) / 1e3), 3),
            "tokens": n, "cores": 4, "kind": "reference",
            "sample": "one 16-token sentence, beam 4, 32 target tokens, NUM_THREADS=4 (the reference's default)"}


def translation_bytes(shard, G=132):
    """Host bytes of one nllb_translate call through the public API: sources
    and offsets in; token ids [n][max_gen], lengths and scores out."""
    h2d = 4 * (sum(len(x) for x in shard) + len(shard) + 1)
    d2h = 4 * (len(shard) * G + 2 * len(shard))
    return h2d, d2h


def measure_translation(args, rank, world, local_rank, smi_index, host_cpus):
    """The headline: translated tokens/s of the sentence-batched workload,
    sharded by sentence over the ranks (no collective on the data path).

    value: K translate calls of the rank's shard back to back, timed with
    CUDA events (the model, its weights and caches resident in HBM; each call
    is synchronous), max over ranks; tokens summed over ranks.
    e2e: the same through the Python API a user calls (source lists in, token
    lists out, host buffers), wall clock, max over ranks.
    profile: one more call with nllb_translate_profile on: per kernel class
    its launches, time and algorithmic work -> the roofline of the dominant
    class and the attention kernels' HBM rates inside the translation."""
    import torch
    import torch.distributed as dist
    import nllb_attn as na
    from nllb_attn import sharding, synth_model as sm

    dev = torch.device("cuda", local_rank)
    if local_rank == 0:
        sm.ensure_model(SYNTH_MODEL, seed=0)
    if world > 1:
        dist.barrier()
    sources = config4_sources(args.translate_sentences)
    shards = sharding.plan_shards([len(x) for x in sources], world, max_gen=132)
    mine = [sources[i] for i in shards[rank]]
    tgt = sm.LANG["fra_Latn"]

    def barrier():
        if world > 1:
            dist.barrier()

    def max_over_ranks(x):
        t = torch.tensor([x], dtype=torch.float64, device=dev)
        if world > 1:
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    def sum_over_ranks(x):
        t = torch.tensor([x], dtype=torch.float64, device=dev)
        if world > 1:
            dist.all_reduce(t, op=dist.ReduceOp.SUM)
        return float(t.item())

    res = {}
    with na.Model(SYNTH_MODEL, device=local_rank, max_sentences=max(1, len(mine)), max_src=132,
                  max_gen=132) as m:
        if world == 1:
            src0 = sm.source_ids(0, 16)
            m.translate([src0], tgt, max_gen=36)  # warm-up
            best = None
            for _ in range(3):
                _, _, st = m.translate([src0], tgt, max_gen=36)
                if best is None or st.decode_ms < best.decode_ms:
                    best = st
            res["config0"] = {
                "workload": "one 16-token sentence, beam 4, 32 target tokens (main.c rules)",
                "tokens": int(best.tokens_out),
                "tok_s_decode": round(best.tokens_out / (best.decode_ms / 1e3), 1),
                "tok_s_total": round(best.tokens_out / ((best.encode_ms + best.decode_ms) / 1e3), 1),
                "ms_encode": round(best.encode_ms, 2), "ms_decode": round(best.decode_ms, 2)}
        for _ in range(args.warmup):
            m.translate(mine, tgt, max_gen=132)
        # ---- timed region: K calls, CUDA events, clocks sampled
        clk = ClockSampler(smi_index).start()
        barrier()
        torch.cuda.synchronize(dev)
        clk.mark()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        tokens = 0
        for _ in range(args.steps):
            _, _, st = m.translate(mine, tgt, max_gen=132)
            tokens += int(st.tokens_out)
        e1.record()
        torch.cuda.synchronize(dev)
        clk.stop()
        barrier()
        t_dev = max_over_ranks(e0.elapsed_time(e1) / 1e3)
        tok_all = sum_over_ranks(tokens)
        res["value"] = tok_all / t_dev
        res["ms_per_step"] = t_dev / args.steps * 1e3
        res["tokens_per_step"] = tok_all / args.steps
        res["clocks"] = clk.summary()
        # ---- e2e through the public API (host lists in and out), wall clock
        e2e_calls = 2
        barrier()
        t0 = time.perf_counter()
        tok_e2e = 0
        for _ in range(e2e_calls):
            toks, _, _ = m.translate([list(x) for x in mine], tgt, max_gen=132)
            tok_e2e += sum(len(t) for t in toks)
        t_e2e = max_over_ranks(time.perf_counter() - t0)
        tok_e2e = sum_over_ranks(tok_e2e)
        h2d = sum_over_ranks(translation_bytes(mine)[0])
        d2h = sum_over_ranks(translation_bytes(mine)[1])
        res["e2e"] = {"value": round(tok_e2e / t_e2e, 1), "unit": "tokens/s",
                      "h2d_bytes_per_step": int(h2d), "d2h_bytes_per_step": int(d2h),
                      "how": "nllb_translate through the Python API (source id lists in, token id lists out, "
                             f"host buffers), {e2e_calls} calls, wall clock, max over ranks"}
        if host_cpus:
            res["e2e"]["host_cpus_per_rank"] = host_cpus
        # ---- kernel classes of one call (events around every launch of a class)
        m.profile(True)
        m.translate(mine, tgt, max_gen=132)
        prof = m.profile_read()
        m.profile(False)
    res["profile"] = prof
    res["shard"] = {"sentences": len(mine), "source_tokens": sum(len(x) for x in mine)}
    return res, sources


def _gemm_traffic_sample():
    """DRAM traffic of one captured launch of the GEMM kernel against its
    algorithmic bytes (profiles/gemm_pair_traffic.json): the class's launches
    differ in shape, so no single per-launch traffic figure stands for them."""
    tf = os.path.join(REPO, "profiles", "gemm_pair_traffic.json")
    if not os.path.exists(tf):
        return None
    with open(tf) as f:
        d = json.load(f)
    return {"kernel": d["kernel"], "shape": d["shape"],
            "dram_bytes": d["dram_bytes_read"] + d["dram_bytes_write"],
            "algorithmic_bytes": d["algorithmic_bytes"], "ratio": d["ratio"]}


def roofline_from_profile(prof, hbm_peak, tflops_sust, peak_kind):
    """The dominant kernel class of the translation (largest summed time):
    its algorithmic rate against the measured peak; the attention classes'
    HBM rates beside it."""
    total = sum(v["ms"] for v in prof.values()) or 1.0
    top = max(prof, key=lambda k: prof[k]["ms"])
    v = prof[top]
    if v["flops"] > 0:
        ach = v["flops"] / (v["ms"] / 1e3) / 1e12
        roof = {"bound": "tensor", "achieved": round(ach, 1), "peak": tflops_sust, "unit": "TFLOP/s",
                "frac": round(ach / tflops_sust, 4),
                "note": "dense FLOPs 2*M*N*K of the linear layers; each product runs as two fp16 MMAs "
                        "(activations split into two fp16 parts), so the tensor pipe does 2x this work",
                "mma_frac": round(2 * ach / tflops_sust, 4),
                "peak_which": "bf16_tflops_sustained (kernel timed inside a long run)"}
    else:
        ach = v["bytes"] / (v["ms"] / 1e3) / 1e9
        roof = {"bound": "hbm", "achieved": round(ach, 1), "peak": hbm_peak, "unit": "GB/s",
                "frac": round(ach / hbm_peak, 4)}
    roof.update({"kernel_class": top, "share_of_kernel_time": round(v["ms"] / total, 4),
                 "launches": v["launches"], "avg_launch_us": round(v["ms"] / max(1, v["launches"]) * 1e3, 2),
                 "traffic": None, "traffic_sample": _gemm_traffic_sample() if v["flops"] > 0 else None,
                 "peak_kind": peak_kind,
                 "how": "algorithmic work of the class's launches / their summed durations, CUDA events "
                        "around each launch on the engine's stream in one profiled call of the same shard"})
    classes = {}
    for k, c in prof.items():
        if not c["launches"]:
            continue
        e = {"launches": c["launches"], "ms": round(c["ms"], 2), "share": round(c["ms"] / total, 4)}
        if c["flops"]:
            e["tflops"] = round(c["flops"] / (c["ms"] / 1e3) / 1e12, 1)
        if c["bytes"] and k in ("decode_self", "cross", "logsoftmax_topk"):
            gbs = c["bytes"] / (c["ms"] / 1e3) / 1e9
            e["gbs"] = round(gbs, 1)
            e["frac_of_hbm_peak"] = round(gbs / hbm_peak, 4)
        classes[k] = e
    return roof, classes


def ncu_case(which: str) -> None:
    """Small, fixed cases for ncu captures (a few launches of one kernel each)."""
    import torch
    import nllb_attn as na
    dev = torch.device("cuda:0")
    g = torch.Generator(device=dev)
    g.manual_seed(5)
    if which == "decode":
        # 32 sentences x 4 beams x 16 heads, sweep to length 256 (last launches: 268 MB > L2)
        S, T = 32, 256
        c = na.Context(0, n_layers=1, max_sentences=S, n_beams=BEAMS, max_tgt=T, max_src=1)
        q, k, v = (torch.randn((S, BEAMS, DMODEL), generator=g, device=dev) for _ in range(3))
        out = torch.empty_like(q)
        par = torch.argsort(torch.rand((S, BEAMS), generator=g, device=dev), -1).to(torch.int32)
        for t in range(T):
            c.reorder(S, par)
            c.decode_self(0, t, S, q, k, v, out)
    elif which == "decode1":
        # one sentence (the decode-op configuration), sweep to length 256
        T = 256
        c = na.Context(0, n_layers=1, max_sentences=1, n_beams=BEAMS, max_tgt=T, max_src=1)
        q, k, v = (torch.randn((BEAMS, DMODEL), generator=g, device=dev) for _ in range(3))
        out = torch.empty_like(q)
        par = torch.argsort(torch.rand((1, BEAMS), generator=g, device=dev), -1).to(torch.int32)
        for t in range(T):
            c.reorder(1, par)
            c.decode_self(0, t, 1, q, k, v, out)
    elif which == "cross":
        c = na.Context(0, n_layers=1, max_sentences=1, n_beams=BEAMS, max_tgt=4, max_src=512)
        Km, Vm = (torch.randn((HEADS, 512, HEAD_DIM), generator=g, device=dev) for _ in range(2))
        c.set_memory(0, 0, 512, Km, Vm, 512 * HEAD_DIM, HEAD_DIM)
        qc = torch.randn((BEAMS, DMODEL), generator=g, device=dev)
        oc = torch.empty_like(qc)
        for _ in range(3):
            c.cross(0, 1, qc, oc)
    elif which == "linear":
        # INT8 linear on the engine's path (weights prepared once, TMA-fed tcgen05):
        # 256 rows x 1024 -> 1024 (split-K cluster kernel), then the vocabulary
        # projection 256 x 1024 -> 256206 (persistent kernel); 3 launches each
        x = torch.randn((256, 1024), generator=g, device=dev)
        for n_out in (1024, 256206):
            w = torch.randint(-127, 128, (n_out, 1024), generator=g, device=dev, dtype=torch.int8)
            sc = torch.full((n_out,), 3666.19, device=dev)
            with na.PreparedLinear(w, sc) as lin:
                for _ in range(3):
                    lin(x)
                torch.cuda.synchronize()
                assert lin.status() == 0
        print("ncu case linear: ok")
        return
    elif which == "linear512":
        # the decoder's linear layers at 512 rows (a step of 128 sentences x 4 beams, the
        # per-GPU share of config 4 on 8 GPUs): 1024 -> 3072 (q/k/v), 1024 -> 1024 (output),
        # 1024 -> 4096 (fc1), 4096 -> 1024 (fc2); 3 launches each
        for n_in, n_out in ((1024, 3072), (1024, 1024), (1024, 4096), (4096, 1024)):
            x = torch.randn((512, n_in), generator=g, device=dev)
            w = torch.randint(-127, 128, (n_out, n_in), generator=g, device=dev, dtype=torch.int8)
            sc = torch.full((n_out,), 3666.19, device=dev)
            with na.PreparedLinear(w, sc) as lin:
                for _ in range(3):
                    lin(x)
                torch.cuda.synchronize()
                assert lin.status() == 0
        print("ncu case linear512: ok")
        return
    elif which == "translate":
        # the translation engine on 64 sentences of config 4's workload, 40 target tokens at most
        # (after a 4-sentence warm-up): the launch list of a decode-dominated run
        from nllb_attn import synth_model as sm
        sm.ensure_model(SYNTH_MODEL, seed=0)
        srcs = config4_sources(1024)[:64]
        with na.Model(SYNTH_MODEL, device=0, max_sentences=64, max_src=132, max_gen=132) as m:
            m.translate(srcs[:4], sm.LANG["fra_Latn"], max_gen=8)
            _, _, st = m.translate(srcs, sm.LANG["fra_Latn"], max_gen=40)
        print(f"ncu case translate: ok, {st.tokens_out} tokens in {st.steps} steps")
        return
    elif which == "cross128":
        # cross-attention at the 8-GPU shard's size: 128 sentences x 4 beams, memories of 18..130
        # rows (config 4's source lengths + 2), written once; 3 calls
        n = 128
        lens = [int(len(x)) for x in config4_sources(n)]
        c = na.Context(0, n_layers=1, max_sentences=n, n_beams=BEAMS, max_tgt=4, max_src=max(lens))
        for s_, L in enumerate(lens):
            Km, Vm = (torch.randn((L, DMODEL), generator=g, device=dev) for _ in range(2))
            c.set_memory(0, s_, L, Km, Vm, HEAD_DIM, DMODEL)
        qc = torch.randn((n, BEAMS, DMODEL), generator=g, device=dev)
        oc = torch.empty_like(qc)
        for _ in range(3):
            c.cross(0, n, qc, oc)
    elif which == "topk":
        # log-softmax + top-8 over the vocabulary for 512 rows (a decode step of
        # 128 sentences x 4 beams): 525 MB of logits > L2; 3 calls
        V, R = 256206, 512
        logits = torch.randn((R, V), generator=g, device=dev) * 3.0
        for _ in range(3):
            na.logsoftmax_topk(logits, 8)
        torch.cuda.synchronize()
        print("ncu case topk: ok")
        return
    elif which == "prefill":
        B, S = 8, 128
        c = na.Context(0, n_layers=0, max_sentences=0)
        qp, kp, vp = (torch.randn((B, HEADS, S, HEAD_DIM), generator=g, device=dev) for _ in range(3))
        op = torch.empty_like(qp)
        vl = (S - torch.randint(0, 32, (B,), generator=g, device=dev)).to(torch.int32)
        a = c.prefill_args(qp, kp, vp, op, B, HEADS, S, (HEADS * S * 64, S * 64, 64), vl)
        for _ in range(3):
            c.prefill(a)
    else:
        raise SystemExit(f"unknown --ncu-case {which}")
    c.sync()
    c.close()
    print(f"ncu case {which}: ok")


_RESULT_FD = None


def emit(line: dict) -> None:
    """Write the one JSON result line to the process's original stdout."""
    text = json.dumps(line) + "\n"
    if _RESULT_FD is None:
        sys.stdout.write(text)
        sys.stdout.flush()
    else:
        os.write(_RESULT_FD, text.encode())


def main():
    global _RESULT_FD
    args = parse_args()
    if not args.ncu_case:
        # Libraries (NCCL's version banner, CUDA, torch) may print on stdout;
        # keep stdout for the result line alone and send the rest to stderr.
        sys.stdout.flush()
        _RESULT_FD = os.dup(1)
        os.dup2(2, 1)
    if args.ncu_case:
        ncu_case(args.ncu_case)
        return
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    n_sent = args.translate_sentences
    config = {"workload": (f"sentence-batched translation: {n_sent} sources of U[16,128] tokens (ids U[4,256000), "
                           "seed 4), beam 4, at most 128 target tokens (main.c rules), synthetic "
                           "NLLB-600M-shaped INT8 model (random init, seed 0)"),
              "sentences": n_sent, "beam": BEAMS, "max_target_tokens": 128, "d_model": DMODEL, "heads": HEADS,
              "layers": "12 encoder + 12 decoder", "ffn": 4096, "vocab": 256206,
              "step": f"one translation of the rank's shard of the {n_sent} sentences",
              "l2": "inputs larger than L2: 1.8 GB of weights and the KV caches are read every step",
              "parallelism": f"sentence-sharded x{args.gpus} (LPT plan, no collective on the data path)"}
    metric = "translated tokens/sec"

    if args.impl == "reference":
        if rank != 0:
            return
        # each step a bounded sample of the workload: procs programs on
        # consecutive sentences, encode + a short beam-search window each
        from nllb_attn import synth_model as sm
        sm.ensure_model(SYNTH_MODEL, seed=0)
        procs = max(1, host_threads() // REF_THREADS)
        window = max(1.0, min(3.0, 90.0 / max(1, args.steps)))
        for w_ in range(args.warmup):
            reference_program_rate(SYNTH_MODEL, reference_sample(10_000 + w_, 1), 0.5, 1)
        vals, secs = [], []
        for k_ in range(args.steps):
            t0 = time.perf_counter()
            v, per = reference_program_rate(SYNTH_MODEL, reference_sample(k_, procs), window, procs)
            secs.append(time.perf_counter() - t0)
            vals.append(v)
        value = statistics.median(vals)
        sample = (f"per step {procs} reference programs at once ({REF_THREADS} threads each, "
                  f"{procs * REF_THREADS} threads in all) on {procs} consecutive sentences of the workload; each "
                  f"timed from start to the end of its encode, then over a {window:.1f} s window of beam-search "
                  "steps; tokens/s of translating each whole sentence (max_out tokens) at those speeds, summed")
        line = {"metric": metric, "value": round(value, 3), "unit": "tokens/s", "impl": "reference",
                "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
                "ms_per_step": round(statistics.median(secs) * 1e3, 1), "higher_is_better": True,
                "scaling": "strong", "vs_baseline": None, "dtype": "f32", "data": "synthetic", "config": config,
                "cpu_baseline": {"value": round(value, 3), "unit": "tokens/s", "cores": procs * REF_THREADS,
                                 "kind": "reference", "sample": sample},
                "e2e": {"value": round(value, 3), "unit": "tokens/s", "h2d_bytes_per_step": 0,
                        "d2h_bytes_per_step": 0}}
        emit(line)
        return

    import torch
    import torch.distributed as dist
    if world > 1:
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local_rank))
    vis = os.environ.get("CUDA_VISIBLE_DEVICES", "")
    smi_index = vis.split(",")[local_rank] if vis else str(local_rank)
    # each rank on its GPU's socket (the CPU baseline, later, gets all CPUs back)
    props = torch.cuda.get_device_properties(local_rank)
    pci_id = f"{props.pci_domain_id:08X}:{props.pci_bus_id:02X}:{props.pci_device_id:02X}.0"
    host_cpus = bind_to_gpu_cpus(smi_index, pci_id)
    torch.cuda.set_device(local_rank)

    tr, sources = measure_translation(args, rank, world, local_rank, smi_index, host_cpus)
    hbm_peak, tflops_peak, peak_kind = load_peaks()
    tflops_sust = tflops_peak
    pk = os.path.join(REPO, "MEASURED_PEAKS.json")
    if os.path.exists(pk):
        with open(pk) as f:
            tflops_sust = float(json.load(f).get("bf16_tflops_sustained", tflops_peak))
    sweep, ops = (None, None)
    if not args.no_sweep:
        sweep, ops = measure_attention_sweep(args, rank, world, local_rank, host_cpus)
    cpu = None
    if rank == 0 and world == 1:
        try:
            if _HOST_CPUS_ALL:
                os.sched_setaffinity(0, _HOST_CPUS_ALL)  # the CPU baseline uses every host CPU
            procs = max(1, host_threads() // REF_THREADS)
            v, per = reference_program_rate(SYNTH_MODEL, reference_sample(0, procs), args.cpu_sample_s, procs)
            cpu = {"value": round(v, 3), "unit": "tokens/s", "cores": procs * REF_THREADS, "kind": "reference",
                   "sample": (f"{procs} reference programs at once ({REF_THREADS} threads each) on the first "
                              f"{procs} sentences of the workload, each timed from start to the end of its encode "
                              f"and over a {args.cpu_sample_s:.0f} s window of beam-search steps; tokens/s of "
                              "translating each whole sentence at those speeds, summed"),
                   "per_program": per}
        except Exception as e:  # reported, not fatal
            cpu = {"value": None, "unit": "tokens/s", "cores": host_threads(), "kind": "reference",
                   "sample": f"unavailable: {e}"}
    if rank == 0:
        roof, classes = roofline_from_profile(tr["profile"], hbm_peak, tflops_sust, peak_kind)
        launches = sum(c["launches"] for c in tr["profile"].values())
        line = {
            "metric": metric, "value": round(tr["value"], 1), "unit": "tokens/s",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(tr["ms_per_step"], 2), "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": config,
            "roofline": roof,
            "cpu_baseline": cpu,
            "e2e": tr["e2e"],
            # our kernels launched in the timed region: rank 0's profiled call's launches (every
            # class is one kernel launch) x steps x ranks (the shards are alike)
            "gpu_launches": int(launches * args.steps * world),
            "clocks": tr["clocks"],
            "tokens_per_step": tr["tokens_per_step"],
            "shard_rank0": tr["shard"],
            "kernel_classes_rank0": classes,
            "decode_attn_in_translation": {
                k: classes[k] for k in ("decode_self", "cross") if k in classes},
        }
        if "config0" in tr:
            line["config0"] = tr["config0"]
            ref0 = reference_translate_rate(SYNTH_MODEL) if world == 1 else None
            if ref0:
                line["config0"]["reference_cpu"] = ref0
        if sweep:
            line["decode_attn_sweep"] = sweep
        if ops:
            line["ops"] = ops
        emit(line)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
