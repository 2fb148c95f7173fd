#!/usr/bin/env python
"""Benchmark of the GDN decode hot path (config 4 at N=8).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

One process per GPU (torchrun for N > 1).  A step is one decode of one token for
every (sequence, v-head) of the rank's batch: B=256 sequences per rank, Hq=16,
Hv=32, d=128, fp32 state in the k-last layout.  Scaling is weak: each rank owns
its own 256 sequences and their states (sharding by sequence, no collective on
the data path), so at N=8 the job is BASELINE config 4 (B=2048).

Metric: decode state-stream throughput in GB/s, counted with the algorithmic
131,844 bytes per (sequence, v-head) per step (2 x 64 KiB state + q/k share + v +
o + gates), summed over ranks and divided by the max-over-ranks device time of
the K timed steps.  ``ms_per_step`` is that time per step; ``decode_us_per_step``
the same in microseconds.  The state ping-pongs between two 512 MiB buffers per
rank, larger than the 126 MB L2, so no step reads a cached state.

Extra keys: ``roofline`` (dominant kernel vs the measured HBM copy peak),
``cpu_baseline`` (the C restatement of the reference recurrence on the host
cores, rank 0 at N=1), ``e2e`` (the public ``gdn_b200.decode.run`` call with
per-step inputs copied from pinned host memory and the output read back),
``clocks`` (SM clocks sampled through NVML during the timed region), and
``prefill`` (chunked prefill tokens/s on BASELINE config 3's shape, heads
sharded over ranks).

``--impl reference`` times the reference's CPU implementation of the same
step (the C restatement of definitions/gdn/gdn_decode_qk4_v8_d128_k_last.md:61-133
in oracle/gdn_oracle.c, all host threads) on rank 0 and prints the same line
with ``"impl": "reference"``.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import sys
import threading
import time
from datetime import timedelta
from pathlib import Path

REPO = Path(__file__).resolve().parent
sys.path.insert(0, str(REPO / "mlsys-flashlinfer-contest_b200"))
sys.path.insert(0, str(REPO))

import torch  # noqa: E402

HQ, HV, D = 16, 32, 128
B_PER_RANK = 256
UNIT_BYTES = 2 * D * D * 4 + D * 2 + D * 2 + D * 2 + 4  # 131,844 B per (seq, v-head)
METRIC = "gdn_decode_state_GBps"
UNIT = "GB/s"


def env_int(name, default):
    try:
        return int(os.environ.get(name, default))
    except ValueError:
        return default


# ---------------------------------------------------------------- clocks
class ClockSampler:
    """Polls SM clock, max clock and clock-event reasons through NVML."""

    REASONS = {
        0x1: "gpu_idle", 0x2: "applications_clocks_setting", 0x4: "sw_power_cap",
        0x8: "hw_slowdown", 0x10: "sync_boost", 0x20: "sw_thermal_slowdown",
        0x40: "hw_thermal_slowdown", 0x80: "hw_power_brake_slowdown",
        0x100: "display_clock_setting",
    }

    def __init__(self, device_index: int, period_s: float = 0.005):
        self.samples, self.reasons = [], 0
        self.period = period_s
        self.ok = False
        self._stop = threading.Event()
        try:
            import pynvml
            pynvml.nvmlInit()
            idx = device_index
            vis = os.environ.get("CUDA_VISIBLE_DEVICES")
            if vis:
                parts = [p.strip() for p in vis.split(",") if p.strip()]
                if device_index < len(parts) and parts[device_index].isdigit():
                    idx = int(parts[device_index])
            self.h = pynvml.nvmlDeviceGetHandleByIndex(idx)
            self.nv = pynvml
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self.h, pynvml.NVML_CLOCK_SM)
            self.ok = True
        except Exception as e:  # pragma: no cover - depends on the box
            self.err = repr(e)

    def _run(self):
        nv = self.nv
        while not self._stop.is_set():
            try:
                self.samples.append(nv.nvmlDeviceGetClockInfo(self.h, nv.NVML_CLOCK_SM))
                try:
                    r = nv.nvmlDeviceGetCurrentClocksEventReasons(self.h)
                except AttributeError:
                    r = nv.nvmlDeviceGetCurrentClocksThrottleReasons(self.h)
                self.reasons |= int(r)
            except Exception:
                pass
            time.sleep(self.period)

    def __enter__(self):
        if self.ok:
            self.t = threading.Thread(target=self._run, daemon=True)
            self.t.start()
        return self

    def __exit__(self, *exc):
        if self.ok:
            self._stop.set()
            self.t.join()

    def summary(self):
        if not self.ok:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "note": "nvml unavailable"}
        names = [n for bit, n in self.REASONS.items() if self.reasons & bit]
        return {"sm_mhz": statistics.median(self.samples) if self.samples else None,
                "sm_max_mhz": self.max_mhz, "reasons": names, "samples": len(self.samples)}


# ---------------------------------------------------------------- helpers
def measured_peaks():
    p = REPO / "MEASURED_PEAKS.json"
    if p.exists():
        try:
            d = json.loads(p.read_text())
            return float(d["hbm_gbs"]), float(d.get("bf16_tflops", 1590.0)), \
                float(d.get("bf16_tflops_sustained", 1400.0)), "measured"
        except Exception:
            pass
    return 6650.0, 1590.0, 1400.0, "fallback"


def profiled_traffic(name: str):
    """dram bytes per launch from a committed ncu summary (profiles/<name>),
    a line 'dram_bytes_per_launch: <int>'."""
    p = REPO / "profiles" / name
    if not p.exists():
        return None
    for line in p.read_text().splitlines():
        if line.strip().startswith("dram_bytes_per_launch:"):
            try:
                return int(float(line.split(":", 1)[1].split()[0]))
            except ValueError:
                return None
    return None


def cpu_count_info():
    n = os.cpu_count() or 1
    model = ""
    try:
        for line in open("/proc/cpuinfo"):
            if line.startswith("model name"):
                model = line.split(":", 1)[1].strip()
                break
    except OSError:
        pass
    return n, model


def time_cpu_decode(budget_s: float = 10.0, max_steps: int = 400):
    """The C restatement of the reference decode on the host cores, on the same
    B=256 x Hv=32 workload; repeats full steps until the budget is spent."""
    from oracle import c_oracle
    from gdn_b200 import workloads as W
    inp = W.make_decode_inputs(B_PER_RANK, HQ, HV, seed=1234)
    nthreads = c_oracle.max_threads()
    out = torch.empty_like(inp.v)
    ns = torch.empty_like(inp.state)
    args = list(inp.args())
    c_oracle.decode(*args, nthreads=nthreads, out=out, new_state=ns)  # warm-up
    steps, t0 = 0, time.perf_counter()
    while True:
        c_oracle.decode(*args, nthreads=nthreads, out=out, new_state=ns)
        steps += 1
        el = time.perf_counter() - t0
        if el >= budget_s or steps >= max_steps:
            break
    per_step = el / steps
    value = B_PER_RANK * HV * UNIT_BYTES / per_step / 1e9
    n, model = cpu_count_info()
    return {"value": round(value, 3), "unit": UNIT, "cores": nthreads, "kind": "port",
            "sample": f"{steps} full decode steps (B={B_PER_RANK}, Hv={HV}) of the C restatement "
                      f"in oracle/gdn_oracle.c, {el:.2f} s, {nthreads} threads on {n} cpus "
                      f"({model})",
            "s_per_step": per_step}


# ---------------------------------------------------------------- our arm
def run_ours(args, rank, world, local_rank, dist):
    from gdn_b200 import decode, workloads as W
    from gdn_b200 import _native as NAT

    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    L = NAT.lib()
    inp = W.make_decode_inputs(B_PER_RANK, HQ, HV, seed=1000 + rank, device=dev)
    s0 = inp.state
    s1 = torch.empty_like(s0)
    out = torch.empty_like(inp.v)
    stream = torch.cuda.current_stream(dev)
    sh = NAT.stream_handle(dev)
    P = NAT.ptr
    scale = float(inp.scale)
    fixed = [P(inp.q), P(inp.k), P(inp.v)]
    gates = [P(inp.A_log), P(inp.a), P(inp.dt_bias), P(inp.b)]

    def step(src, dst):
        rc = L.gdn_decode(fixed[0], fixed[1], fixed[2], P(src), gates[0], gates[1], gates[2],
                          gates[3], scale, P(out), P(dst), B_PER_RANK, HQ, HQ, HV, D, sh)
        if rc:
            NAT.check(rc, "gdn_decode")

    bufs = (s0, s1)
    for i in range(args.warmup):
        step(bufs[i % 2], bufs[(i + 1) % 2])
    torch.cuda.synchronize()

    evs = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps + 1)]
    sampler = ClockSampler(local_rank)
    if dist:
        dist.barrier()
    torch.cuda.synchronize()
    with sampler:
        evs[0].record(stream)
        for i in range(args.steps):
            step(bufs[i % 2], bufs[(i + 1) % 2])
            evs[i + 1].record(stream)
        torch.cuda.synchronize()
    if dist:
        dist.barrier()
    total_ms = evs[0].elapsed_time(evs[-1])
    per_launch = [evs[i].elapsed_time(evs[i + 1]) for i in range(args.steps)]
    t = torch.tensor([total_ms], dtype=torch.float64, device=dev)
    if dist:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    max_ms = float(t.item())
    bytes_per_step_rank = B_PER_RANK * HV * UNIT_BYTES
    value = bytes_per_step_rank * world * args.steps / (max_ms / 1e3) / 1e9
    ms_per_step = max_ms / args.steps
    launch_ms = statistics.mean(per_launch)
    hbm_peak, _, _, peak_src = measured_peaks()
    achieved = bytes_per_step_rank / (launch_ms / 1e3) / 1e9
    roofline = {"bound": "hbm", "kernel": "gdn_decode_kernel<4,true>", "achieved": round(achieved, 1),
                "peak": hbm_peak, "unit": "GB/s", "frac": round(achieved / hbm_peak, 4),
                "peak_source": f"{peak_src} (MEASURED_PEAKS.json hbm_gbs, copy)" if peak_src == "measured" else peak_src,
                "algorithmic_bytes_per_launch": bytes_per_step_rank,
                "launch_ms": round(launch_ms, 5),
                "traffic": profiled_traffic("gdn_decode_b256.md")}

    # ---- end to end through the public API: per-step q/k/v/a/b from pinned
    # host memory, output read back to pinned host memory; the state stays
    # resident in HBM across steps (the decode state cache).
    e2e = None
    if not args.no_e2e:
        e2e = run_e2e(args, inp, dev, stream, dist, world)

    prefill = None
    if not args.no_prefill:
        prefill = run_prefill_bench(args, rank, world, local_rank, dev, dist)

    pool = None
    if world == 1 and not args.no_pool:
        pool = run_pool_bench(args, dev)

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu:
        cpu = time_cpu_decode(args.cpu_budget)
        cpu.pop("s_per_step", None)

    if rank == 0:
        line = {
            "metric": METRIC, "value": round(value, 2), "unit": UNIT, "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms_per_step, 5),
            "decode_us_per_step": round(ms_per_step * 1e3, 2),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic (seeded; BASELINE config distributions)",
            "config": {"workload": "GDN decode, BASELINE config 1 per rank (B=256, T=1, Hq=Hk=16, "
                                   "Hv=32, d=128, fp32 k-last state); N ranks = B=256*N "
                                   "(N=8 is config 4)",
                       "batch_per_rank": B_PER_RANK, "global_batch": B_PER_RANK * world,
                       "num_q_heads": HQ, "num_v_heads": HV, "head_size": D,
                       "parallelism": f"dp{world} (sequence shards, no collective)",
                       "l2": "inputs larger than L2: 512 MiB state per rank, ping-pong buffers"},
            "gpu_launches": args.steps,
            "roofline": roofline,
            "clocks": sampler.summary(),
            "e2e": e2e,
            "cpu_baseline": cpu,
            "prefill": prefill,
            "decode_pool": pool,
        }
        print(json.dumps(line), flush=True)


def run_e2e(args, inp, dev, stream, dist, world):
    """End to end through the public destination-passing API (decode.launch): every
    step copies its q, k, v, a, b from pinned host memory and reads its output back
    to pinned host memory, inside the timed region; the state stays resident in
    HBM (the decode state cache).  As a serving loop would, the copies run on their
    own streams with two device buffer sets, so step i+1's inputs cross PCIe while
    step i's kernel runs and step i's output comes back during step i+1."""
    from gdn_b200 import decode
    host, dbuf = {}, [{}, {}]
    B = inp.v.shape[0]
    nsteps_host = 2
    for name in ("q", "k", "v", "a", "b"):
        t = getattr(inp, name)
        # a distinct pinned source per step parity (a fresh token batch each step)
        host[name] = [torch.empty(t.shape, dtype=t.dtype, pin_memory=True).copy_(t.cpu())
                      for _ in range(nsteps_host)]
        for i in range(2):
            dbuf[i][name] = torch.empty_like(t)
    o_dev = [torch.empty_like(inp.v) for _ in range(2)]
    o_host = [torch.empty(inp.v.shape, dtype=torch.bfloat16, pin_memory=True) for _ in range(2)]
    states = [inp.state.clone(), torch.empty_like(inp.state)]
    h2d = sum(t[0].numel() * t[0].element_size() for t in host.values())
    d2h = o_host[0].numel() * o_host[0].element_size()
    steps = max(args.steps // 4, 10)
    s_in, s_out = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
    ev_in = [torch.cuda.Event() for _ in range(2)]     # inputs of buffer i landed
    ev_used = [torch.cuda.Event() for _ in range(2)]   # kernel done with buffer i
    ev_out = [torch.cuda.Event() for _ in range(2)]    # output i copied back

    def issue(i):
        j = i % 2
        with torch.cuda.stream(s_in):
            s_in.wait_event(ev_used[j])
            for n in host:
                dbuf[j][n].copy_(host[n][i % nsteps_host], non_blocking=True)
            ev_in[j].record(s_in)
        stream.wait_event(ev_in[j])
        stream.wait_event(ev_out[j])  # output buffer j read back
        d = dbuf[j]
        decode.launch(d["q"], d["k"], d["v"], states[i % 2], inp.A_log, d["a"], inp.dt_bias, d["b"],
                      inp.scale, o_dev[j], states[(i + 1) % 2])
        ev_used[j].record(stream)
        with torch.cuda.stream(s_out):
            s_out.wait_event(ev_used[j])
            o_host[j].copy_(o_dev[j], non_blocking=True)
            ev_out[j].record(s_out)

    for i in range(4):
        issue(i)
    torch.cuda.synchronize()
    if dist:
        dist.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    s_in.wait_stream(stream)
    s_out.wait_stream(stream)
    for i in range(steps):
        issue(i)
    stream.wait_event(ev_out[(steps - 1) % 2])
    stream.wait_event(ev_out[steps % 2])
    e1.record(stream)
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1)
    t = torch.tensor([ms], dtype=torch.float64, device=dev)
    if dist:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms = float(t.item())
    value = B_PER_RANK * HV * UNIT_BYTES * world * steps / (ms / 1e3) / 1e9
    return {"value": round(value, 2), "unit": UNIT, "h2d_bytes_per_step": h2d,
            "d2h_bytes_per_step": d2h, "steps": steps, "us_per_step": round(ms / steps * 1e3, 2),
            "api": "gdn_b200.decode.launch (destination passing)",
            "pipelining": "H2D of step i+1 and D2H of step i-1 overlap step i's kernel (two buffer sets, "
                          "copy streams); every copy is inside the timed region",
            "state": "resident in HBM across steps"}

def run_pool_bench(args, dev):
    """Pooled decode (C ABI gdn_decode_pool) at the config-1 batch: B = 256 sequences
    x Hv = 32 heads, pool of 256 slots updated in place, fp32 and bf16 state, one
    token and four tokens per sequence.  Algorithmic bytes per (sequence, v-head):
    the state read and written once (2 x 64 KiB fp32, 2 x 32 KiB bf16) plus, per
    token, v, o (256 B each), q, k (256 B, shared by the GVA pair) and a, b."""
    from gdn_b200 import decode, workloads as W
    hbm_peak, _, _, _ = measured_peaks()
    res = {}
    for name, bf16, T in (("f32_t1", False, 1), ("bf16_t1", True, 1), ("bf16_t4", True, 4)):
        inp = W.make_decode_pool_inputs(B_PER_RANK, T, HQ, HV, B_PER_RANK, seed=4242, device=dev,
                                        state_bf16=bf16)
        slots = torch.arange(B_PER_RANK, dtype=torch.int32, device=dev)
        out = torch.empty_like(inp.v)

        def step():
            decode.run_pool(inp.q, inp.k, inp.v, inp.A_log, inp.a, inp.dt_bias, inp.b, inp.scale,
                            inp.pool, slots, output=out)

        for _ in range(max(args.warmup, 3)):
            step()
        torch.cuda.synchronize()
        steps = max(args.steps // 5, 20)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(steps):
            step()
        e1.record()
        torch.cuda.synchronize()
        us = e0.elapsed_time(e1) / steps * 1e3
        unit = 2 * D * D * (2 if bf16 else 4) + T * (256 + 256 + 256 + 4)
        gbs = B_PER_RANK * HV * unit / (us / 1e6) / 1e9
        res[name] = {"state_dtype": "bf16" if bf16 else "f32", "tokens_per_seq": T,
                     "us_per_step": round(us, 2), "tokens_per_s": round(B_PER_RANK * T / (us / 1e6), 1),
                     "GB_per_s": round(gbs, 1), "roofline_frac": round(gbs / hbm_peak, 4),
                     "algorithmic_bytes_per_step": B_PER_RANK * HV * unit}
    return {"api": "gdn_b200.decode.run_pool (C ABI gdn_decode_pool)", "batch": B_PER_RANK,
            "num_v_heads": HV, "pool": "256 slots, in place; larger than L2 in every case",
            "results": res}


def run_prefill_bench(args, rank, world, local_rank, dev, dist):
    """Prefill tokens/s on BASELINE config 3's shape (4 x 16384 tokens): each
    rank owns Hv/N v-heads (whole GVA groups) of every sequence; the output
    all-gather over NCCL is timed separately (only callers that need every
    head on every rank pay it)."""
    from gdn_b200 import prefill, sharding as S, workloads as W
    if HQ % world:
        return None
    sh = S.head_shard(HQ, HV, world, rank)
    hq, hv = sh.num_q_heads, sh.num_v_heads
    lengths = [args.prefill_len] * args.prefill_seqs
    inp = W.make_prefill_inputs(lengths, hq, hv, seed=77 + rank, device=dev)
    T, Nseq = sum(lengths), len(lengths)
    out = torch.empty_like(inp.v)
    ns = torch.empty_like(inp.state)

    def once():
        prefill.launch(*inp.args(), out, ns)

    for _ in range(2):
        once()
    torch.cuda.synchronize()
    reps = args.prefill_steps
    stream = torch.cuda.current_stream(dev)
    if dist:
        dist.barrier()
    evs = [torch.cuda.Event(enable_timing=True) for _ in range(reps + 1)]
    evs[0].record(stream)
    for i in range(reps):
        once()
        evs[i + 1].record(stream)
    torch.cuda.synchronize()
    per = [evs[i].elapsed_time(evs[i + 1]) for i in range(reps)]
    t = torch.tensor([statistics.mean(per)], dtype=torch.float64, device=dev)
    if dist:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms = float(t.item())
    # algorithmic traffic and work of one call on this rank
    tok_bytes = 2 * hq * D * 2 + 2 * hv * D * 2 + 2 * hv * 2     # q,k + v,o + a,b
    bytes_call = T * tok_bytes + Nseq * hv * 2 * D * D * 4        # + state in and out
    flops_call = T * hv * 163840                                 # 5.24 MFLOP/token at Hv=32
    hbm_peak, tc_burst, _, peak_src = measured_peaks()
    t_hbm = bytes_call / (hbm_peak * 1e9)
    t_tc = flops_call / (tc_burst * 1e12)
    bound = "hbm" if t_hbm >= t_tc else "tensor"
    # a head shard with few (sequence, head) pairs takes the segmented form
    seg_bound = prefill.segments_for(T, Nseq, hv)
    path = ("gdn_b200.prefill.launch: segmented prefill (job builder, pass 1, combine, pass 2; "
            f"pieces picked on the device under a bound of {seg_bound})" if seg_bound > 1
            else "gdn_b200.prefill.launch (fused chunked kernel)")
    res = {"metric": "gdn_prefill_tokens_per_s", "value": round(T / (ms / 1e3), 1),
           "unit": "tokens/s", "ms_per_call": round(ms, 4), "steps": reps,
           "workload": f"BASELINE config 3: {args.prefill_seqs} x {args.prefill_len} tokens, "
                       f"Hq={HQ}, Hv={HV} ({hv} v-heads on each of {world} ranks), random fp32 "
                       f"initial states", "path": path,
           "gpu_launches_per_call": 4 if seg_bound > 1 else 1,
           "roofline": {"bound": bound, "algorithmic_bytes_per_call": bytes_call,
                        "algorithmic_flops_per_call": flops_call,
                        "achieved_GBps": round(bytes_call / (ms / 1e3) / 1e9, 1),
                        "achieved_TFLOPs": round(flops_call / (ms / 1e3) / 1e12, 2),
                        "hbm_peak_GBps": hbm_peak, "tc_peak_TFLOPs": tc_burst,
                        "roofline_ms": round(max(t_hbm, t_tc) * 1e3, 4),
                        "frac": round(max(t_hbm, t_tc) * 1e3 / ms, 4), "peak_source": peak_src}}
    full = profiled_traffic("gdn_prefill_chunked_config3.md")  # ncu, 1-GPU config-3 launch
    if full is not None and args.prefill_seqs == 4 and args.prefill_len == 16384 and seg_bound == 1:
        res["roofline"]["traffic"] = int(full * hv / HV)  # this rank's heads
    if dist and world > 1:
        from gdn_b200.sharding import all_gather_heads
        for _ in range(2):
            all_gather_heads(out)
        torch.cuda.synchronize()
        dist.barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(reps):
            full = all_gather_heads(out)
        e1.record(stream)
        torch.cuda.synchronize()
        ag = torch.tensor([e0.elapsed_time(e1) / reps], dtype=torch.float64, device=dev)
        dist.all_reduce(ag, op=dist.ReduceOp.MAX)
        recv = (world - 1) * out.numel() * out.element_size()
        res["allgather_o"] = {"ms": round(float(ag.item()), 4), "bytes_received_per_rank": recv,
                              "GBps_per_rank": round(recv / (float(ag.item()) / 1e3) / 1e9, 1),
                              "value_with_gather": round(T / ((ms + float(ag.item())) / 1e3), 1)}
        # the same gather fused into the kernel: every rank's output tiles go to every
        # rank's full buffer over NVLink (peer-mapped), no collective
        from gdn_b200.sharding import PeerOutputs, prefill_gathered
        bufs = PeerOutputs(T, HV, dev)
        ns_g = torch.empty_like(ns)
        for _ in range(2):
            prefill_gathered(inp, sh.v0, bufs, ns_g)
        torch.cuda.synchronize()
        dist.barrier()
        e0.record(stream)
        for _ in range(reps):
            prefill_gathered(inp, sh.v0, bufs, ns_g)
        e1.record(stream)
        torch.cuda.synchronize()
        fg = torch.tensor([e0.elapsed_time(e1) / reps], dtype=torch.float64, device=dev)
        dist.all_reduce(fg, op=dist.ReduceOp.MAX)
        dist.barrier()  # every rank's stores have landed in every buffer
        same = torch.tensor([1 if torch.equal(bufs.output, full) else 0], device=dev)
        dist.all_reduce(same, op=dist.ReduceOp.MIN)
        dist.barrier()
        bufs.close()
        res["allgather_fused"] = {
            "ms_per_call_with_gather": round(float(fg.item()), 4),
            "value_with_gather": round(T / (float(fg.item()) / 1e3), 1),
            "matches_nccl_allgather": bool(same.item()),
            "how": "C ABI gdn_prefill_chunked_peers: the kernel's output TMA stores also target "
                   "every peer's full output buffer (CUDA IPC mapping); no collective"}
        del full
    return res


# ---------------------------------------------------------------- reference arm
def run_reference(args, rank, world):
    if rank != 0:
        return
    cpu = time_cpu_decode(args.cpu_budget)
    per_step = cpu.pop("s_per_step")
    line = {
        "metric": METRIC, "value": cpu["value"], "unit": UNIT, "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(per_step * 1e3, 3),
        "decode_us_per_step": round(per_step * 1e6, 1), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic (seeded; BASELINE config distributions)",
        "config": {"workload": "GDN decode, BASELINE config 1 (B=256, T=1, Hq=Hk=16, Hv=32, "
                               "d=128); rank 0 only", "batch_per_rank": B_PER_RANK,
                   "global_batch": B_PER_RANK, "num_q_heads": HQ, "num_v_heads": HV,
                   "head_size": D, "parallelism": "host cpu threads"},
        "impl": "reference",
        "cpu_baseline": cpu,
        "e2e": {"value": cpu["value"], "unit": UNIT, "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
        "gpu_launches": 0,
    }
    print(json.dumps(line), flush=True)


def run_replay(args):
    """Contest-shape replay (qk4_v8 geometry: Hq = Hk = 4, Hv = 8): latency of the
    public ``run`` entry points over seeded synthetic shapes spanning the contest
    workloads' axes, next to the C restatement of the reference on the host cores.
    Back-to-back calls with inputs resident on the device, as a Solution harness
    calls them; per case: median of 5 batches of 20 calls (CUDA events)."""
    from gdn_b200 import decode, prefill, workloads as W
    from oracle import c_oracle
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    hq, hv = W.CONTEST_HQ, W.CONTEST_HV
    cpu_left = args.cpu_budget * 6

    def gpu_us(fn):
        for _ in range(3):
            fn()
        torch.cuda.synchronize()
        ts = []
        for _ in range(5):
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            for _ in range(20):
                fn()
            e1.record()
            torch.cuda.synchronize()
            ts.append(e0.elapsed_time(e1) / 20 * 1e3)
        return sorted(ts)[2]

    def cpu_us(fn):
        nonlocal cpu_left
        if cpu_left <= 0:
            return None
        t0 = time.perf_counter()
        fn()
        dt = time.perf_counter() - t0
        cpu_left -= dt
        return dt * 1e6

    rows_d, rows_p, ratios = [], [], []
    for B in W.CONTEST_DECODE_BATCHES:
        inp = W.make_decode_inputs(B, hq, hv, seed=500 + B)
        c_us = cpu_us(lambda: c_oracle.decode(*inp.args()))
        dinp = W.make_decode_inputs(B, hq, hv, seed=500 + B, device=dev)
        g_us = gpu_us(lambda: decode.run(*dinp.args()))
        from gdn_b200.graphs import DecodeGraph
        dg = DecodeGraph(dinp.q, dinp.k, dinp.v, dinp.state.clone(), dinp.A_log, dinp.a, dinp.dt_bias,
                         dinp.b, dinp.scale)
        gr_us = gpu_us(dg.step)
        r = None if c_us is None else c_us / g_us
        if r:
            ratios.append(r)
        rows_d.append({"batch": B, "us": round(g_us, 2), "graph_replay_us": round(gr_us, 2),
                       "cpu_us": c_us and round(c_us, 1), "speedup_vs_cpu": r and round(r, 1)})
    for i, lengths in enumerate(W.contest_prefill_cases()):
        inp = W.make_prefill_inputs(lengths, hq, hv, seed=700 + i)
        c_us = cpu_us(lambda: c_oracle.prefill(*inp.args()))
        dinp = W.make_prefill_inputs(lengths, hq, hv, seed=700 + i, device=dev)
        g_us = gpu_us(lambda: prefill.run(*dinp.args()))
        r = None if c_us is None else c_us / g_us
        if r:
            ratios.append(r)
        rows_p.append({"num_seqs": len(lengths), "total_seq_len": sum(lengths), "us": round(g_us, 2),
                       "cpu_us": c_us and round(c_us, 1), "speedup_vs_cpu": r and round(r, 1)})
    geo = math.exp(sum(math.log(r) for r in ratios) / len(ratios)) if ratios else None
    print(json.dumps({
        "metric": "contest-shape replay latency (qk4_v8: Hq=Hk=4, Hv=8, d=128)", "unit": "us",
        "data": "synthetic (seeded shapes spanning the contest workload axes)",
        "api": "gdn_b200.decode.run / gdn_b200.prefill.run, device-resident inputs",
        "cpu": {"impl": "oracle/gdn_oracle.c (C restatement of the reference definitions)",
                "cores": c_oracle.max_threads()},
        "geomean_speedup_vs_cpu": geo and round(geo, 1),
        "decode": rows_d, "prefill": rows_p}), flush=True)


def main():
    global B_PER_RANK
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=1000)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--no-prefill", action="store_true")
    ap.add_argument("--no-pool", action="store_true", help="skip the pooled-decode leg")
    ap.add_argument("--pool-only", action="store_true",
                    help="run only the pooled-decode leg and print its JSON (profiling runs)")
    ap.add_argument("--cpu-budget", type=float, default=10.0)
    ap.add_argument("--batch-per-rank", type=int, default=256,
                    help="sequences per rank (default 256 = BASELINE config 1; smaller only for profiling)")
    ap.add_argument("--prefill-seqs", type=int, default=4)
    ap.add_argument("--prefill-len", type=int, default=16384)
    ap.add_argument("--prefill-steps", type=int, default=10)
    ap.add_argument("--prefill-only", action="store_true",
                    help="run only the prefill leg and print its JSON (profiling runs)")
    ap.add_argument("--replay", action="store_true",
                    help="contest-shape replay (qk4_v8 geometry) instead of the headline line")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)
    B_PER_RANK = args.batch_per_rank

    world = env_int("WORLD_SIZE", 1)
    rank = env_int("RANK", 0)
    local_rank = env_int("LOCAL_RANK", 0)
    if args.replay:
        if rank == 0:
            run_replay(args)
        return
    if args.impl == "reference":
        run_reference(args, rank, world)
        return
    dist = None
    if world > 1:
        import torch.distributed as tdist
        torch.cuda.set_device(local_rank)
        tdist.init_process_group("nccl", timeout=timedelta(seconds=120),
                                 device_id=torch.device("cuda", local_rank))
        dist = tdist
    try:
        if args.pool_only:
            dev = torch.device("cuda", local_rank)
            torch.cuda.set_device(dev)
            if rank == 0:
                print(json.dumps(run_pool_bench(args, dev)), flush=True)
            return
        if args.prefill_only:
            dev = torch.device("cuda", local_rank)
            torch.cuda.set_device(dev)
            res = run_prefill_bench(args, rank, world, local_rank, dev, dist)
            if rank == 0:
                print(json.dumps(res), flush=True)
            return
        run_ours(args, rank, world, local_rank, dist)
    finally:
        if dist:
            dist.barrier()
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
