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

    library = None
    if world == 1 and not args.no_library:
        library = run_library_baseline(args, dev)

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
            "library_baseline": library,
        }
        print(json.dumps(line), flush=True)


def run_e2e(args, inp, dev, stream, dist, world):
    """End to end through the public destination-passing API (decode.launch): every
    step copies its q, k, v, a, b from pinned host memory and reads its output back
    to pinned host memory, inside the timed region; the state stays resident in
    HBM (the decode state cache).  As a serving loop would, the copies run on their
    own streams with two device buffer sets, so step i+1's inputs cross PCIe while
    step i's kernel runs and step i's output comes back during step i+1.  The loop
    is timed twice: issued step by step from Python ("eager"), and as replays of a
    CUDA graph that holds 100 such pipelined steps (copies, kernel launches and their
    cross-stream event order, captured once), which is how a serving loop drives
    it without the host's per-step launch cost.  The graph replays give the value:
    the eager loop measures the host's Python speed as much as the transfer (its
    windows are reported beside it)."""
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
    steps = max(args.steps // 20, 40)  # per window; 5 windows: >= 200 steps
    windows = 5
    s_in, s_out = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
    ev_in = [torch.cuda.Event() for _ in range(2)]     # inputs of buffer i landed
    ev_used = [torch.cuda.Event() for _ in range(2)]   # kernel done with buffer i
    ev_out = [torch.cuda.Event() for _ in range(2)]    # output i copied back

    def issue(i, main, first=False):
        # first: inside a graph capture, the first use of buffer i % 2 (nothing of
        # this capture to wait for yet)
        j = i % 2
        with torch.cuda.stream(s_in):
            if not first:
                s_in.wait_event(ev_used[j])
            for n in host:
                dbuf[j][n].copy_(host[n][i % nsteps_host], non_blocking=True)
            ev_in[j].record(s_in)
        main.wait_event(ev_in[j])
        if not first:
            main.wait_event(ev_out[j])  # output buffer j read back
        d = dbuf[j]
        decode.launch(d["q"], d["k"], d["v"], states[i % 2], inp.A_log, d["a"], inp.dt_bias, d["b"],
                      inp.scale, o_dev[j], states[(i + 1) % 2])
        ev_used[j].record(main)
        with torch.cuda.stream(s_out):
            s_out.wait_event(ev_used[j])
            o_host[j].copy_(o_dev[j], non_blocking=True)
            ev_out[j].record(s_out)

    def timed_windows(run_window, nsteps):
        ms_list = []
        for _ in range(windows):
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            run_window()
            e1.record(stream)
            torch.cuda.synchronize()
            ms_list.append(e0.elapsed_time(e1))
        t = torch.tensor(ms_list, dtype=torch.float64, device=dev)
        if dist:
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms_list = [float(x) for x in t.tolist()]
        per = sorted(w / nsteps * 1e3 for w in ms_list)
        return sum(ms_list), per

    def summary(ms, per, nsteps):
        med = statistics.median(per)
        return {"steps": nsteps * windows, "us_per_step": round(ms / (nsteps * windows) * 1e3, 2),
                "us_per_step_median_window": round(med, 2),
                "us_per_step_windows": [round(x, 2) for x in per],
                "spread_pct": round((per[-1] - per[0]) / med * 100, 2)}

    # eager: five windows of `steps` pipelined steps issued from Python
    for i in range(4):
        issue(i, stream)
    torch.cuda.synchronize()
    if dist:
        dist.barrier()

    def eager_window():
        s_in.wait_stream(stream)
        s_out.wait_stream(stream)
        for i in range(steps):
            issue(i, stream)
        stream.wait_event(ev_out[(steps - 1) % 2])
        stream.wait_event(ev_out[steps % 2])

    eager_ms, eager_per = timed_windows(eager_window, steps)

    # graph: 100 pipelined steps captured once (side streams forked from and joined
    # back to the capture stream), replayed; a replay starts with its first upload
    # and ends with its last read-back, ~0.7 % of 100 steps
    g_steps = 100
    graph = torch.cuda.CUDAGraph()
    cap = torch.cuda.Stream(dev)
    cap.wait_stream(stream)
    torch.cuda.synchronize()
    with torch.cuda.graph(graph, stream=cap):
        s_in.wait_stream(cap)
        s_out.wait_stream(cap)
        for i in range(g_steps):
            issue(i, cap, first=i < 2)
        cap.wait_stream(s_in)
        cap.wait_stream(s_out)
    reps = max(steps // g_steps, 1)
    for _ in range(2):
        graph.replay()
    torch.cuda.synchronize()
    if dist:
        dist.barrier()

    def graph_window():
        for _ in range(reps):
            graph.replay()

    g_ms, g_per = timed_windows(graph_window, reps * g_steps)
    total_steps = reps * g_steps * windows
    value = B_PER_RANK * HV * UNIT_BYTES * world * total_steps / (g_ms / 1e3) / 1e9
    eager_value = B_PER_RANK * HV * UNIT_BYTES * world * steps * windows / (eager_ms / 1e3) / 1e9
    out = {"value": round(value, 2), "unit": UNIT, "h2d_bytes_per_step": h2d,
           "d2h_bytes_per_step": d2h}
    out.update(summary(g_ms, g_per, reps * g_steps))
    out.update({"api": "gdn_b200.decode.launch (destination passing), 100 pipelined steps "
                       "captured in a CUDA graph and replayed",
                "pipelining": "H2D of step i+1 and D2H of step i-1 overlap step i's kernel (two "
                              "buffer sets, copy streams); every copy is inside the timed region",
                "eager": dict(value=round(eager_value, 2), **summary(eager_ms, eager_per, steps)),
                "state": "resident in HBM across steps"})
    del graph
    return out


def run_pool_bench(args, dev):
    """Pooled decode (C ABI gdn_decode_pool) at the config-1 batch: B = 256 sequences
    x Hv = 32 heads, pool of 256 slots updated in place, fp32 and bf16 state, one
    token and four tokens per sequence.  Algorithmic bytes per (sequence, v-head):
    the state read and written once (2 x 64 KiB fp32, 2 x 32 KiB bf16) plus, per
    token, v, o (256 B each), q, k (256 B, shared by the GVA pair) and a, b."""
    from gdn_b200 import decode, workloads as W
    hbm_peak, _, _, _ = measured_peaks()
    res = {}
    # bf16_t4 and bf16_t8 take the tensor-core closed form (gdn_decode_pool_tc.cu, 3..16 tokens),
    # f32_t4 the fp32 multi-token kernel
    for name, bf16, T in (("f32_t1", False, 1), ("f32_t4", False, 4), ("bf16_t1", True, 1),
                          ("bf16_t4", True, 4), ("bf16_t8", True, 8)):
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
                     "kernel": "gdn_decode_pool_tc_kernel (tcgen05 closed form)" if bf16 and 3 <= T <= 16
                     else "gdn_decode_pool_f32_mtp_kernel (token by token, 64-row CTAs)"
                     if not bf16 and T > 1 else "gdn_decode_pool kernels (token by token)",
                     "us_per_step": round(us, 2), "tokens_per_s": round(B_PER_RANK * T / (us / 1e6), 1),
                     "GB_per_s": round(gbs, 1), "roofline_frac": round(gbs / hbm_peak, 4),
                     "algorithmic_bytes_per_step": B_PER_RANK * HV * unit}
    return {"api": "gdn_b200.decode.run_pool (C ABI gdn_decode_pool)", "batch": B_PER_RANK,
            "num_v_heads": HV, "pool": "256 slots, in place; larger than L2 in every case",
            "results": res}


def prefill_unit_costs(T, Nseq, hq, hv):
    """Algorithmic bytes and FLOPs of one prefill call (q, k, v, o, a, b per token,
    the state read and written once per (sequence, v-head); 163,840 FLOP per token
    and v-head)."""
    tok_bytes = 2 * hq * D * 2 + 2 * hv * D * 2 + 2 * hv * 2
    return T * tok_bytes + Nseq * hv * 2 * D * D * 4, T * hv * 163840


def prefill_roofline(T, Nseq, hq, hv, ms):
    bytes_call, flops_call = prefill_unit_costs(T, Nseq, hq, hv)
    hbm_peak, tc_burst, _, peak_src = measured_peaks()
    t_hbm = bytes_call / (hbm_peak * 1e9)
    t_tc = flops_call / (tc_burst * 1e12)
    return {"bound": "hbm" if t_hbm >= t_tc else "tensor", "algorithmic_bytes_per_call": bytes_call,
            "algorithmic_flops_per_call": flops_call,
            "achieved_GBps": round(bytes_call / (ms / 1e3) / 1e9, 1),
            "achieved_TFLOPs": round(flops_call / (ms / 1e3) / 1e12, 2),
            "hbm_peak_GBps": hbm_peak, "tc_peak_TFLOPs": tc_burst,
            "roofline_ms": round(max(t_hbm, t_tc) * 1e3, 4),
            "frac": round(max(t_hbm, t_tc) * 1e3 / ms, 4),
            "peak_source": f"{peak_src} (MEASURED_PEAKS.json hbm_gbs copy / bf16_tflops burst)"
            if peak_src == "measured" else peak_src}


def time_calls(fn, reps, dev, dist):
    """Mean device time per call (ms), CUDA events on the current stream around
    each call after two warm-up calls, max over ranks."""
    for _ in range(2):
        fn()
    torch.cuda.synchronize()
    stream = torch.cuda.current_stream(dev)
    if dist:
        dist.barrier()
    evs = [torch.cuda.Event(enable_timing=True) for _ in range(reps + 1)]
    evs[0].record(stream)
    for i in range(reps):
        fn()
        evs[i + 1].record(stream)
    torch.cuda.synchronize()
    per = [evs[i].elapsed_time(evs[i + 1]) for i in range(reps)]
    t = torch.tensor([statistics.mean(per)], dtype=torch.float64, device=dev)
    if dist:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item()), per


def prefill_e2e(cpu_inp, dev, reps, dist):
    """End to end through the public destination-passing API (prefill.launch): each
    call copies q, k, v, a, b, cu_seqlens and the initial states from pinned host
    memory, runs, and copies o and the final states back to pinned host memory, all
    inside the timed region.  As a server taking a stream of prefill requests would,
    the copies run on their own streams with two device buffer sets: call i+1's
    inputs cross PCIe while call i's kernels run, and call i's outputs come back
    during call i+1 (PCIe carries both directions at once)."""
    from gdn_b200 import prefill
    names = ("q", "k", "v", "state", "a", "b", "cu_seqlens")
    host = {n: getattr(cpu_inp, n).pin_memory() for n in names if getattr(cpu_inp, n) is not None}
    devb = [{n: torch.empty_like(t, device=dev) for n, t in host.items()} for _ in range(2)]
    A_log, dt_bias = cpu_inp.A_log.to(dev), cpu_inp.dt_bias.to(dev)
    Nseq = cpu_inp.cu_seqlens.numel() - 1
    hv = cpu_inp.v.shape[1]
    o_dev = [torch.empty_like(devb[0]["v"]) for _ in range(2)]
    ns_dev = [torch.empty((Nseq, hv, D, D), dtype=torch.float32, device=dev) for _ in range(2)]
    o_host = [torch.empty(o_dev[0].shape, dtype=o_dev[0].dtype, pin_memory=True) for _ in range(2)]
    ns_host = [torch.empty(ns_dev[0].shape, dtype=ns_dev[0].dtype, pin_memory=True)
               for _ in range(2)]
    ws_bytes = prefill.workspace_bytes(cpu_inp.q.shape[0], Nseq, cpu_inp.q.shape[1], hv)
    ws = torch.empty(max(ws_bytes, 1), dtype=torch.uint8, device=dev)
    stream = torch.cuda.current_stream(dev)
    s_in, s_out = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
    ev_in = [torch.cuda.Event() for _ in range(2)]     # inputs of set j landed
    ev_used = [torch.cuda.Event() for _ in range(2)]   # the call is done with set j
    ev_out = [torch.cuda.Event() for _ in range(2)]    # outputs of set j copied back

    def issue(i):
        j = i % 2
        with torch.cuda.stream(s_in):
            s_in.wait_event(ev_used[j])
            for n, t in host.items():
                devb[j][n].copy_(t, non_blocking=True)
            ev_in[j].record(s_in)
        stream.wait_event(ev_in[j])
        stream.wait_event(ev_out[j])
        d = devb[j]
        prefill.launch(d["q"], d["k"], d["v"], d.get("state"), A_log, d["a"], dt_bias, d["b"],
                       d["cu_seqlens"], cpu_inp.scale, o_dev[j], ns_dev[j],
                       workspace=ws if ws_bytes else None)
        ev_used[j].record(stream)
        with torch.cuda.stream(s_out):
            s_out.wait_event(ev_used[j])
            o_host[j].copy_(o_dev[j], non_blocking=True)
            ns_host[j].copy_(ns_dev[j], non_blocking=True)
            ev_out[j].record(s_out)

    for i in range(3):
        issue(i)
    torch.cuda.synchronize()
    if dist:
        dist.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    s_in.wait_stream(stream)
    s_out.wait_stream(stream)
    for i in range(reps):
        issue(i)
    stream.wait_event(ev_out[(reps - 1) % 2])
    stream.wait_event(ev_out[reps % 2])
    e1.record(stream)
    torch.cuda.synchronize()
    t = torch.tensor([e0.elapsed_time(e1)], dtype=torch.float64, device=dev)
    if dist:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms = float(t.item()) / reps
    h2d = sum(t.numel() * t.element_size() for t in host.values())
    d2h = o_host[0].numel() * o_host[0].element_size() + ns_host[0].numel() * ns_host[0].element_size()
    T = cpu_inp.q.shape[0]
    return {"value": round(T / (ms / 1e3), 1), "unit": "tokens/s", "h2d_bytes_per_step": h2d,
            "d2h_bytes_per_step": d2h, "ms_per_call": round(ms, 4), "calls": reps,
            "api": "gdn_b200.prefill.launch (destination passing)",
            "copies": "H2D of every input and D2H of o and the final states inside the timed "
                      "region; copies on their own streams with two buffer sets, so call "
                      "i+1's inputs and call i-1's outputs cross PCIe while call i runs"}


def cpu_prefill(lengths, hq, hv, seed, zero_every_other):
    """The C restatement of the reference prefill recurrence on all host threads,
    on the same workload (whole: every sequence and head)."""
    from oracle import c_oracle
    from gdn_b200 import workloads as W
    inp = W.make_prefill_inputs(lengths, hq, hv, seed=seed, zero_state_every_other=zero_every_other)
    nthreads = c_oracle.max_threads()
    t0 = time.perf_counter()
    c_oracle.prefill(*inp.args(), nthreads=nthreads)
    el = time.perf_counter() - t0
    n, model = cpu_count_info()
    T = sum(lengths)
    return {"value": round(T / el, 1), "unit": "tokens/s", "cores": nthreads, "kind": "port",
            "sample": f"the whole workload ({len(lengths)} sequences, {T} tokens, Hv={hv}) once through "
                      f"oracle/gdn_oracle.c, {el:.2f} s, {nthreads} threads on {n} cpus ({model})"}


def run_prefill_bench(args, rank, world, local_rank, dev, dist):
    """Prefill tokens/s on BASELINE config 3 (4 x 16384 tokens) and config 2 (16
    varlen sequences, ~U[64, 1024] tokens, half zero states): each rank owns Hv/N
    v-heads (whole GVA groups) of every sequence.  Per config: the device time of
    prefill.launch with inputs resident in HBM and its roofline, the same call end
    to end with host buffers (e2e), and the C restatement of the reference on the
    host cores (rank 0, N = 1).  At N > 1 the output all-gather (NCCL, and fused
    into the kernel's stores) is timed separately on config 3."""
    from gdn_b200 import prefill, sharding as S, workloads as W
    if HQ % world:
        return None
    sh = S.head_shard(HQ, HV, world, rank)
    hq, hv = sh.num_q_heads, sh.num_v_heads
    cfgs = [("config3", [args.prefill_len] * args.prefill_seqs, 77, False,
             f"BASELINE config 3: {args.prefill_seqs} x {args.prefill_len} tokens, Hq={HQ}, Hv={HV} "
             f"({hv} v-heads on each of {world} ranks), random fp32 initial states"),
            ("config2", W.config_lengths("prefill_varlen"), 2, True,
             f"BASELINE config 2: 16 sequences, lengths ~U[64,1024] (seeded), Hq={HQ}, Hv={HV} "
             f"({hv} v-heads on each of {world} ranks), zero initial state for every other sequence")]
    res = {}
    for name, lengths, seed, zero_eo, desc in cfgs:
        T, Nseq = sum(lengths), len(lengths)
        cpu_inp = W.make_prefill_inputs(lengths, hq, hv, seed=seed + rank, zero_state_every_other=zero_eo)
        inp = W.make_prefill_inputs(lengths, hq, hv, seed=seed + rank, device=dev,
                                    zero_state_every_other=zero_eo)
        out = torch.empty_like(inp.v)
        ns = torch.empty_like(inp.state)
        ws_bytes = prefill.workspace_bytes(T, Nseq, hq, hv)
        ws = torch.empty(max(ws_bytes, 1), dtype=torch.uint8, device=dev)
        reps = args.prefill_steps if name == "config3" else max(args.prefill_steps * 5, 20)
        ms, per = time_calls(lambda: prefill.launch(*inp.args(), out, ns, workspace=ws if ws_bytes else None),
                             reps, dev, dist)
        seg_bound = prefill.segments_for(T, Nseq, hv)
        path = ("gdn_b200.prefill.launch: segmented prefill (job builder, pass 1, combine, pass 2; "
                f"pieces picked on the device under a bound of {seg_bound})" if seg_bound > 1
                else "gdn_b200.prefill.launch (fused chunked kernel)")
        # every rank walks all T tokens for its heads: the job's rate is T / (max-over-ranks time)
        r = {"metric": "gdn_prefill_tokens_per_s", "value": round(T / (ms / 1e3), 1),
             "unit": "tokens/s", "ms_per_call": round(ms, 4),
             "ms_per_call_median_rank0": round(statistics.median(per), 4), "steps": reps,
             "workload": desc,
             "total_tokens": T, "num_seqs": Nseq, "path": path,
             "gpu_launches_per_call": 4 if seg_bound > 1 else 1,
             "roofline": prefill_roofline(T, Nseq, hq, hv, ms)}
        if name == "config3":
            full = profiled_traffic("gdn_prefill_chunked_config3.md")  # ncu, 1-GPU config-3 launch
            if full is not None and args.prefill_seqs == 4 and args.prefill_len == 16384 and seg_bound == 1:
                r["roofline"]["traffic"] = int(full * hv / HV)  # this rank's heads
        if not args.no_e2e:
            r["e2e"] = prefill_e2e(cpu_inp, dev, 8 if name == "config3" else 30, dist)
        if rank == 0 and world == 1 and not args.no_cpu:
            r["cpu_baseline"] = cpu_prefill(lengths, hq, hv, seed, zero_eo)
        res[name] = r
        del inp, out, ns, ws, cpu_inp
    # the headline prefill object stays config 3; config 2 rides beside it
    top = res["config3"]
    top["config2"] = res["config2"]
    if dist and world > 1:
        lengths = [args.prefill_len] * args.prefill_seqs
        T = sum(lengths)
        inp = W.make_prefill_inputs(lengths, hq, hv, seed=77 + rank, device=dev)
        out = torch.empty_like(inp.v)
        ns = torch.empty_like(inp.state)
        prefill.launch(*inp.args(), out, ns)
        torch.cuda.synchronize()
        ms = top["ms_per_call"]
        reps = args.prefill_steps
        stream = torch.cuda.current_stream(dev)
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
        top["allgather_o"] = {"ms": round(float(ag.item()), 4), "bytes_received_per_rank": recv,
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
        top["allgather_fused"] = {
            "ms_per_call_with_gather": round(float(fg.item()), 4),
            "value_with_gather": round(T / (float(fg.item()) / 1e3), 1),
            "bytes_received_per_rank": recv,
            "nvlink_GBps_per_rank": round(recv / (float(fg.item()) / 1e3) / 1e9, 1),
            "matches_nccl_allgather": bool(same.item()),
            "how": "C ABI gdn_prefill_chunked_peers: the kernel's output TMA stores also target "
                   "every peer's full output buffer (CUDA IPC mapping); no collective"}
        del full
    return top


# ---------------------------------------------------------------- library baselines
def run_library_baseline(args, dev):
    """FlashInfer's Blackwell GDN kernels, the bars the reference measures itself
    against (reference_solutions/baseline/gdn/gdn_prefill_qk4_v8_d128_k_last/
    flashinfer_wrapper_123ca6.md:30-59 and .../gdn_decode_qk4_v8_d128_k_last/
    flashinfer_wrapper_9b7f1e.md:24-55), called as libraries on the same box and
    the same inputs as our kernels.  Prefill: chunk_gated_delta_rule_sm100, the
    CuTe-DSL SM100 kernel that flashinfer.chunk_gated_delta_rule dispatches to on
    sm_100a (called directly: the dispatcher picks it only under a CUDA 13 torch);
    its gates are formed in torch first, as the wrapper does.  Decode:
    gated_delta_rule_decode_pretranspose on the fp32 k-last state, in place.
    Each line gives the library's time, ours on the same inputs, ours' speed-up
    (library time / our time) and the largest difference between the outputs."""
    import torch.nn.functional as F
    from gdn_b200 import decode, prefill, workloads as W
    out = {}
    try:
        import flashinfer
        out["flashinfer_version"] = flashinfer.__version__
    except Exception as e:  # pragma: no cover - depends on the box
        return {"unavailable": f"flashinfer import failed: {e!r}"[:400]}

    def dev_time(fn, reps):
        for _ in range(3):
            fn()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(reps):
            fn()
        e1.record()
        torch.cuda.synchronize()
        return e0.elapsed_time(e1) / reps

    try:
        from flashinfer.gdn_kernels import chunk_gated_delta_rule_sm100 as fi_prefill
        if fi_prefill is None:
            raise ImportError("flashinfer.gdn_kernels.chunk_gated_delta_rule_sm100 is None")
    except Exception as e:  # pragma: no cover
        fi_prefill = None
        out["prefill_unavailable"] = f"{e!r}"[:400]
    cases = [("config3", [16384] * 4, HQ, HV, 77, False),
             ("config2", W.config_lengths("prefill_varlen"), HQ, HV, 2, True),
             ("contest_8192x1_qk4_v8", [8192], 4, 8, 5, False),
             ("contest_even_8192x4_qk4_v8", W.even_lengths(8192, 4), 4, 8, 6, False)]
    for name, lengths, hq, hv, seed, zeo in cases if fi_prefill is not None else []:
        try:
            inp = W.make_prefill_inputs(lengths, hq, hv, seed=seed, device=dev, zero_state_every_other=zeo)
            T, Nseq = sum(lengths), len(lengths)
            reps = 10 if T > 20000 else 30
            o_ours = torch.empty_like(inp.v)
            ns_ours = torch.empty_like(inp.state)
            ws_bytes = prefill.workspace_bytes(T, Nseq, hq, hv)
            ws = torch.empty(max(ws_bytes, 1), dtype=torch.uint8, device=dev)
            ours_ms = dev_time(lambda: prefill.launch(*inp.args(), o_ours, ns_ours,
                                                      workspace=ws if ws_bytes else None), reps)
            cu32 = inp.cu_seqlens.to(torch.int32)
            o_fi = torch.empty_like(inp.v)
            ns_fi = torch.empty_like(inp.state)

            def gates():
                g = -torch.exp(inp.A_log.float()) * F.softplus(inp.a.float() + inp.dt_bias.float())
                return g.contiguous(), torch.sigmoid(inp.b.float()).contiguous()

            g, beta = gates()
            kern = lambda: fi_prefill(inp.q, inp.k, inp.v, g, beta, o_fi, cu32, inp.state, ns_fi,
                                      float(inp.scale))

            def wrapper():
                gg, bb = gates()
                fi_prefill(inp.q, inp.k, inp.v, gg, bb, o_fi, cu32, inp.state, ns_fi, float(inp.scale))

            t0 = time.perf_counter()
            kern()  # first call compiles the CuTe-DSL kernel
            torch.cuda.synchronize()
            compile_s = time.perf_counter() - t0
            lib_ms = dev_time(kern, reps)
            lib_wrap_ms = dev_time(wrapper, reps)
            kern()
            prefill.launch(*inp.args(), o_ours, ns_ours, workspace=ws if ws_bytes else None)
            torch.cuda.synchronize()
            d_o = (o_ours.float() - o_fi.float()).abs().max().item()
            ref = ns_ours.reshape(-1, D * D)
            d_s = ((ns_fi.reshape(-1, D * D) - ref).norm(dim=1) / ref.norm(dim=1).clamp_min(1e-30)).max().item()
            out[f"prefill_{name}"] = {
                "workload": f"{Nseq} sequences, {T} tokens, Hq={hq}, Hv={hv}",
                "library_kernel_ms": round(lib_ms, 4), "library_with_gates_ms": round(lib_wrap_ms, 4),
                "ours_ms": round(ours_ms, 4),
                "library_tokens_per_s": round(T / (lib_wrap_ms / 1e3), 1),
                "ours_tokens_per_s": round(T / (ours_ms / 1e3), 1),
                "speedup_ours_vs_library": round(lib_wrap_ms / ours_ms, 3),
                "speedup_ours_vs_library_kernel_only": round(lib_ms / ours_ms, 3),
                "max_abs_diff_o": d_o, "max_state_rel_diff": d_s,
                "library_first_call_s": round(compile_s, 1)}
            del inp, o_ours, ns_ours, o_fi, ns_fi, ws
        except Exception as e:  # pragma: no cover
            out[f"prefill_{name}"] = {"unavailable": f"{e!r}"[:400]}
    try:
        from flashinfer.gdn_decode import gated_delta_rule_decode_pretranspose as fi_decode
        inp = W.make_decode_inputs(B_PER_RANK, HQ, HV, seed=1000, device=dev)
        st_fi = inp.state.clone()
        st_ours = inp.state.clone()
        o_fi = torch.empty_like(inp.v)
        o_ours = torch.empty_like(inp.v)
        kern = lambda: fi_decode(inp.q, inp.k, inp.v, st_fi, inp.A_log, inp.a, inp.dt_bias, inp.b,
                                 scale=float(inp.scale), output=o_fi, use_qk_l2norm=False)
        ours = lambda: decode.launch(inp.q, inp.k, inp.v, st_ours, inp.A_log, inp.a, inp.dt_bias, inp.b,
                                     inp.scale, o_ours, st_ours)
        t0 = time.perf_counter()
        kern()
        torch.cuda.synchronize()
        compile_s = time.perf_counter() - t0
        lib_ms = dev_time(kern, 100)
        ours_ms = dev_time(ours, 100)
        # one step each from the same state: outputs and states compared
        st_fi.copy_(inp.state)
        st_ours.copy_(inp.state)
        kern()
        ours()
        torch.cuda.synchronize()
        ref = st_ours.reshape(-1, D * D)
        d_s = ((st_fi.reshape(-1, D * D) - ref).norm(dim=1) / ref.norm(dim=1).clamp_min(1e-30)).max().item()
        out["decode_config1"] = {
            "workload": f"B={B_PER_RANK}, Hq={HQ}, Hv={HV}, fp32 state updated in place",
            "library_us_per_step": round(lib_ms * 1e3, 2), "ours_us_per_step": round(ours_ms * 1e3, 2),
            "library_GBps": round(B_PER_RANK * HV * UNIT_BYTES / (lib_ms / 1e3) / 1e9, 1),
            "ours_GBps": round(B_PER_RANK * HV * UNIT_BYTES / (ours_ms / 1e3) / 1e9, 1),
            "speedup_ours_vs_library": round(lib_ms / ours_ms, 3),
            "max_abs_diff_o": (o_ours.float() - o_fi.float()).abs().max().item(),
            "max_state_rel_diff": d_s, "library_first_call_s": round(compile_s, 1)}
        del inp, st_fi, st_ours
    except Exception as e:  # pragma: no cover
        out["decode_config1"] = {"unavailable": f"{e!r}"[:400]}
    return out


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
    """Contest-record replay (qk4_v8 geometry: Hq = Hk = 4, Hv = 8): latency of the
    public ``run`` entry points on every workload record of the reference's
    workloads/gdn/*.md, with seeded synthetic tensors of each record's shape: the
    54 decode records (batch_size) and the 100 prefill records (total_seq_len,
    num_seqs) under both cu_seqlens rewrites of the reference's scripts ("even",
    "uneven").  Back-to-back calls with inputs resident on the device, as a
    Solution harness calls them; per record: median of 5 batches of 20 calls (CUDA
    events), next to the C restatement of the reference on the host cores (within
    a time budget)."""
    from gdn_b200 import decode, prefill, workloads as W
    from gdn_b200.graphs import DecodeGraph
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
    by_batch = {}
    for i, B in enumerate(W.contest_decode_records()):
        if B not in by_batch:  # records share batch sizes: time each size once
            inp = W.make_decode_inputs(B, hq, hv, seed=500 + B)
            c_us = cpu_us(lambda: c_oracle.decode(*inp.args()))
            dinp = W.make_decode_inputs(B, hq, hv, seed=500 + B, device=dev)
            g_us = gpu_us(lambda: decode.run(*dinp.args()))
            dg = DecodeGraph(dinp.q, dinp.k, dinp.v, dinp.state.clone(), dinp.A_log, dinp.a,
                             dinp.dt_bias, dinp.b, dinp.scale)
            by_batch[B] = (g_us, gpu_us(dg.step), c_us)
        g_us, gr_us, c_us = by_batch[B]
        r = None if c_us is None else c_us / g_us
        if r:
            ratios.append(r)
        rows_d.append({"record": i, "batch": B, "us": round(g_us, 2), "graph_replay_us": round(gr_us, 2),
                       "cpu_us": c_us and round(c_us, 1), "speedup_vs_cpu": r and round(r, 1)})
    for j, (rec, split, lengths) in enumerate(W.contest_prefill_records()):
        inp = W.make_prefill_inputs(lengths, hq, hv, seed=700 + j)
        c_us = cpu_us(lambda: c_oracle.prefill(*inp.args()))
        dinp = W.make_prefill_inputs(lengths, hq, hv, seed=700 + j, device=dev)
        g_us = gpu_us(lambda: prefill.run(*dinp.args()))
        r = None if c_us is None else c_us / g_us
        if r:
            ratios.append(r)
        rows_p.append({"record": rec, "split": split, "num_seqs": len(lengths),
                       "total_seq_len": sum(lengths), "us": round(g_us, 2),
                       "cpu_us": c_us and round(c_us, 1), "speedup_vs_cpu": r and round(r, 1)})
    geo = math.exp(sum(math.log(r) for r in ratios) / len(ratios)) if ratios else None
    print(json.dumps({
        "metric": "contest-record replay latency (qk4_v8: Hq=Hk=4, Hv=8, d=128)", "unit": "us",
        "data": "synthetic tensors with the shapes of every contest workload record "
                "(54 decode, 100 prefill x {even, uneven} cu_seqlens)",
        "api": "gdn_b200.decode.run / gdn_b200.prefill.run, device-resident inputs",
        "cpu": {"impl": "oracle/gdn_oracle.c (C restatement of the reference definitions)",
                "cores": c_oracle.max_threads(), "note": "timed until the CPU budget is spent"},
        "geomean_speedup_vs_cpu": geo and round(geo, 1),
        "prefill_us_total": {s: round(sum(r["us"] for r in rows_p if r["split"] == s), 1)
                             for s in ("even", "uneven")},
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
    ap.add_argument("--no-library", action="store_true",
                    help="skip the FlashInfer library-baseline leg")
    ap.add_argument("--library-only", action="store_true",
                    help="run only the FlashInfer library-baseline leg and print its JSON")
    ap.add_argument("--pool-only", action="store_true",
                    help="run only the pooled-decode leg and print its JSON (profiling runs)")
    ap.add_argument("--cpu-budget", type=float, default=10.0)
    ap.add_argument("--batch-per-rank", type=int, default=256,
                    help="sequences per rank (default 256 = BASELINE config 1; smaller only for profiling)")
    ap.add_argument("--prefill-seqs", type=int, default=4)
    ap.add_argument("--prefill-len", type=int, default=16384)
    ap.add_argument("--prefill-steps", type=int, default=20)
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
        if args.library_only:
            dev = torch.device("cuda", local_rank)
            torch.cuda.set_device(dev)
            if rank == 0:
                print(json.dumps(run_library_baseline(args, dev)), flush=True)
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
