"""Per-phase cycle breakdown of the fused chunked prefill kernel.

    python -m gdn_b200.profile_prefill [--len 16384] [--hq 16] [--hv 32] [--head 5]

Runs the diagnostic entry point ``gdn_prefill_chunked_debug`` (the same kernel,
built with SM-clock counters at its phase boundaries) on one synthetic sequence
and prints, for the CTA of (sequence 0, ``--head``), the cycles thread 0 spent in
each phase per chunk.  This is the counterpart of the reference's optional
%globaltimer warp profiler in its state-scan kernel (cuda_h_v2b.cu:56-121).
"""
from __future__ import annotations

import argparse
import json

import torch

from . import _native as N
from . import workloads as W

# order of the DBG_CLK slots written by the kernel
PHASES = ["wait state update (prev chunk)", "gates read", "state pass + signal", "wait MMA1",
          "A/P TMEM load", "A/P compute", "A/P sync", "inverse level 2b", "T tiles + signal", "wait MMA2",
          "W drain + signal", "next gates + wait MMA3", "Vn drain + signal", "wait PV",
          "O epilogue", "inverse level 0", "inverse level 1", "(unused)",
          "inverse level 2a"]
# issue thread (warp 16): waits on the compute warps / TMA, and MMA issue
MMA_PHASES = ["wait S tile", "issue QS", "wait T tiles", "issue MMA2", "wait W tile", "issue WS",
              "wait next K/Q/V", "issue next MMA1", "wait Vn tiles", "issue PV", "issue state update",
              "wait state update", "issue TMA", "(unused)", "(unused)", "(unused)"]
DEBUG_TAIL = 48  # DBG_CLK (32 floats), DBG_MCLK (16): the end of the dump


def phase_cycles(L: int, Hq: int, Hv: int, head: int, seed: int = 3):
    inp = W.make_prefill_inputs([L], Hq, Hv, seed=seed, device="cuda")
    lib = N.lib()
    nf = lib.gdn_prefill_chunked_debug_floats()
    dbg = torch.zeros(nf, dtype=torch.float32, device="cuda")
    out = torch.empty_like(inp.v)
    ns = torch.empty_like(inp.state)
    for _ in range(2):  # first call warms up
        rc = lib.gdn_prefill_chunked_debug(
            N.ptr(inp.q), N.ptr(inp.k), N.ptr(inp.v), N.ptr(inp.state), N.ptr(inp.A_log),
            N.ptr(inp.a), N.ptr(inp.dt_bias), N.ptr(inp.b), N.ptr(inp.cu_seqlens),
            float(inp.scale), N.ptr(out), N.ptr(ns), L, 1, Hq, Hq, Hv, 128, N.ptr(dbg), nf, 0,
            head, 0, N.stream_handle(inp.q.device))
        N.check(rc, "gdn_prefill_chunked_debug")
    torch.cuda.synchronize()
    clk = dbg[nf - DEBUG_TAIL:].cpu().tolist()
    nch = (L + 63) // 64
    comp = {name: clk[i] / nch for i, name in enumerate(PHASES)}
    issue = {name: clk[32 + i] / nch for i, name in enumerate(MMA_PHASES)}
    return comp, issue


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--len", type=int, default=16384)
    ap.add_argument("--hq", type=int, default=16)
    ap.add_argument("--hv", type=int, default=32)
    ap.add_argument("--head", type=int, default=5)
    ap.add_argument("--json", action="store_true")
    a = ap.parse_args()
    comp, issue = phase_cycles(a.len, a.hq, a.hv, a.head)
    tot = sum(comp.values())
    if a.json:
        print(json.dumps({"len": a.len, "cycles_per_chunk": comp, "issue_thread": issue,
                          "total": tot}))
        return
    print(f"sequence length {a.len}, Hq={a.hq}, Hv={a.hv}: {tot:.0f} SM cycles per chunk")
    print("compute warps (thread 0):")
    for name, v in comp.items():
        print(f"  {name:32s} {v:8.0f}  {100 * v / tot:5.1f}%")
    print("issue thread (warp 16):")
    for name, v in issue.items():
        print(f"  {name:32s} {v:8.0f}  {100 * v / tot:5.1f}%")

if __name__ == "__main__":
    main()
