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
PHASES = ["top barrier + store issue", "gates read", "state pass + signal", "wait MMA1",
          "A/P TMEM load", "A/P compute", "A/P sync", "inverse level 2b", "T tiles + signal",
          "(unused 9)", "(unused 10)", "next gates + wait Vn MMAs", "Vn drain + signal", "wait PV",
          "O epilogue", "KS drain | inverse level 0", "inverse level 1",
          "wait state update (prev chunk)", "inverse level 2a"]
# issue thread (warp 16): waits on the compute warps / TMA, and MMA issue
MMA_PHASES = ["wait S tile", "issue [K;Q] S", "wait T tiles", "issue T~V - T^KS", "(unused 4)",
              "(unused 5)", "wait next K/Q/V", "issue next MMA1", "wait Vn tiles", "issue PV",
              "issue state update", "wait state update", "issue TMA", "(unused 13)", "(unused 14)",
              "(unused 15)"]
CLK_SLOTS = 20  # per compute warp
EV_FLOATS = 96
DEBUG_TAIL = 16 * CLK_SLOTS + 16 + EV_FLOATS  # DBG_CLK [16][20], DBG_MCLK [16], DBG_EV [96]


def phase_cycles(L: int, Hq: int, Hv: int, head: int, seed: int = 3, chunk: int = 0):
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
            head, chunk, N.stream_handle(inp.q.device))
        N.check(rc, "gdn_prefill_chunked_debug")
    torch.cuda.synchronize()
    clk = dbg[nf - DEBUG_TAIL:].cpu().tolist()
    nch = (L + 63) // 64
    per_warp = [[clk[w * CLK_SLOTS + i] / nch for i in range(len(PHASES))] for w in range(16)]
    comp = {name: per_warp[0][i] for i, name in enumerate(PHASES)}
    issue = {name: clk[16 * CLK_SLOTS + i] / nch for i, name in enumerate(MMA_PHASES)}
    ev = dbg[nf - EV_FLOATS:].cpu().tolist()
    events = {"compute": [ev[w * 5:w * 5 + 5] for w in range(16)], "issue": ev[80:86]}
    return comp, issue, per_warp, events

def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--len", type=int, default=16384)
    ap.add_argument("--hq", type=int, default=16)
    ap.add_argument("--hv", type=int, default=32)
    ap.add_argument("--head", type=int, default=5)
    ap.add_argument("--json", action="store_true")
    ap.add_argument("--chunk", type=int, default=100, help="chunk whose handoff timestamps print")
    ap.add_argument("--warps", action="store_true", help="also print every warp's phase cycles")
    a = ap.parse_args()
    comp, issue, per_warp, events = phase_cycles(a.len, a.hq, a.hv, a.head, chunk=a.chunk)
    tot = sum(comp.values())
    if a.json:
        print(json.dumps({"len": a.len, "cycles_per_chunk": comp, "issue_thread": issue,
                          "per_warp": per_warp, "total": tot}))
        return
    print(f"sequence length {a.len}, Hq={a.hq}, Hv={a.hv}: {tot:.0f} SM cycles per chunk")
    print("compute warps: warp 0, then min / max over the 16 warps (lane 0 of each)")
    for i, (name, v) in enumerate(comp.items()):
        col = [per_warp[w][i] for w in range(16)]
        print(f"  {name:32s} {v:8.0f}  {100 * v / tot:5.1f}%   min {min(col):6.0f}  max {max(col):6.0f}"
              f"  (argmax warp {col.index(max(col))})")
    if a.warps:
        print("  " + " " * 32 + "".join(f"{w:6d}" for w in range(16)))
        for i, name in enumerate(comp):
            print(f"  {name:32s}" + "".join(f"{per_warp[w][i]:6.0f}" for w in range(16)))
    print("issue thread (warp 16):")
    for name, v in issue.items():
        print(f"  {name:32s} {v:8.0f}  {100 * v / tot:5.1f}%")
    iv = events["issue"]
    t0 = iv[0]
    print(f"handoff timestamps around chunk {a.chunk + 2} (cycles after the issue thread saw the Vn tiles):")
    for name, v in zip(["PV committed", "state update committed", "state update seen done",
                        "next loads issued", "next S tile seen"], iv[1:]):
        print(f"  issue: {name:28s} {v - t0:8.0f}")
    for w in range(16):
        e = [x - t0 for x in events["compute"][w]]
        print(f"  warp {w:2d}: Vn signalled {e[0]:6.0f}  PV seen {e[1]:6.0f}  O done {e[2]:6.0f}"
              f"  state seen {e[3]:6.0f}  barrier exit {e[4]:6.0f}")

if __name__ == "__main__":
    main()
