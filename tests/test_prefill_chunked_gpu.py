"""GPU parity of the fused chunked (tcgen05) prefill kernel: one chunk's
intermediates against the fp64 chunk algebra, then end-to-end outputs against
the recurrence oracle (numpy for small cases, the C restatement for large ones)
and the golden fixtures, plus size-independent properties at BASELINE sizes."""
import ctypes

import numpy as np
import pytest
import torch

import golden_io as G
import parity as PT
from oracle import c_oracle as C
from oracle import gdn_oracle as O
from gdn_b200 import _native as N, prefill, workloads as W

pytestmark = pytest.mark.gpu

DBG_NAMES = [("gam", 64), ("bet", 64), ("A", 4096), ("P", 4096), ("T", 4096), ("U", 8192),
             ("KS", 8192), ("Vn", 8192), ("QS", 8192), ("PV", 8192), ("St", 16384), ("clk", 320), ("mclk", 16), ("ev", 96)]


def chunked(q, k, v, state, A_log, a, dt_bias, b, cu_seqlens, scale):
    T, Nseq = q.shape[0], cu_seqlens.shape[0] - 1
    Hq, Hv = q.shape[1], v.shape[1]
    out = torch.empty_like(v)
    ns = torch.empty((Nseq, Hv, 128, 128), dtype=torch.float32, device=v.device)
    rc = N.lib().gdn_prefill_chunked(N.ptr(q), N.ptr(k), N.ptr(v), N.ptr(state), N.ptr(A_log),
                                     N.ptr(a), N.ptr(dt_bias), N.ptr(b), N.ptr(cu_seqlens),
                                     float(scale), N.ptr(out), N.ptr(ns), T, Nseq, Hq, Hq, Hv, 128,
                                     N.stream_handle(q.device))
    N.check(rc, "gdn_prefill_chunked")
    return out, ns


def debug_dump(inp, n, h, c):
    d = PT.to_device(inp)
    T, Nseq = d.q.shape[0], d.cu_seqlens.shape[0] - 1
    Hq, Hv = d.q.shape[1], d.v.shape[1]
    L = N.lib()
    nf = L.gdn_prefill_chunked_debug_floats()
    dbg = torch.full((nf,), float("nan"), dtype=torch.float32, device="cuda")
    out = torch.empty_like(d.v)
    ns = torch.empty((Nseq, Hv, 128, 128), dtype=torch.float32, device="cuda")
    rc = L.gdn_prefill_chunked_debug(N.ptr(d.q), N.ptr(d.k), N.ptr(d.v), N.ptr(d.state),
                                     N.ptr(d.A_log), N.ptr(d.a), N.ptr(d.dt_bias), N.ptr(d.b),
                                     N.ptr(d.cu_seqlens), float(d.scale), N.ptr(out), N.ptr(ns), T,
                                     Nseq, Hq, Hq, Hv, 128, N.ptr(dbg), nf, n, h, c,
                                     N.stream_handle(d.q.device))
    N.check(rc, "gdn_prefill_chunked_debug")
    torch.cuda.synchronize()
    x = dbg.cpu().numpy().astype(np.float64)
    res, off = {}, 0
    for name, size in DBG_NAMES:
        res[name] = x[off:off + size]
        off += size
    shapes = dict(A=(64, 64), P=(64, 64), T=(64, 64), U=(64, 128), KS=(64, 128), Vn=(64, 128),
                  QS=(64, 128), PV=(64, 128), St=(128, 128))
    for k_, s in shapes.items():
        res[k_] = res[k_].reshape(s)
    return res


def _rel(x, r, rows=None):
    if rows is not None:
        x, r = x[rows], r[rows]
    return float(np.linalg.norm(x - r) / max(np.linalg.norm(r), 1e-30))


@pytest.mark.parametrize("lengths,n,h,c", [([150], 0, 1, 1), ([40, 130], 1, 6, 2), ([64], 0, 0, 0)])
def test_chunk_intermediates(lengths, n, h, c):
    inp = W.make_prefill_inputs(lengths, 4, 8, seed=sum(lengths) + n + h)
    ref = O.chunk_intermediates(*PT.np_args(inp)[:9], n, h, c)
    got = debug_dump(inp, n, h, c)
    v = ref["valid"]
    assert np.allclose(got["gam"], ref["gam"], rtol=1e-5, atol=1e-5)
    assert np.allclose(got["bet"], ref["bet"], rtol=1e-5, atol=1e-6)
    assert np.abs(got["A"] - ref["A"]).max() < 1e-4
    assert _rel(got["P"], ref["P"], v) < 1e-5          # fp32 values before bf16 packing
    assert _rel(got["T"], ref["T"]) < 1e-4
    errs = {k_: _rel(got[k_], ref[k_], v) for k_ in ("KS", "Vn", "QS", "PV")}
    errs["St"] = _rel(got["St"], ref["St"])
    assert errs["KS"] < 1e-2, errs                       # bf16 S operand
    assert errs["QS"] < 1e-2 and errs["Vn"] < 2e-2, errs  # bf16 S operand
    assert errs["PV"] < 2e-2, errs
    assert errs["St"] < 1e-3, errs


CASES = [[1, 2], [63], [64], [65], [130, 0, 7], [200, 64, 1], [0, 5, 0], [129, 128, 127],
         [300], [1, 1, 1, 1]]


@pytest.mark.parametrize("lengths", CASES)
@pytest.mark.parametrize("geom", [(4, 8), (16, 32)])
def test_chunked_parity_small(lengths, geom):
    inp = W.make_prefill_inputs(lengths, geom[0], geom[1], seed=len(lengths) * 7 + sum(lengths),
                                zero_state_every_other=True)
    o_ref, s_ref = O.prefill(*PT.np_args(inp))
    o, ns = chunked(*PT.to_device(inp).args())
    torch.cuda.synchronize()
    PT.assert_o_close(o, o_ref)
    PT.assert_state_close(ns, s_ref, PT.STATE_REL)


@pytest.mark.parametrize("name", G.names("prefill"))
def test_chunked_matches_reference_golden(name):
    meta, z = G.load(name)
    inp = G.regenerate_inputs(meta)
    o, ns = chunked(*PT.to_device(inp).args())
    PT.assert_o_close(o, z["o"])
    G.check_state(O.to_numpy(ns), z, rtol=2e-3, atol=2e-4, sum_rtol=2e-3)


def test_chunked_state_none():
    inp = W.make_prefill_inputs([70, 9, 200], 4, 8, seed=12, with_state=False)
    o_ref, s_ref = O.prefill(*PT.np_args(inp))
    o, ns = chunked(*PT.to_device(inp).args())
    PT.assert_o_close(o, o_ref)
    PT.assert_state_close(ns, s_ref, PT.STATE_REL)


def test_chunked_slow_decay_long():
    # slow decay keeps the state alive across many chunks (the hard case for
    # bf16 operands); 1000 tokens, compared with the C recurrence
    inp = W.make_prefill_inputs([1000, 333], 4, 8, seed=21)
    inp.dt_bias[:] = -6.0
    o_ref, s_ref = C.prefill(*inp.args(), nthreads=8)
    o, ns = chunked(*PT.to_device(inp).args())
    PT.assert_o_close(o, o_ref)
    PT.assert_state_close(ns, s_ref.numpy(), PT.STATE_REL)


def test_chunked_config2_varlen():
    # 16 sequences, len ~ U[64, 1024], half zero states
    lens = W.config_lengths("prefill_varlen")
    inp = W.make_prefill_inputs(lens, 16, 32, seed=2, zero_state_every_other=True)
    o_ref, s_ref = C.prefill(*inp.args())
    o, ns = prefill.run(*PT.to_device(inp).args())
    PT.assert_o_close(o, o_ref)
    PT.assert_state_close(ns, s_ref.numpy(), PT.STATE_REL)


def test_chunked_config3_full_size_against_c_oracle():
    """BASELINE config 3 (4 x 16384 tokens, Hq=16, Hv=32, random fp32 initial
    states) through the chunked kernel; sequence 0 (all 32 v-heads, 16384 tokens)
    against the C oracle (the reference recurrence, definitions/gdn/
    gdn_prefill_qk4_v8_d128_k_last.md:62-142, on all host threads), and all four
    sequences against the token-recurrent kernel (fp32 throughout)."""
    cpu = W.make_prefill_inputs([16384] * 4, 16, 32, seed=3)
    L0 = 16384
    seq0 = W.PrefillInputs(cpu.q[:L0], cpu.k[:L0], cpu.v[:L0], cpu.state[:1], cpu.A_log,
                           cpu.a[:L0], cpu.dt_bias, cpu.b[:L0],
                           torch.tensor([0, L0], dtype=torch.int64), cpu.scale)
    o_ref, s_ref = C.prefill(*seq0.args())
    inp = PT.to_device(W.make_prefill_inputs([16384] * 4, 16, 32, seed=3))
    o1, s1 = chunked(*inp.args())
    torch.cuda.synchronize()
    PT.assert_o_close(o1[:L0], o_ref)
    err = PT.assert_state_close(s1[:1], s_ref.numpy(), PT.STATE_REL)
    print(f"config 3 sequence 0 (16384 tokens x 32 heads): state rel err {err:.3e} (bound 1e-3)")
    o2, s2 = prefill.run_recurrent(*inp.args())
    torch.cuda.synchronize()
    PT.assert_o_close(o1, o2)
    PT.assert_state_close(s1, s2.cpu().numpy(), PT.STATE_REL)


def test_chunked_deterministic():
    inp = PT.to_device(W.make_prefill_inputs([300, 77], 4, 8, seed=5))
    o1, s1 = chunked(*inp.args())
    o2, s2 = chunked(*inp.args())
    assert torch.equal(o1, o2) and torch.equal(s1, s2)


@pytest.mark.parametrize("lengths", [
    # 40 sequences at 8 heads (320 pairs, more than the SMs): both halves of the
    # kernel's 64-sequence ranking, equal lengths, empty sequences, long ones late
    [5, 700, 64, 64, 0, 130, 1, 900, 63, 300] * 4,
    # 24 sequences (192 pairs): 23 one-token sequences and the long one last
    [1] * 23 + [1500],
    # 64 sequences, the most the kernel ranks (lengths rising, so the order reverses)
    [1 + 37 * i for i in range(64)],
    # 65 sequences: more than it ranks, run in input order
    [1 + 37 * i for i in range(65)],
])
def test_chunked_multiwave_longest_first_bitwise(lengths):
    """A call with more (sequence, head) pairs than SMs hands its CTAs out
    longest sequence first (by chunk count).  A pair computes the same wherever its CTA sits in
    the grid, so the call must equal, bit for bit, one call per sequence (a
    single wave, not reordered), and the C oracle within the contract bounds."""
    cpu = W.make_prefill_inputs(lengths, 4, 8, seed=len(lengths) + 11, zero_state_every_other=True)
    o_ref, s_ref = C.prefill(*cpu.args())
    inp = PT.to_device(cpu)
    o, ns = chunked(*inp.args())
    torch.cuda.synchronize()
    PT.assert_o_close(o, o_ref)
    PT.assert_state_close(ns, s_ref.numpy(), PT.STATE_REL)
    cu = cpu.cu_seqlens.tolist()
    for i in range(len(lengths)):
        b0, e0 = cu[i], cu[i + 1]
        if e0 == b0:  # empty: zero final state (a call of no tokens is not made)
            assert not torch.any(ns[i]), f"sequence {i} is empty: its final state must be zero"
            continue
        one = W.PrefillInputs(inp.q[b0:e0], inp.k[b0:e0], inp.v[b0:e0], inp.state[i:i + 1],
                              inp.A_log, inp.a[b0:e0], inp.dt_bias, inp.b[b0:e0],
                              torch.tensor([0, e0 - b0], dtype=torch.int64, device="cuda"), inp.scale)
        o1, s1 = chunked(*one.args())
        assert torch.equal(o1, o[b0:e0]), f"sequence {i} ({e0 - b0} tokens): output differs"
        assert torch.equal(s1[0], ns[i]), f"sequence {i} ({e0 - b0} tokens): final state differs"


@pytest.mark.parametrize("geom", [(4, 8), (16, 32)])
def test_chunked_staged_state_matches_plain_bitwise(geom):
    """Calls of short sequences (T <= 1024 N) with an initial state read it through
    shared memory (TMA) instead of from global memory.  One 1100-token sequence
    alone (18 chunks on average: the plain kernel) and with an empty sequence beside
    it (9 on average: the staged kernel) must give the same output and final state
    bit for bit, the empty one a zero state."""
    Hq, Hv = geom
    one = W.make_prefill_inputs([1100], Hq, Hv, seed=23)
    d1 = PT.to_device(one)
    o1, s1 = chunked(*d1.args())
    state2 = torch.cat([d1.state, torch.randn_like(d1.state)])
    cu2 = torch.tensor([0, 1100, 1100], dtype=torch.int64, device="cuda")
    d2 = W.PrefillInputs(d1.q, d1.k, d1.v, state2, d1.A_log, d1.a, d1.dt_bias, d1.b, cu2, d1.scale)
    o2, s2 = chunked(*d2.args())
    torch.cuda.synchronize()
    assert torch.equal(o1, o2)
    assert torch.equal(s1[0], s2[0])
    assert not torch.any(s2[1])
    o_ref, s_ref = C.prefill(*W.make_prefill_inputs([1100], Hq, Hv, seed=23).args())
    PT.assert_o_close(o1, o_ref)
    PT.assert_state_close(s1, s_ref.numpy(), PT.STATE_REL)


def test_no_timeout_status_after_runs():
    st = ctypes.c_uint32(0)
    N.check(N.lib().gdn_read_status(ctypes.byref(st), 1))
    assert st.value & 1 == 0


def test_wait_probe_times_out_and_reports():
    L = N.lib()
    st = ctypes.c_uint32(0)
    N.check(L.gdn_read_status(ctypes.byref(st), 1))
    res = torch.full((1,), 7, dtype=torch.int32, device="cuda")
    N.check(L.gdn_wait_probe(20_000_000, N.ptr(res), N.stream_handle(res.device)))
    torch.cuda.synchronize()
    assert int(res.item()) == 0
    N.check(L.gdn_read_status(ctypes.byref(st), 1))
    assert st.value & 2
    N.check(L.gdn_read_status(ctypes.byref(st), 0))
    assert st.value == 0
