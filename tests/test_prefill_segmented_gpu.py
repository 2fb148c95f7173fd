"""GPU parity of the segmented (sequence-parallel) prefill, C ABI gdn_prefill_segmented:
sequences cut into pieces whose start states come from each piece's transition
matrix (S_{g+1} = S_g P_g + F_g), against the CPU oracles on the same inputs.
Cases cover cut and uncut sequences in one call, empty and partial-chunk
sequences, zero and given initial states, slow decay (the state carries across
every piece boundary), q/k L2 norm, automatic cuts whose first piece is longer
than the others, the gdn_prefill dispatch with a workspace, and the fused-gather
routing that the multi-GPU path uses."""
import ctypes

import numpy as np
import pytest
import torch

import parity as PT
from oracle import c_oracle as C
from oracle import gdn_oracle as O
from gdn_b200 import _native as N, prefill, workloads as W

pytestmark = pytest.mark.gpu

CASES = [
    ([300], 2),                   # two pieces: piece 1 starts from piece 0's final state
    ([700], 3),                   # one middle piece (F, P, one combine)
    ([1000, 333], 4),             # the second sequence is cut too (333 tokens = 6 chunks)
    ([129, 513, 64, 5, 0], 3),    # short sequences stay whole next to a cut one
    ([640, 64 * 9 + 17], 5),      # partial last chunk in the last piece
]


@pytest.mark.parametrize("lengths,G", CASES)
@pytest.mark.parametrize("geom", [(4, 8), (16, 32)])
def test_segmented_matches_oracle(lengths, G, geom):
    inp = W.make_prefill_inputs(lengths, geom[0], geom[1], seed=sum(lengths) + G,
                                zero_state_every_other=True)
    o_ref, s_ref = C.prefill(*inp.args(), nthreads=8)
    o, ns = prefill.run_segmented(*PT.to_device(inp).args(), segments=G)
    torch.cuda.synchronize()
    PT.assert_o_close(o, o_ref)
    PT.assert_state_close(ns, s_ref.numpy(), PT.STATE_REL)


@pytest.mark.parametrize("G", [3, 6])
def test_segmented_slow_decay(G):
    # dt_bias = -6: the per-token decay is ~0.9975, so the state carries across
    # every piece boundary and the start states depend on the combine
    inp = W.make_prefill_inputs([1500, 700], 4, 8, seed=31 + G)
    inp.dt_bias[:] = -6.0
    o_ref, s_ref = C.prefill(*inp.args(), nthreads=8)
    o, ns = prefill.run_segmented(*PT.to_device(inp).args(), segments=G)
    PT.assert_o_close(o, o_ref)
    PT.assert_state_close(ns, s_ref.numpy(), PT.STATE_REL)


def test_segmented_state_none_and_l2norm():
    inp = W.make_prefill_inputs([900, 260], 4, 8, seed=5, with_state=False, normalized_qk=False)
    o_ref, s_ref = O.prefill(*PT.np_args(inp), qk_l2norm=True)
    o, ns = prefill.run_segmented(*PT.to_device(inp).args(), segments=4, use_qk_l2norm=True)
    PT.assert_o_close(o, o_ref)
    PT.assert_state_close(ns, s_ref, PT.STATE_REL)


@pytest.mark.parametrize("lengths", [[4096] * 4, [4096, 2048, 1024, 512], [8192, 64, 64, 300]])
def test_segmented_close_to_chunked_long(lengths):
    # a head shard of a multi-GPU call, and ragged batches: the automatic form
    # picks each sequence's pieces on the device; against the one-chain kernel
    inp = PT.to_device(W.make_prefill_inputs(lengths, 4, 4, seed=8 + len(lengths)))
    assert prefill.segments_for(sum(lengths), len(lengths), 4) >= 3
    o1, s1 = prefill.run_chunked(*inp.args())
    o2, s2 = prefill.run_segmented(*inp.args(), segments=0)
    PT.assert_o_close(o2, o1)
    PT.assert_state_close(s2, s1.cpu().numpy(), PT.STATE_REL)


# Automatic cuts with piece 0 of two shares (w = 2 under the job builder's rules):
# 64 or 32 (sequence, head) pairs leave too few SMs for one wave of F/P jobs of
# equal pieces, so the F/P jobs take two waves while piece 0 runs twice as long.
# (lengths, Hq, Hv): a ragged batch at 16 heads (5 and 4 pieces, two sequences
# whole), 4 x 4096 at 8 heads (4 pieces each).
UNEVEN = [([4096, 3000, 2048, 1024], 8, 16), ([4096] * 4, 4, 8)]


@pytest.mark.parametrize("lengths,hq,hv", UNEVEN)
def test_segmented_uneven_pieces_match_oracle(lengths, hq, hv):
    inp = W.make_prefill_inputs(lengths, hq, hv, seed=60 + len(lengths) + hv,
                                zero_state_every_other=True)
    assert prefill.segments_for(sum(lengths), len(lengths), hv) >= 3
    o_ref, s_ref = C.prefill(*inp.args(), nthreads=8)
    o, ns = prefill.run_segmented(*PT.to_device(inp).args(), segments=0)
    torch.cuda.synchronize()
    PT.assert_o_close(o, o_ref)
    PT.assert_state_close(ns, s_ref.numpy(), PT.STATE_REL)


def test_segmented_uneven_slow_decay():
    # the state carries across every piece boundary (dt_bias = -6: per-token decay
    # ~0.9975).  At this decay the bf16 state operand of the chunk step bounds the
    # accuracy of any path (the one-chain kernel reaches ~1.0e-3 at 2048 such
    # tokens), and a cut of 64 pairs pays only for sequences of more than ~2300
    # tokens; so the cut is held to the one-chain kernel's own error on the same
    # inputs (it must add none), and both stay within twice the contract bound
    inp = W.make_prefill_inputs([4096, 3000, 2048, 1024], 8, 16, seed=77)
    inp.dt_bias[:] = -6.0
    o_ref, s_ref = C.prefill(*inp.args(), nthreads=8)
    d = PT.to_device(inp)
    o, ns = prefill.run_segmented(*d.args(), segments=0)
    _, ns1 = prefill.run_chunked(*d.args())
    torch.cuda.synchronize()
    PT.assert_o_close(o, o_ref)
    err = PT.state_rel_per_head(ns, s_ref.numpy())
    err1 = PT.state_rel_per_head(ns1, s_ref.numpy())
    assert err <= 1.05 * err1 + 1e-5, (err, err1)
    assert err1 <= 2 * PT.STATE_REL, err1


def test_dispatch_with_workspace_takes_segmented():
    # gdn_prefill (the reference-shaped entry) cuts when given the workspace it asks for
    inp = PT.to_device(W.make_prefill_inputs([8192], 4, 8, seed=12))
    d = inp
    T, Hq, Hv, Nseq = 8192, 4, 8, 1
    L = N.lib()
    assert L.gdn_prefill_segments(T, Nseq, Hv) > 1
    ws_bytes = prefill.workspace_bytes(T, Nseq, Hq, Hv)
    assert ws_bytes > 0
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device="cuda")
    out = torch.empty_like(d.v)
    ns = torch.empty((Nseq, Hv, 128, 128), dtype=torch.float32, device="cuda")
    rc = L.gdn_prefill(N.ptr(d.q), N.ptr(d.k), N.ptr(d.v), N.ptr(d.state), N.ptr(d.A_log),
                       N.ptr(d.a), N.ptr(d.dt_bias), N.ptr(d.b), N.ptr(d.cu_seqlens),
                       float(d.scale), N.ptr(out), N.ptr(ns), T, Nseq, Hq, Hq, Hv, 128, N.ptr(ws),
                       ws_bytes, N.stream_handle(torch.device("cuda")))
    N.check(rc, "gdn_prefill")
    o2, s2 = prefill.run_segmented(*d.args())
    torch.cuda.synchronize()
    assert torch.equal(out, o2) and torch.equal(ns, s2)  # same pieces, same kernels
    o_ref, s_ref = C.prefill(*W.make_prefill_inputs([8192], 4, 8, seed=12).args(), nthreads=8)
    PT.assert_o_close(out, o_ref)
    PT.assert_state_close(ns, s_ref.numpy(), PT.STATE_REL)


def test_segmented_rejects_small_workspace():
    inp = PT.to_device(W.make_prefill_inputs([700], 4, 8, seed=2))
    d = inp
    L = N.lib()
    need = L.gdn_prefill_segmented_workspace_bytes(1, 8, 3)
    ws = torch.empty(need, dtype=torch.uint8, device="cuda")
    out = torch.empty_like(d.v)
    ns = torch.empty((1, 8, 128, 128), dtype=torch.float32, device="cuda")
    rc = L.gdn_prefill_segmented(N.ptr(d.q), N.ptr(d.k), N.ptr(d.v), N.ptr(d.state),
                                 N.ptr(d.A_log), N.ptr(d.a), N.ptr(d.dt_bias), N.ptr(d.b),
                                 N.ptr(d.cu_seqlens), float(d.scale), N.ptr(out), N.ptr(ns), 700,
                                 1, 4, 4, 8, 128, 0, 3, N.ptr(ws), need - 256,
                                 N.stream_handle(torch.device("cuda")))
    assert rc == N.GDN_ERR_VALUE
    assert b"workspace" in L.gdn_last_error()


def test_segmented_fused_gather_routing():
    # the peers entry with no peers: this call's heads land at head_offset of a
    # wider output buffer, cut into pieces like the plain call
    full = W.make_prefill_inputs([2048, 1024], 4, 8, seed=40)
    o_ref, s_ref = C.prefill(*full.args(), nthreads=8)
    d = PT.to_device(full)
    lo, hi = 4, 8   # heads 4-7 of 8, q/k heads 2-3 (GVA 2)
    qs, ks = d.q[:, 2:4].contiguous(), d.k[:, 2:4].contiguous()
    vs, a_s, bs = d.v[:, lo:hi].contiguous(), d.a[:, lo:hi].contiguous(), d.b[:, lo:hi].contiguous()
    st = d.state[:, lo:hi].contiguous()
    out = torch.zeros((3072, 8, 128), dtype=torch.bfloat16, device="cuda")
    ns = torch.empty_like(st)
    L = N.lib()
    G = 4
    need = L.gdn_prefill_segmented_workspace_bytes(2, 4, G)
    ws = torch.empty(need, dtype=torch.uint8, device="cuda")
    arr = (ctypes.c_void_p * 1)()
    rc = L.gdn_prefill_chunked_peers(N.ptr(qs), N.ptr(ks), N.ptr(vs), N.ptr(st),
                                     N.ptr(d.A_log[lo:hi].contiguous()), N.ptr(a_s),
                                     N.ptr(d.dt_bias[lo:hi].contiguous()), N.ptr(bs),
                                     N.ptr(d.cu_seqlens), float(d.scale), N.ptr(out), N.ptr(ns),
                                     3072, 2, 2, 2, 4, 128, 8, lo,
                                     ctypes.cast(arr, ctypes.c_void_p), 0, G, N.ptr(ws), need,
                                     N.stream_handle(torch.device("cuda")))
    N.check(rc, "gdn_prefill_chunked_peers")
    torch.cuda.synchronize()
    PT.assert_o_close(out[:, lo:hi].contiguous(), o_ref[:, lo:hi].contiguous())
    assert torch.count_nonzero(out[:, :lo]) == 0
    PT.assert_state_close(ns, np.ascontiguousarray(s_ref.numpy()[:, lo:hi]), PT.STATE_REL)
