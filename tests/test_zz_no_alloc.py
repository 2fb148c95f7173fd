"""The no-allocation prefill entry, gdn_prefill_segmented_noalloc (C ABI).

Some callers cannot allocate device memory per call: a host whose device memory
belongs to its own allocator, or one that cannot afford the synchronisation that
cudaMalloc / cudaFree bring.  This entry runs the segmented prefill with its
scratch in a device array inside the library (GDN_NOALLOC_SCRATCH_BYTES per GPU)
instead of a caller's workspace.  Its outputs are checked against the entry that
takes a workspace (gdn_prefill_segmented) on two calls in a row, of different
shapes, so that the second call also shows that what the first left in the
shared array does not leak into it.  Both entries run the same job builder and
kernels in the same order on the same inputs, so the results must be bitwise
equal: a start state perturbed by stale scratch would differ.  This file is collected last: when it fails,
a run that stops at the first failure has run every other test already."""
import ctypes

import pytest
import torch

import parity as PT
from oracle import c_oracle as C
from gdn_b200 import _native as N, workloads as W

NOALLOC_BYTES = 16 << 20


def _args(d, out, ns):
    T = d.q.shape[0]
    Nseq = d.cu_seqlens.shape[0] - 1
    return [N.ptr(d.q), N.ptr(d.k), N.ptr(d.v), N.ptr(d.state), N.ptr(d.A_log), N.ptr(d.a),
            N.ptr(d.dt_bias), N.ptr(d.b), N.ptr(d.cu_seqlens), float(d.scale), N.ptr(out),
            N.ptr(ns), T, Nseq, d.q.shape[1], d.k.shape[1], d.v.shape[1], 128]


def _both(d, segments):
    """(no-alloc output, new_state), (workspace-entry output, new_state)."""
    L = N.lib()
    Nseq, Hv = d.cu_seqlens.shape[0] - 1, d.v.shape[1]
    stream = N.stream_handle(torch.device("cuda"))
    o1, s1 = torch.empty_like(d.v), torch.empty((Nseq, Hv, 128, 128), dtype=torch.float32,
                                                 device="cuda")
    rc = L.gdn_prefill_segmented_noalloc(*_args(d, o1, s1), 0, segments, stream)
    N.check(rc, "gdn_prefill_segmented_noalloc")
    need = L.gdn_prefill_segmented_workspace_bytes(Nseq, Hv, segments)
    assert 0 < need <= NOALLOC_BYTES
    ws = torch.empty(need, dtype=torch.uint8, device="cuda")
    o2, s2 = torch.empty_like(d.v), torch.empty_like(s1)
    rc = L.gdn_prefill_segmented(*_args(d, o2, s2), 0, segments, N.ptr(ws), need, stream)
    N.check(rc, "gdn_prefill_segmented")
    torch.cuda.synchronize()
    return (o1, s1), (o2, s2)


@pytest.mark.gpu
def test_noalloc_matches_workspace_entry_twice():
    L = N.lib()
    # call 1: one long and one short sequence, 8 heads, the automatic cut (segments
    # 0: the device picks each sequence's pieces)
    d1 = PT.to_device(W.make_prefill_inputs([8192, 700], 4, 8, seed=70))
    assert L.gdn_prefill_segments(8892, 2, 8) > 1
    (o1, s1), (r1, t1) = _both(d1, 0)
    assert torch.equal(o1, r1) and torch.equal(s1, t1)
    # call 2: another shape and a forced piece count through the same scratch (a
    # head shard of 4 x 4096 tokens, 4 heads, slow decay so the start states matter)
    w2 = W.make_prefill_inputs([4096] * 4, 2, 4, seed=71)
    w2.dt_bias[:] = -6.0
    ref_o, ref_s = C.prefill(*w2.args())  # the C oracle, on the CPU inputs
    d2 = PT.to_device(w2)
    (o2, s2), (r2, t2) = _both(d2, 5)
    assert torch.equal(o2, r2) and torch.equal(s2, t2)
    # and the pair is a correct prefill: call 2 against the oracle
    PT.assert_o_close(o2, ref_o)
    PT.assert_state_close(s2, ref_s.numpy(), PT.STATE_REL)


def test_noalloc_rejects_oversize():
    """Pieces that need more scratch than the array holds fail before any launch."""
    L = N.lib()
    P = ctypes.c_void_p
    need = L.gdn_prefill_segmented_workspace_bytes(64, 32, 8)
    assert need > NOALLOC_BYTES
    rc = L.gdn_prefill_segmented_noalloc(P(1 << 20), P(1 << 20), P(1 << 20), None, P(1 << 20),
                                         P(1 << 20), P(1 << 20), P(1 << 20), P(1 << 20), 0.0,
                                         P(1 << 20), P(1 << 21), 1 << 20, 64, 16, 16, 32, 128, 0,
                                         8, None)
    assert rc == N.GDN_ERR_VALUE
    msg = L.gdn_last_error().decode()
    assert "scratch" in msg and str(NOALLOC_BYTES) in msg
