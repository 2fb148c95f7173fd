"""Fused output all-gather of the head-sharded chunked prefill.  Two-rank checks on
two GPUs of one box (skipped with fewer): the output all-gather
fused into the chunked prefill kernel (every rank's output tiles written into every
rank's peer-mapped full buffer) must give every rank exactly the all-heads output of
a one-GPU call, and the head shards' new states must match it too.  With long
sequences a head shard has few (sequence, head) pairs and the call cuts them into
pieces (segmented prefill), so there the comparison is within the contract
tolerances (outputs atol = rtol = 1e-2, states 1e-3 relative per head).  The same
kernel path with 2, 4 and 8 ranks emulated on one GPU (the "peer" buffers are local
allocations) runs on any box."""
import os
import socket

import pytest
import torch

pytestmark = pytest.mark.gpu


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _close(out, ref, ns, s_ref):
    o, r = out.float(), ref.float()
    ok_o = bool(((o - r).abs() <= 1e-2 + 1e-2 * r.abs()).all())
    a, b = ns.double().flatten(2), s_ref.double().flatten(2)
    rel = (a - b).norm(dim=2) / b.norm(dim=2).clamp_min(1e-30)
    return ok_o, bool(rel.max() <= 1e-3)


def _rank_main(rank, world, port, result_path, long_seqs=False):
    import torch.distributed as dist
    from datetime import timedelta
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=60),
                            device_id=dev)
    try:
        from gdn_b200 import prefill, sharding as S, workloads as W
        lengths = [4096, 2048] if long_seqs else [300, 77, 129]
        full = W.make_prefill_inputs(lengths, 4, 8, seed=31, device=dev)
        o_ref, s_ref = prefill.run_chunked(*full.args())
        sh = S.head_shard(4, 8, world, rank)
        loc = S.slice_prefill_heads(full, sh)
        Hv_loc = sh.v1 - sh.v0
        cut = prefill.segments_for(sum(lengths), len(lengths), Hv_loc) > 1
        assert cut == long_seqs
        bufs = S.PeerOutputs(full.q.shape[0], 8, dev)
        out, ns = S.prefill_gathered(loc, sh.v0, bufs)
        torch.cuda.synchronize()
        dist.barrier()
        if long_seqs:
            ok_o, ok_s = _close(out, o_ref, ns, s_ref[:, sh.v0:sh.v1])
        else:
            ok_o = torch.equal(out, o_ref)
            ok_s = torch.equal(ns, s_ref[:, sh.v0:sh.v1])
        dist.barrier()
        bufs.close()
        with open(f"{result_path}.{rank}", "w") as f:
            f.write(f"{int(ok_o)} {int(ok_s)}")
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
@pytest.mark.parametrize("long_seqs", [False, True])
def test_fused_gather_prefill_two_ranks(tmp_path, long_seqs):
    import torch.multiprocessing as mp
    res = str(tmp_path / "res")
    mp.spawn(_rank_main, args=(2, _free_port(), res, long_seqs), nprocs=2, join=True)
    for r in range(2):
        assert open(f"{res}.{r}").read() == "1 1", f"rank {r}"


def _emulated_ranks(world, lengths, segments, seed):
    """The fused gather of `world` ranks emulated on one GPU: rank r's call (its head
    shard) stores its output tiles into its own full buffer and into the other
    world - 1 buffers, passed as "peer" pointers (local allocations here, so the
    kernel's multi-destination stores run without a second GPU).  The ranks' calls
    run one after another on one stream."""
    import ctypes
    from gdn_b200 import _native as N, prefill, sharding as S, workloads as W
    from gdn_b200._checks import HEAD, resolve_scale
    dev = torch.device("cuda", 0)
    Hq, Hv = 8, 16
    full = W.make_prefill_inputs(lengths, Hq, Hv, seed=seed, device=dev)
    o_ref, s_ref = prefill.run_chunked(*full.args())
    T = full.q.shape[0]
    nseq = len(lengths)
    bufs = [torch.full((T, Hv, HEAD), float("nan"), dtype=torch.bfloat16, device=dev)
            for _ in range(world)]
    states = []
    L = N.lib()
    for r in range(world):
        sh = S.head_shard(Hq, Hv, world, r)
        loc = S.slice_prefill_heads(full, sh)
        hl = sh.v1 - sh.v0
        ns = torch.empty((nseq, hl, HEAD, HEAD), dtype=torch.float32, device=dev)
        peers = [N.ptr(bufs[j]) for j in range(world) if j != r]
        arr = (ctypes.c_void_p * len(peers))(*peers)
        ws_bytes = L.gdn_prefill_segmented_workspace_bytes(nseq, hl, segments)
        ws = torch.empty(max(ws_bytes, 1), dtype=torch.uint8, device=dev)
        rc = L.gdn_prefill_chunked_peers(
            N.ptr(loc.q), N.ptr(loc.k), N.ptr(loc.v), N.ptr(loc.state), N.ptr(loc.A_log),
            N.ptr(loc.a), N.ptr(loc.dt_bias), N.ptr(loc.b), N.ptr(loc.cu_seqlens),
            resolve_scale(loc.scale), N.ptr(bufs[r]), N.ptr(ns), T, nseq, loc.q.shape[1],
            loc.k.shape[1], hl, HEAD, Hv, sh.v0, ctypes.cast(arr, ctypes.c_void_p), len(peers),
            segments, N.ptr(ws), ws_bytes, N.stream_handle(dev))
        N.check(rc, "gdn_prefill_chunked_peers")
        states.append(ns)
    torch.cuda.synchronize()
    return bufs, torch.cat(states, dim=1), o_ref, s_ref


@pytest.mark.parametrize("world", [2, 4, 8])
def test_fused_gather_emulated_ranks_one_gpu(world):
    # uncut (segments = 1): every buffer must hold exactly the one-call output
    bufs, ns, o_ref, s_ref = _emulated_ranks(world, [300, 77, 129], 1, seed=31)
    for r, b in enumerate(bufs):
        assert torch.equal(b, o_ref), f"buffer {r}"
    assert torch.equal(ns, s_ref)


@pytest.mark.parametrize("world", [2, 8])
def test_fused_gather_emulated_ranks_cut_one_gpu(world):
    # automatic cut (segments = 0): long sequences on 16 / world heads per call are
    # cut into pieces; every buffer gets the same stores, so they agree bitwise with
    # each other, and with the one-call output within the contract tolerances
    bufs, ns, o_ref, s_ref = _emulated_ranks(world, [4096, 2048], 0, seed=32)
    for r, b in enumerate(bufs):
        assert torch.equal(b, bufs[0]), f"buffer {r}"
    ok_o, ok_s = _close(bufs[0], o_ref, ns, s_ref)
    assert ok_o and ok_s
