"""Two-rank checks on two GPUs of one box (skipped with fewer): the output all-gather
fused into the chunked prefill kernel (every rank's output tiles written into every
rank's peer-mapped full buffer) must give every rank exactly the all-heads output of
a one-GPU call, and the head shards' new states must match it too.  With long
sequences a head shard has few (sequence, head) pairs and the call cuts them into
pieces (segmented prefill), so there the comparison is within the contract
tolerances (outputs atol = rtol = 1e-2, states 1e-3 relative per head)."""
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
