"""Host-side multi-rank logic on CPU: shard arithmetic, the head all-gather
reassembly over a world of 2 gloo ranks, and failure detection (a rank that
raises before the collective makes the others fail fast instead of hanging)."""
import os
import socket
import sys
import traceback

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from gdn_b200 import sharding as S
from gdn_b200 import workloads as W
from oracle import gdn_oracle as O


def test_head_shard_covers_all_heads_in_gva_groups():
    for Hq, Hv in [(16, 32), (4, 8), (8, 32)]:
        for world in [1, 2, 4, 8]:
            if Hq % world:
                with pytest.raises(ValueError):
                    S.head_shard(Hq, Hv, world, 0)
                continue
            shards = [S.head_shard(Hq, Hv, world, r) for r in range(world)]
            assert shards[0].v0 == 0 and shards[-1].v1 == Hv
            for a, b in zip(shards, shards[1:]):
                assert a.v1 == b.v0 and a.q1 == b.q0
            for s in shards:
                # every v-head's q/k head lives on the same rank
                for h in range(s.v0, s.v1):
                    assert s.q0 <= h // (Hv // Hq) < s.q1


def test_batch_shard_balanced():
    for B in [1, 7, 256, 2048]:
        for world in [1, 2, 3, 8]:
            parts = [S.batch_shard(B, world, r) for r in range(world)]
            assert parts[0][0] == 0 and parts[-1][1] == B
            sizes = [b - a for a, b in parts]
            assert max(sizes) - min(sizes) <= 1


def test_head_sharded_oracle_equals_full():
    # the recurrence is per head: computing each shard separately and
    # concatenating the heads reproduces the full-problem result exactly
    inp = W.make_prefill_inputs([20, 7], 4, 8, seed=3)
    full_o, full_s = O.prefill(*[O.to_numpy(x) if isinstance(x, torch.Tensor) else x
                                 for x in inp.args()])
    os_, ss_ = [], []
    for r in range(2):
        sh = S.slice_prefill_heads(inp, S.head_shard(4, 8, 2, r))
        o, s = O.prefill(*[O.to_numpy(x) if isinstance(x, torch.Tensor) else x for x in sh.args()])
        os_.append(o)
        ss_.append(s)
    assert np.array_equal(np.concatenate(os_, axis=1), full_o)
    assert np.array_equal(np.concatenate(ss_, axis=1), full_s)


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, mode, q):
    try:
        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        from datetime import timedelta
        dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=20))
        if mode == "gather":
            T, Hv, D = 5, 8, 128
            full = torch.arange(T * Hv * D, dtype=torch.float32).reshape(T, Hv, D)
            sh = S.head_shard(4, Hv, world, rank)
            out = S.all_gather_heads(full[:, sh.v0:sh.v1].contiguous())
            q.put((rank, bool(torch.equal(out, full))))
        elif mode == "fail":
            if rank == 1:
                raise RuntimeError("injected failure before the all-gather")
            try:
                S.all_gather_heads(torch.zeros(3, 4, 128))
                q.put((rank, "no-error"))
            except Exception as e:  # the collective must fail, not hang
                q.put((rank, "error:" + type(e).__name__))
        dist.destroy_process_group()
    except Exception:
        q.put((rank, "raised:" + traceback.format_exc().splitlines()[-1]))


def _run(world, mode, timeout=90):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, mode, q)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout)
    alive = [p for p in procs if p.is_alive()]
    for p in alive:
        p.kill()
    res = {}
    while not q.empty():
        r, v = q.get()
        res[r] = v
    return res, alive


def test_all_gather_heads_two_gloo_ranks():
    res, alive = _run(2, "gather")
    assert not alive
    assert res == {0: True, 1: True}


def test_rank_failure_is_detected_not_hung():
    res, alive = _run(2, "fail")
    assert not alive, "a surviving rank hung in the collective"
    assert res[1].startswith("raised:")
    assert res[0].startswith("error:") or res[0].startswith("raised:"), res
