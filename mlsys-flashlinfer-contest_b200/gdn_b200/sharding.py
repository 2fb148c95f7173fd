"""Partitioning of the GDN path over the GPUs of one box.

The reference runs on one GPU (its definitions are already a TP=4 head slice of
Qwen3-Next, definitions/gdn/gdn_decode_qk4_v8_d128_k_last.md:7,16-18).  Across
GPUs the work splits into independent units with no data-path collective:

* decode: every (sequence, v-head) state is independent -> shard by sequence
  (``batch_shard``) or by v-head (``head_shard``); each rank keeps its state
  shard resident in its own HBM;
* prefill: heads are independent and the chunk scan stays per (sequence,
  head) -> shard v-heads in whole GVA groups (a q/k head and its Hv/Hq
  v-heads stay on one rank).  The only exchange is an optional all-gather of
  the output ``o`` when a caller needs all heads on every rank
  (``all_gather_heads``), one NCCL ``all_gather_into_tensor``.
"""
from __future__ import annotations

from dataclasses import dataclass

import torch


@dataclass(frozen=True)
class HeadShard:
    q0: int  # first q/k head of this rank
    q1: int  # one past the last
    v0: int  # first v-head
    v1: int

    @property
    def num_q_heads(self) -> int:
        return self.q1 - self.q0

    @property
    def num_v_heads(self) -> int:
        return self.v1 - self.v0


def head_shard(Hq: int, Hv: int, world: int, rank: int) -> HeadShard:
    """Contiguous v-heads in whole GVA groups: rank r gets q/k heads
    [r*Hq/W, (r+1)*Hq/W) and the v-heads that read them."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError("bad world/rank")
    if Hv % Hq:
        raise ValueError("num_v_heads must be a multiple of num_q_heads")
    if Hq % world:
        raise ValueError(f"num_q_heads={Hq} does not split over {world} ranks")
    rep = Hv // Hq
    per = Hq // world
    q0 = rank * per
    return HeadShard(q0, q0 + per, q0 * rep, (q0 + per) * rep)


def batch_shard(B: int, world: int, rank: int) -> tuple:
    """[start, stop) of the sequences owned by ``rank`` (balanced, contiguous)."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError("bad world/rank")
    base, rem = divmod(B, world)
    start = rank * base + min(rank, rem)
    return start, start + base + (1 if rank < rem else 0)


def slice_prefill_heads(inp, shard: HeadShard):
    """Per-rank copy of a PrefillInputs restricted to ``shard``'s heads
    (contiguous tensors, ready for the kernels)."""
    from .workloads import PrefillInputs
    v = slice(shard.v0, shard.v1)
    qs = slice(shard.q0, shard.q1)
    c = lambda t: t.contiguous()  # noqa: E731
    return PrefillInputs(c(inp.q[:, qs]), c(inp.k[:, qs]), c(inp.v[:, v]),
                         None if inp.state is None else c(inp.state[:, v]),
                         c(inp.A_log[v]), c(inp.a[:, v]), c(inp.dt_bias[v]), c(inp.b[:, v]),
                         inp.cu_seqlens, inp.scale)


def slice_decode_batch(inp, start: int, stop: int):
    from .workloads import DecodeInputs
    s = slice(start, stop)
    return DecodeInputs(inp.q[s].contiguous(), inp.k[s].contiguous(), inp.v[s].contiguous(),
                        None if inp.state is None else inp.state[s].contiguous(),
                        inp.A_log, inp.a[s].contiguous(), inp.dt_bias, inp.b[s].contiguous(),
                        inp.scale)


def all_gather_heads(o_local: torch.Tensor, group=None) -> torch.Tensor:
    """Gather head-sharded prefill outputs [T, Hv/W, D] from every rank into
    [T, Hv, D] (rank r's heads at [r*Hv/W, (r+1)*Hv/W)).  One
    all_gather_into_tensor into a rank-major buffer, then one permute copy."""
    import torch.distributed as dist
    world = dist.get_world_size(group)
    T, hl, D = o_local.shape
    buf = torch.empty((world * T, hl, D), dtype=o_local.dtype, device=o_local.device)
    dist.all_gather_into_tensor(buf, o_local.contiguous(), group=group)
    return buf.view(world, T, hl, D).permute(1, 0, 2, 3).reshape(T, world * hl, D)
