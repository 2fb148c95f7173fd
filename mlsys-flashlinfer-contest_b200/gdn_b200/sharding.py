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
  the output ``o`` when a caller needs all heads on every rank: either one NCCL
  ``all_gather_into_tensor`` after the kernel (``all_gather_heads``), or fused into
  the kernel (``PeerOutputs`` + ``prefill_gathered``): every rank's chunked kernel
  writes its output tiles into every rank's full output buffer over NVLink
  (buffers peer-mapped through CUDA IPC), so no collective runs at all.
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


class _DevBuf:
    """A raw device allocation seen by torch through __cuda_array_interface__."""

    def __init__(self, ptr: int, shape, typestr: str):
        self.__cuda_array_interface__ = {"shape": tuple(shape), "typestr": typestr,
                                         "data": (int(ptr), False), "version": 3}


class PeerOutputs:
    """Full prefill output buffers [T, Hv, 128] bf16, one per rank, each mapped into
    every other rank's address space (CUDA IPC), for ``prefill_gathered``.

    Collective to create (an all_gather_object of the IPC handles); ``close()``
    unmaps the peers' buffers and frees this rank's (it must run on every rank,
    after the last kernel that writes into the buffers has completed everywhere).
    The buffers are plain cudaMalloc allocations, outside torch's caching
    allocator, so the IPC handles cover exactly them."""

    def __init__(self, T: int, Hv: int, device, group=None):
        import torch.distributed as dist
        from cuda.bindings import runtime as rt
        self._rt = rt
        self.T, self.Hv = int(T), int(Hv)
        self.device = torch.device(device)
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        nbytes = max(self.T * self.Hv * 128 * 2, 16)
        with torch.cuda.device(self.device):
            err, ptr = rt.cudaMalloc(nbytes)
            self._check(err, "cudaMalloc")
            self._ptr = int(ptr)
            err, h = rt.cudaIpcGetMemHandle(self._ptr)
            self._check(err, "cudaIpcGetMemHandle")
        handles = [None] * self.world
        dist.all_gather_object(handles, bytes(h.reserved), group=group)
        self.peer_ptrs = []
        with torch.cuda.device(self.device):
            for r in range(self.world):
                if r == self.rank:
                    continue
                hr = rt.cudaIpcMemHandle_t()
                hr.reserved = handles[r]
                err, pp = rt.cudaIpcOpenMemHandle(hr, rt.cudaIpcMemLazyEnablePeerAccess)
                self._check(err, "cudaIpcOpenMemHandle")
                self.peer_ptrs.append(int(pp))
        raw = torch.as_tensor(_DevBuf(self._ptr, (self.T, self.Hv, 128), "<i2"), device=self.device)
        self.output = raw.view(torch.bfloat16)  # this rank's full output buffer

    def _check(self, err, what):
        if int(err) != 0:
            raise RuntimeError(f"{what} failed: {err}")

    def close(self):
        rt = self._rt
        with torch.cuda.device(self.device):
            for pp in self.peer_ptrs:
                rt.cudaIpcCloseMemHandle(pp)
            self.peer_ptrs = []
            if self._ptr:
                rt.cudaFree(self._ptr)
                self._ptr = 0


def prefill_gathered(inp_local, head_offset: int, bufs: PeerOutputs, new_state=None,
                     segments: int = 0, workspace=None):
    """Chunked prefill of this rank's heads (``inp_local`` as ``slice_prefill_heads``
    builds it) whose output tiles go to heads [head_offset, head_offset + Hv_local)
    of every rank's full output buffer (C ABI gdn_prefill_chunked_peers).  Returns
    (this rank's full output buffer, this rank's new states).  The buffer holds all
    heads only after every rank's call has completed: synchronise and barrier first.
    ``segments``: 0 = the automatic sequence-parallel cut (a head shard has few
    (sequence, head) pairs), 1 = none; the workspace is allocated when not given."""
    import ctypes
    from . import _native as N
    from ._checks import HEAD, resolve_scale
    q, k, v = inp_local.q, inp_local.k, inp_local.v
    T, Hq, _ = q.shape
    Hv = v.shape[1]
    Nseq = inp_local.cu_seqlens.shape[0] - 1
    if new_state is None:
        new_state = torch.empty((Nseq, Hv, HEAD, HEAD), dtype=torch.float32, device=q.device)
    peers = (ctypes.c_void_p * max(len(bufs.peer_ptrs), 1))(*bufs.peer_ptrs)
    L = N.lib()
    ws_bytes = L.gdn_prefill_segmented_workspace_bytes(Nseq, Hv, segments)
    if workspace is None and ws_bytes > 0:
        workspace = torch.empty(ws_bytes, dtype=torch.uint8, device=q.device)
    with torch.cuda.device(q.device):
        rc = L.gdn_prefill_chunked_peers(
            N.ptr(q), N.ptr(k), N.ptr(v), N.ptr(inp_local.state), N.ptr(inp_local.A_log),
            N.ptr(inp_local.a), N.ptr(inp_local.dt_bias), N.ptr(inp_local.b),
            N.ptr(inp_local.cu_seqlens), resolve_scale(inp_local.scale), N.ptr(bufs.output),
            N.ptr(new_state), T, Nseq, Hq, k.shape[1], Hv, HEAD, bufs.Hv, head_offset,
            ctypes.cast(peers, ctypes.c_void_p), len(bufs.peer_ptrs), segments, N.ptr(workspace),
            ws_bytes, N.stream_handle(q.device))
    N.check(rc, "gdn_prefill_chunked_peers")
    return bufs.output, new_state

