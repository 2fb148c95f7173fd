"""GDN decode entry point with the solution signature of the reference.

``run(q, k, v, state, A_log, a, dt_bias, b, scale) -> (output, new_state)`` is the
drop-in for ``gdn_decode/solution/python/gdn_decode_final.py::run`` (:23-36): same
argument order and meaning (definition input order, scale 0/None = 1/sqrt(128),
``state`` optional), same return tuple.  The reference returns fresh tensors for
B < 8 and updates ``state`` in place for B >= 8
(gdn_decode_kernel_large_batch.py:348,405-406); here ``run`` is out-of-place for
every B (definition-exact) and ``run_inplace`` is the explicit in-place form.
Both launch the single fused sm_100a decode kernel through the C ABI
(``gdn_decode`` in include/gdn_b200.h) on the current CUDA stream, by way of the
torch-tensor binding ``_gdn_torch`` (checks and output allocation in C++) when it
is built, else through ctypes after the Python checks below.
"""
from __future__ import annotations

import torch

from . import _native as N
from ._checks import HEAD, cuda_contig, dim, dtype, resolve_scale, same_device


def _validate(q, k, v, state, A_log, a, dt_bias, b, output, new_state):
    for name, t in (("q", q), ("k", k), ("v", v), ("A_log", A_log), ("a", a), ("dt_bias", dt_bias),
                    ("b", b), ("output", output), ("new_state", new_state)):
        cuda_contig(name, t)
    for name, t, d in (("q", q, 4), ("k", k, 4), ("v", v, 4), ("A_log", A_log, 1), ("a", a, 3),
                       ("dt_bias", dt_bias, 1), ("b", b, 3), ("output", output, 4),
                       ("new_state", new_state, 4)):
        dim(name, t, d)
    if state is not None:
        cuda_contig("state", state)
        dim("state", state, 4)
        dtype("state", state, torch.float32)
    same_device(q, k=k, v=v, state=state, A_log=A_log, a=a, dt_bias=dt_bias, b=b, output=output,
                new_state=new_state)
    for name, t in (("q", q), ("k", k), ("v", v), ("a", a), ("b", b), ("output", output)):
        dtype(name, t, torch.bfloat16)
    for name, t in (("A_log", A_log), ("dt_bias", dt_bias), ("new_state", new_state)):
        dtype(name, t, torch.float32)
    B, T, Hq, K = q.shape
    Hk, Hv, V = k.shape[2], v.shape[2], v.shape[3]
    if k.shape[0] != B or v.shape[0] != B:
        raise ValueError("batch mismatch among q/k/v")
    if k.shape[1] != T or v.shape[1] != T:
        raise ValueError("sequence length mismatch among q/k/v")
    if T != 1:
        raise ValueError("decode requires T=1")
    if K != HEAD or k.shape[3] != HEAD or V != HEAD:
        raise ValueError("head size must be 128")
    if Hk != Hq:
        raise ValueError("num_k_heads must equal num_q_heads")
    if Hv % Hq != 0:
        raise ValueError("HV must be divisible by Hq")
    if tuple(a.shape) != (B, T, Hv):
        raise ValueError("a must have shape [B, T, HV]")
    if tuple(b.shape) != (B, T, Hv):
        raise ValueError("b must have shape [B, T, HV]")
    if tuple(A_log.shape) != (Hv,):
        raise ValueError("A_log must have shape [HV]")
    if tuple(dt_bias.shape) != (Hv,):
        raise ValueError("dt_bias must have shape [HV]")
    if tuple(output.shape) != (B, T, Hv, V):
        raise ValueError("output must have shape [B, T, HV, V]")
    if tuple(new_state.shape) != (B, Hv, V, K):
        raise ValueError("new_state must have shape [B, HV, V, K]")
    if state is not None and tuple(state.shape) != (B, Hv, V, K):
        raise ValueError("state must have shape [B, HV, V, K]")
    return B, Hq, Hk, Hv


def launch(q, k, v, state, A_log, a, dt_bias, b, scale, output, new_state):
    """Destination-passing form: writes ``output`` and ``new_state`` (which may be
    ``state`` itself) and returns them."""
    ext = N.torch_ext()
    if ext is not None:
        return ext.decode(q, k, v, state, A_log, a, dt_bias, b, resolve_scale(scale), output,
                          new_state)
    B, Hq, Hk, Hv = _validate(q, k, v, state, A_log, a, dt_bias, b, output, new_state)
    with torch.cuda.device(q.device):
        rc = N.lib().gdn_decode(N.ptr(q), N.ptr(k), N.ptr(v), N.ptr(state), N.ptr(A_log), N.ptr(a),
                                N.ptr(dt_bias), N.ptr(b), resolve_scale(scale), N.ptr(output),
                                N.ptr(new_state), B, Hq, Hk, Hv, HEAD, N.stream_handle(q.device))
    N.check(rc, "gdn_decode")
    return output, new_state


def run(q, k, v, state, A_log, a, dt_bias, b, scale):
    """Out-of-place decode: returns (output [B,1,Hv,128] bf16, new_state [B,Hv,128,128] fp32)."""
    ext = N.torch_ext()
    if ext is not None:
        return ext.decode(q, k, v, state, A_log, a, dt_bias, b, resolve_scale(scale))
    output = torch.empty_like(v)
    B, Hv = v.shape[0], v.shape[2]
    new_state = torch.empty((B, Hv, HEAD, HEAD), dtype=torch.float32, device=v.device)
    return launch(q, k, v, state, A_log, a, dt_bias, b, scale, output, new_state)


def run_inplace(q, k, v, state, A_log, a, dt_bias, b, scale):
    """In-place decode (the reference's large-batch behaviour): ``state`` is
    overwritten with the new state and returned as the second element."""
    if state is None:
        raise ValueError("run_inplace needs a state tensor")
    output = torch.empty_like(v)
    return launch(q, k, v, state, A_log, a, dt_bias, b, scale, output, state)


def run_pool(q, k, v, A_log, a, dt_bias, b, scale, state_pool, in_slots, out_slots=None,
             intermediate=None, qk_l2norm: bool = False, no_state_update: bool = False,
             output=None):
    """Pooled multi-token decode (the serving form; C ABI ``gdn_decode_pool``).

    q, k [B,T,Hq,128] bf16; v [B,T,Hv,128] bf16; a, b [B,T,Hv] bf16;
    state_pool [P,Hv,128,128] fp32 or bf16, updated in place: sequence i starts
    from slot in_slots[i] (int32 [B]; negative or >= P = zero state) and its final
    state goes to out_slots[i] (default in_slots; negative or >= P = not written).
    intermediate: optional [B,T,Hv,128,128] tensor of the pool's dtype that gets
    the state after every token.  qk_l2norm normalises q and k per head in the
    kernel.  Returns output [B,T,Hv,128] bf16."""
    ext = N.torch_ext()
    if ext is not None:
        return ext.decode_pool(q, k, v, A_log, a, dt_bias, b, resolve_scale(scale), state_pool,
                               in_slots, out_slots, intermediate, qk_l2norm, no_state_update,
                               output)
    for name, t in (("q", q), ("k", k), ("v", v), ("A_log", A_log), ("a", a), ("dt_bias", dt_bias),
                    ("b", b), ("state_pool", state_pool), ("in_slots", in_slots)):
        cuda_contig(name, t)
    if state_pool.dtype not in (torch.float32, torch.bfloat16):
        raise TypeError("state_pool must be float32 or bfloat16")
    if in_slots.dtype != torch.int32 or (out_slots is not None and out_slots.dtype != torch.int32):
        raise TypeError("slot indices must be int32")
    B, T, Hq, _ = q.shape
    Hv = v.shape[2]
    if output is None:
        output = torch.empty_like(v)
    flags = (1 if qk_l2norm else 0) | (2 if no_state_update else 0)
    with torch.cuda.device(q.device):
        rc = N.lib().gdn_decode_pool(
            N.ptr(q), N.ptr(k), N.ptr(v), N.ptr(A_log), N.ptr(a), N.ptr(dt_bias), N.ptr(b),
            resolve_scale(scale), N.ptr(state_pool), 1 if state_pool.dtype == torch.bfloat16 else 0,
            state_pool.shape[0], N.ptr(in_slots), N.ptr(out_slots), N.ptr(intermediate), flags,
            N.ptr(output), B, T, Hq, k.shape[2], Hv, HEAD, N.stream_handle(q.device))
    N.check(rc, "gdn_decode_pool")
    return output

