"""GDN prefill entry point with the solution signature of the reference.

``run(q, k, v, state, A_log, a, dt_bias, b, cu_seqlens, scale) -> (output, new_state)``
is the drop-in for ``gdn_prefill/solution/python/gdn_prefill_mix.py::run`` (:13-38):
same argument order and meaning, ``state`` optional (None = zero initial states),
``cu_seqlens`` int64 as in the definition (int32 is accepted and widened).
The call allocates the outputs and the workspace from the torch caching
allocator, then makes one C-ABI call (``gdn_prefill``, include/gdn_b200.h) that
enqueues every kernel on the current stream; the torch-tensor binding
``_gdn_torch`` does the checks, the allocation and the call in C++ when it is
built, else ctypes does the call after the Python checks below.  No host synchronisation: the
chunk layout is derived on the device from ``cu_seqlens``.
"""
from __future__ import annotations

import torch

from . import _native as N
from ._checks import HEAD, cuda_contig, dim, dtype, resolve_scale, same_device


def _validate(q, k, v, state, A_log, a, dt_bias, b, cu_seqlens, output, new_state):
    for name, t in (("q", q), ("k", k), ("v", v), ("A_log", A_log), ("a", a), ("dt_bias", dt_bias),
                    ("b", b), ("cu_seqlens", cu_seqlens), ("output", output),
                    ("new_state", new_state)):
        cuda_contig(name, t)
    for name, t, d in (("q", q, 3), ("k", k, 3), ("v", v, 3), ("A_log", A_log, 1), ("a", a, 2),
                       ("dt_bias", dt_bias, 1), ("b", b, 2), ("cu_seqlens", cu_seqlens, 1),
                       ("output", output, 3), ("new_state", new_state, 4)):
        dim(name, t, d)
    T, Hq, K = q.shape
    Nseq = cu_seqlens.shape[0] - 1
    if Nseq <= 0:
        raise ValueError("must have at least one sequence")
    Hk, Hv = k.shape[1], v.shape[1]
    if K != HEAD or k.shape[2] != HEAD or v.shape[2] != HEAD:
        raise ValueError("head size must be 128")
    if k.shape[0] != T or v.shape[0] != T:
        raise ValueError("k/v shape mismatch")
    if Hk != Hq:
        raise ValueError("num_k_heads must equal num_q_heads")
    if Hv % Hq != 0:
        raise ValueError("num_v_heads must be divisible by num_q_heads")
    if tuple(a.shape) != (T, Hv):
        raise ValueError("a shape mismatch")
    if tuple(b.shape) != (T, Hv):
        raise ValueError("b shape mismatch")
    if tuple(A_log.shape) != (Hv,) or tuple(dt_bias.shape) != (Hv,):
        raise ValueError("A_log / dt_bias must have shape [HV]")
    for name, t in (("q", q), ("k", k), ("v", v), ("a", a), ("b", b), ("output", output)):
        dtype(name, t, torch.bfloat16)
    for name, t in (("A_log", A_log), ("dt_bias", dt_bias), ("new_state", new_state)):
        dtype(name, t, torch.float32)
    if cu_seqlens.dtype != torch.int64:
        raise TypeError("cu_seqlens must be int64")
    if tuple(output.shape) != (T, Hv, HEAD):
        raise ValueError("output shape mismatch")
    if tuple(new_state.shape) != (Nseq, Hv, HEAD, HEAD):
        raise ValueError("new_state shape mismatch")
    if state is not None:
        cuda_contig("state", state)
        dim("state", state, 4)
        dtype("state", state, torch.float32)
        if tuple(state.shape) != (Nseq, Hv, HEAD, HEAD):
            raise ValueError("state shape mismatch")
    same_device(q, k=k, v=v, state=state, A_log=A_log, a=a, dt_bias=dt_bias, b=b,
                cu_seqlens=cu_seqlens, output=output, new_state=new_state)
    return T, Nseq, Hq, Hk, Hv


def workspace_bytes(T: int, Nseq: int, Hq: int, Hv: int) -> int:
    return int(N.lib().gdn_prefill_workspace_bytes(T, Nseq, Hq, Hv))


def _widen(cu_seqlens):
    if isinstance(cu_seqlens, torch.Tensor) and cu_seqlens.dtype == torch.int32:
        return cu_seqlens.to(torch.int64)
    return cu_seqlens


def launch(q, k, v, state, A_log, a, dt_bias, b, cu_seqlens, scale, output, new_state,
           workspace=None, recurrent: bool = False, use_qk_l2norm: bool = False,
           chunked: bool = False):
    """Destination-passing form.  ``recurrent=True`` forces the token-recurrent
    CUDA-core kernel (the reference's path for tiny inputs), ``chunked=True`` the
    fused chunked kernel; ``use_qk_l2norm`` L2-normalises q and k per head in the
    kernels (x / sqrt(sum x^2 + 1e-6); C ABI gdn_prefill_ex)."""
    cu_seqlens = _widen(cu_seqlens)
    path = 1 if recurrent else (2 if chunked else 0)
    ext = N.torch_ext()
    if ext is not None and workspace is None:
        return ext.prefill(q, k, v, state, A_log, a, dt_bias, b, cu_seqlens, resolve_scale(scale),
                           output, new_state, path, use_qk_l2norm, 0)
    T, Nseq, Hq, Hk, Hv = _validate(q, k, v, state, A_log, a, dt_bias, b, cu_seqlens, output,
                                    new_state)
    L = N.lib()
    with torch.cuda.device(q.device):
        stream = N.stream_handle(q.device)
        if use_qk_l2norm or chunked:
            rc = L.gdn_prefill_ex(N.ptr(q), N.ptr(k), N.ptr(v), N.ptr(state), N.ptr(A_log),
                                  N.ptr(a), N.ptr(dt_bias), N.ptr(b), N.ptr(cu_seqlens),
                                  resolve_scale(scale), N.ptr(output), N.ptr(new_state), T, Nseq,
                                  Hq, Hk, Hv, HEAD, 1 if use_qk_l2norm else 0, path, stream)
            N.check(rc, "gdn_prefill_ex")
            return output, new_state
        if recurrent:
            rc = L.gdn_prefill_recurrent(N.ptr(q), N.ptr(k), N.ptr(v), N.ptr(state), N.ptr(A_log),
                                         N.ptr(a), N.ptr(dt_bias), N.ptr(b), N.ptr(cu_seqlens),
                                         resolve_scale(scale), N.ptr(output), N.ptr(new_state), T,
                                         Nseq, Hq, Hk, Hv, HEAD, stream)
            N.check(rc, "gdn_prefill_recurrent")
            return output, new_state
        ws_bytes = workspace_bytes(T, Nseq, Hq, Hv)
        if workspace is None and ws_bytes > 0:
            workspace = torch.empty(ws_bytes, dtype=torch.uint8, device=q.device)
        if workspace is not None and workspace.numel() * workspace.element_size() < ws_bytes:
            raise ValueError(f"workspace too small: need {ws_bytes} bytes")
        rc = L.gdn_prefill(N.ptr(q), N.ptr(k), N.ptr(v), N.ptr(state), N.ptr(A_log), N.ptr(a),
                           N.ptr(dt_bias), N.ptr(b), N.ptr(cu_seqlens), resolve_scale(scale),
                           N.ptr(output), N.ptr(new_state), T, Nseq, Hq, Hk, Hv, HEAD,
                           N.ptr(workspace), ws_bytes, stream)
        N.check(rc, "gdn_prefill")
    return output, new_state


def run(q, k, v, state, A_log, a, dt_bias, b, cu_seqlens, scale, use_qk_l2norm: bool = False):
    """Returns (output [T,Hv,128] bf16, new_state [N,Hv,128,128] fp32).
    ``use_qk_l2norm`` (not in the reference's signature; keyword only in practice)
    L2-normalises q and k per head inside the kernels."""
    ext = N.torch_ext()
    if ext is not None:
        return ext.prefill(q, k, v, state, A_log, a, dt_bias, b, _widen(cu_seqlens),
                           resolve_scale(scale), None, None, 0, use_qk_l2norm, 0)
    Nseq = cu_seqlens.shape[0] - 1
    Hv = v.shape[1]
    output = torch.empty_like(v)
    new_state = torch.empty((max(Nseq, 0), Hv, HEAD, HEAD), dtype=torch.float32, device=v.device)
    return launch(q, k, v, state, A_log, a, dt_bias, b, cu_seqlens, scale, output, new_state,
                  use_qk_l2norm=use_qk_l2norm)


def run_recurrent(q, k, v, state, A_log, a, dt_bias, b, cu_seqlens, scale,
                  use_qk_l2norm: bool = False):
    """Token-recurrent prefill (no workspace)."""
    ext = N.torch_ext()
    if ext is not None:
        return ext.prefill(q, k, v, state, A_log, a, dt_bias, b, _widen(cu_seqlens),
                           resolve_scale(scale), None, None, 1, use_qk_l2norm, 0)
    Nseq = cu_seqlens.shape[0] - 1
    output = torch.empty_like(v)
    new_state = torch.empty((max(Nseq, 0), v.shape[1], HEAD, HEAD), dtype=torch.float32,
                            device=v.device)
    return launch(q, k, v, state, A_log, a, dt_bias, b, cu_seqlens, scale, output, new_state,
                  recurrent=True, use_qk_l2norm=use_qk_l2norm)


def run_chunked(q, k, v, state, A_log, a, dt_bias, b, cu_seqlens, scale,
                use_qk_l2norm: bool = False):
    """The fused chunked kernel whatever the size (the default dispatch sends
    tiny inputs to the recurrent kernel)."""
    Nseq = cu_seqlens.shape[0] - 1
    output = torch.empty_like(v)
    new_state = torch.empty((max(Nseq, 0), v.shape[1], HEAD, HEAD), dtype=torch.float32,
                            device=v.device)
    return launch(q, k, v, state, A_log, a, dt_bias, b, cu_seqlens, scale, output, new_state,
                  chunked=True, use_qk_l2norm=use_qk_l2norm)


def segments_for(T: int, Nseq: int, Hv: int) -> int:
    """Upper bound of the automatic piece count of the segmented prefill (1: the call
    is not cut); the device picks each sequence's count under it."""
    return int(N.lib().gdn_prefill_segments(T, Nseq, Hv))


def run_segmented(q, k, v, state, A_log, a, dt_bias, b, cu_seqlens, scale, segments: int = 0,
                  use_qk_l2norm: bool = False, output=None, new_state=None):
    """Sequence-parallel prefill (C ABI gdn_prefill_segmented): sequences of at least
    2 * segments chunks are cut into ``segments`` pieces whose start states follow
    from each piece's transition matrix; ``segments`` 0 = automatic (each sequence's
    count chosen on the device from its length).  Returns (output, new_state)."""
    cu_seqlens = _widen(cu_seqlens)
    ext = N.torch_ext()
    if ext is not None:
        return ext.prefill(q, k, v, state, A_log, a, dt_bias, b, cu_seqlens, resolve_scale(scale),
                           output, new_state, 3, use_qk_l2norm, segments)
    T, Nseq, Hq, Hk, Hv = _validate(q, k, v, state, A_log, a, dt_bias, b, cu_seqlens, output,
                                    new_state)
    if output is None:
        output = torch.empty_like(v)
    if new_state is None:
        new_state = torch.empty((Nseq, Hv, HEAD, HEAD), dtype=torch.float32, device=v.device)
    L = N.lib()
    G = segments
    ws_bytes = int(L.gdn_prefill_segmented_workspace_bytes(Nseq, Hv, G))
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device=q.device) if ws_bytes else None
    with torch.cuda.device(q.device):
        rc = L.gdn_prefill_segmented(N.ptr(q), N.ptr(k), N.ptr(v), N.ptr(state), N.ptr(A_log),
                                     N.ptr(a), N.ptr(dt_bias), N.ptr(b), N.ptr(cu_seqlens),
                                     resolve_scale(scale), N.ptr(output), N.ptr(new_state), T,
                                     Nseq, Hq, Hk, Hv, HEAD, 1 if use_qk_l2norm else 0, G,
                                     N.ptr(ws), ws_bytes, N.stream_handle(q.device))
    N.check(rc, "gdn_prefill_segmented")
    return output, new_state
