"""Parity helpers shared by the GPU tests.

Tolerances: bf16 outputs within atol = rtol = 1e-2 of the
oracle; the fp32 final state within a norm-wise relative error of 1e-3 per
(sequence, v-head).  Kernels that keep the whole update in fp32 (decode,
recurrent prefill) are also held to a tighter bound, STATE_RTOL_FP32, so a
regression shows up long before the contract tolerance is reached.
"""
import numpy as np
import torch

from oracle import gdn_oracle as O

O_ATOL = 1e-2
O_RTOL = 1e-2
STATE_REL = 1e-3
STATE_RTOL_FP32 = 1e-5


def np_args(inp):
    return [O.to_numpy(x) if isinstance(x, torch.Tensor) else x for x in inp.args()]


def o_values(o):
    if isinstance(o, torch.Tensor):
        return O.to_numpy(o).astype(np.float64)
    return O.bf16_to_f32(o).astype(np.float64)


def assert_o_close(o_gpu, o_ref, atol=O_ATOL, rtol=O_RTOL):
    a, r = o_values(o_gpu), o_values(o_ref)
    assert a.shape == r.shape, (a.shape, r.shape)
    bad = np.abs(a - r) > atol + rtol * np.abs(r)
    assert not bad.any(), f"{bad.sum()} output elements outside atol={atol} rtol={rtol}; " \
                          f"max abs err {np.abs(a - r).max():.3e}"


def state_rel_per_head(ns_gpu, ns_ref):
    a = O.to_numpy(ns_gpu).astype(np.float64)
    r = np.asarray(ns_ref, np.float64)
    assert a.shape == r.shape
    a = a.reshape(-1, a.shape[-2] * a.shape[-1])
    r = r.reshape(-1, r.shape[-2] * r.shape[-1])
    num = np.linalg.norm(a - r, axis=1)
    den = np.maximum(np.linalg.norm(r, axis=1), 1e-30)
    rel = np.where(np.linalg.norm(r, axis=1) == 0, num, num / den)
    return float(rel.max()) if rel.size else 0.0


def assert_state_close(ns_gpu, ns_ref, rel=STATE_REL):
    e = state_rel_per_head(ns_gpu, ns_ref)
    assert e <= rel, f"state relative error {e:.3e} > {rel:.1e}"
    return e


def to_device(inp, device="cuda"):
    for f in ("q", "k", "v", "state", "A_log", "a", "dt_bias", "b", "cu_seqlens"):
        if hasattr(inp, f) and getattr(inp, f) is not None:
            setattr(inp, f, getattr(inp, f).to(device))
    return inp
