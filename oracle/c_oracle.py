"""ctypes binding of oracle/libgdn_oracle.so (the C restatement in gdn_oracle.c).

TEST INFRASTRUCTURE ONLY: used by tests/ as a second checker and by bench.py as
the timed CPU baseline.  Inputs are torch CPU tensors in the definition layouts.
"""
from __future__ import annotations

import ctypes
import os
import subprocess
from pathlib import Path

import torch

HERE = Path(__file__).resolve().parent
LIB = HERE / "libgdn_oracle.so"
_lib = None


def build(force: bool = False) -> Path:
    if force or not LIB.exists() or LIB.stat().st_mtime < (HERE / "gdn_oracle.c").stat().st_mtime:
        subprocess.run(["make", "-s", "-C", str(HERE), "libgdn_oracle.so"], check=True)
    return LIB


def lib():
    global _lib
    if _lib is None:
        if not LIB.exists():
            build()
        L = ctypes.CDLL(str(LIB))
        P, I64, F, I = ctypes.c_void_p, ctypes.c_int64, ctypes.c_float, ctypes.c_int
        L.gdn_oracle_decode.argtypes = [P, P, P, P, P, P, P, P, F, P, P, I64, I64, I64, I]
        L.gdn_oracle_prefill.argtypes = [P, P, P, P, P, P, P, P, P, I64, F, P, P, I64, I64, I]
        L.gdn_oracle_max_threads.restype = I
        _lib = L
    return _lib


def _p(t):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def _c(t):
    return None if t is None else t.detach().cpu().contiguous()


def max_threads() -> int:
    return int(lib().gdn_oracle_max_threads())


def decode(q, k, v, state, A_log, a, dt_bias, b, scale, nthreads: int = 0, out=None, new_state=None):
    q, k, v, state, A_log, a, dt_bias, b = map(_c, (q, k, v, state, A_log, a, dt_bias, b))
    B, _, Hq, _ = q.shape
    Hv = v.shape[2]
    if out is None:
        out = torch.empty_like(v)
    if new_state is None:
        new_state = torch.empty((B, Hv, 128, 128), dtype=torch.float32)
    lib().gdn_oracle_decode(_p(q), _p(k), _p(v), _p(state), _p(A_log), _p(a), _p(dt_bias), _p(b),
                            float(scale or 0.0), _p(out), _p(new_state), B, Hq, Hv, nthreads)
    return out, new_state


def prefill(q, k, v, state, A_log, a, dt_bias, b, cu_seqlens, scale, nthreads: int = 0):
    q, k, v, state, A_log, a, dt_bias, b = map(_c, (q, k, v, state, A_log, a, dt_bias, b))
    cu = cu_seqlens.detach().cpu().to(torch.int64).contiguous()
    T, Hq, _ = q.shape
    Hv = v.shape[1]
    N = cu.numel() - 1
    out = torch.zeros_like(v)
    new_state = torch.empty((N, Hv, 128, 128), dtype=torch.float32)
    lib().gdn_oracle_prefill(_p(q), _p(k), _p(v), _p(state), _p(A_log), _p(a), _p(dt_bias), _p(b),
                             _p(cu), N, float(scale or 0.0), _p(out), _p(new_state), Hq, Hv, nthreads)
    return out, new_state
