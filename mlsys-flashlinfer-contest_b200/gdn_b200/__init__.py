"""gdn_b200: B200-native (sm_100a) Gated DeltaNet decode and prefill.

Entry points with the reference solution signatures:
  gdn_b200.decode.run(q, k, v, state, A_log, a, dt_bias, b, scale)
  gdn_b200.prefill.run(q, k, v, state, A_log, a, dt_bias, b, cu_seqlens, scale)
Both return (output, new_state) and call hand-written CUDA kernels through the
C ABI of libgdn_b200.so (include/gdn_b200.h).
"""
from . import decode, prefill, workloads  # noqa: F401
from ._native import LIB_PATH, lib  # noqa: F401

__all__ = ["decode", "prefill", "workloads", "lib", "LIB_PATH"]
