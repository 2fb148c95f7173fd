"""The TVM-FFI module of the gdn_b200 kernels (gdn_b200/gdn_tvm_ffi.so).

The reference's Solutions bind their CUDA kernels as TVM-FFI typed functions and
call them with torch tensors (gdn_decode/solution/python/gdn_decode_small_batch.cu:194-232,
gdn_prefill/solution/python/cuda_recurrent_v1.cu:232-281, loaded by
``tvm_ffi.load_module``).  ``load()`` returns the same kind of module for these
kernels; its exports keep the reference's names and argument order where one
exists (``gdn_decode_small_batch``, ``gdn_prefill_recurrent_v1``,
``prep_meta_v2``) and add ``gdn_decode`` (optional state), ``gdn_prefill`` (the
dispatch, optional workspace), ``gdn_prefill_chunked`` and
``gdn_prefill_workspace_bytes``.  Outputs are caller-allocated; each call runs on
the tensors' current stream.  There is no fallback: a missing module raises.
"""
from __future__ import annotations

from pathlib import Path

MODULE_PATH = Path(__file__).resolve().with_name("gdn_tvm_ffi.so")
EXPORTS = ("gdn_decode_small_batch", "gdn_decode", "gdn_prefill_recurrent_v1", "gdn_prefill",
           "gdn_prefill_chunked", "prep_meta_v2", "gdn_prefill_workspace_bytes")
_mod = None


def load():
    """Load (once) and return the TVM-FFI module."""
    global _mod
    if _mod is None:
        if not MODULE_PATH.exists():
            raise RuntimeError(f"TVM-FFI module not found at {MODULE_PATH}; build it with "
                               "`python mlsys-flashlinfer-contest_b200/build.py`")
        import tvm_ffi
        _mod = tvm_ffi.load_module(str(MODULE_PATH))
    return _mod
