"""ctypes binding of libgdn_b200.so, the C ABI declared in include/gdn_b200.h.

The library is built in-tree by ``mlsys-flashlinfer-contest_b200/build.py``.  There
is no fallback: if the library is missing or fails to load, every entry point
raises, so a run can never silently fall back to a CPU or library path.
"""
from __future__ import annotations

import ctypes
from pathlib import Path

LIB_PATH = Path(__file__).resolve().with_name("libgdn_b200.so")
ABI_VERSION = 1

GDN_OK, GDN_ERR_VALUE, GDN_ERR_TYPE, GDN_ERR_CUDA = 0, 1, 2, 3
_EXC = {GDN_ERR_VALUE: ValueError, GDN_ERR_TYPE: TypeError, GDN_ERR_CUDA: RuntimeError}

# (name, restype, argtypes) for every symbol include/gdn_b200.h declares
P, I64, F, SZ, I = ctypes.c_void_p, ctypes.c_int64, ctypes.c_float, ctypes.c_size_t, ctypes.c_int
SIGNATURES = {
    "gdn_abi_version": (I, []),
    "gdn_last_error": (ctypes.c_char_p, []),
    "gdn_decode": (I, [P, P, P, P, P, P, P, P, F, P, P, I64, I64, I64, I64, I64, P]),
    "gdn_decode_pool": (I, [P, P, P, P, P, P, P, F, P, I, I64, P, P, P, I, P, I64, I64, I64, I64,
                            I64, I64, P]),
    "gdn_prefill": (I, [P, P, P, P, P, P, P, P, P, F, P, P, I64, I64, I64, I64, I64, I64, P, SZ, P]),
    "gdn_prefill_workspace_bytes": (SZ, [I64, I64, I64, I64]),
    "gdn_prefill_ex": (I, [P, P, P, P, P, P, P, P, P, F, P, P, I64, I64, I64, I64, I64, I64, I, I, P]),
    "gdn_prefill_recurrent": (I, [P, P, P, P, P, P, P, P, P, F, P, P, I64, I64, I64, I64, I64, I64, P]),
    "gdn_prep_meta": (I, [P, I64, P, P, I64, P]),
    "gdn_chunk_upper_bound": (I64, [I64, I64]),
    "gdn_prefill_chunked": (I, [P, P, P, P, P, P, P, P, P, F, P, P, I64, I64, I64, I64, I64, I64, P]),
    "gdn_prefill_chunked_peers": (I, [P, P, P, P, P, P, P, P, P, F, P, P, I64, I64, I64, I64, I64,
                                      I64, I64, I64, P, I, I, P, SZ, P]),
    "gdn_prefill_segmented": (I, [P, P, P, P, P, P, P, P, P, F, P, P, I64, I64, I64, I64, I64, I64,
                                  I, I, P, SZ, P]),
    "gdn_prefill_segmented_workspace_bytes": (SZ, [I64, I64, I]),
    "gdn_prefill_segmented_noalloc": (I, [P, P, P, P, P, P, P, P, P, F, P, P, I64, I64, I64, I64, I64,
                                          I64, I, I, P]),
    "gdn_prefill_segments": (I, [I64, I64, I64]),
    "gdn_prefill_chunked_debug": (I, [P, P, P, P, P, P, P, P, P, F, P, P, I64, I64, I64, I64, I64,
                                      I64, P, I64, I64, I64, I64, P]),
    "gdn_prefill_chunked_debug_floats": (I64, []),
    "gdn_read_status": (I, [P, I]),
    "gdn_wait_probe": (I, [ctypes.c_uint64, P, P]),
}

_lib = None


def lib():
    """Load (once) and return the library, with argtypes set."""
    global _lib
    if _lib is not None:
        return _lib
    if not LIB_PATH.exists():
        raise RuntimeError(
            f"gdn_b200 CUDA library not found at {LIB_PATH}; build it with "
            "`python mlsys-flashlinfer-contest_b200/build.py` (there is no CPU fallback)")
    L = ctypes.CDLL(str(LIB_PATH))
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(L, name)
        fn.restype = res
        fn.argtypes = args
    if L.gdn_abi_version() != ABI_VERSION:
        raise RuntimeError(f"libgdn_b200.so ABI {L.gdn_abi_version()} != expected {ABI_VERSION}")
    _lib = L
    return L


_ext = False


def torch_ext():
    """The torch-tensor binding (gdn_b200/_gdn_torch.so, built from
    csrc/gdn_torch.cpp), or None when it was not built: the entry points then
    make the same C-ABI calls through ctypes (same kernels, more host time)."""
    global _ext
    if _ext is False:
        lib()  # the binding links libgdn_b200.so; load and version-check it first
        try:
            from . import _gdn_torch as ext
        except ImportError:
            ext = None
        _ext = ext
    return _ext


def check(rc: int, what: str = "") -> None:
    if rc == GDN_OK:
        return
    msg = lib().gdn_last_error().decode(errors="replace")
    raise _EXC.get(rc, RuntimeError)(f"{what}: {msg}" if what else msg)


def ptr(t) -> ctypes.c_void_p:
    return ctypes.c_void_p(0 if t is None else t.data_ptr())


def stream_handle(device) -> ctypes.c_void_p:
    import torch
    return ctypes.c_void_p(torch.cuda.current_stream(device).cuda_stream)
