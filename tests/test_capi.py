"""CPU tests of the C ABI: the library loads, exports every function
include/gdn_b200.h declares, and rejects bad arguments with the documented
error codes before touching the GPU."""
import ctypes
import re

import pytest
import torch

from conftest import REPO
from gdn_b200 import _native as N


def header_functions():
    text = (REPO / "include" / "gdn_b200.h").read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(gdn_[a-z0-9_]+)\s*\(", text)))


def test_header_matches_binding_table():
    assert header_functions() == sorted(N.SIGNATURES), "binding table out of sync with the header"


def test_library_exports_every_declared_symbol():
    L = N.lib()
    for name in header_functions():
        assert hasattr(L, name), name
    assert L.gdn_abi_version() == N.ABI_VERSION


def test_chunk_upper_bound():
    L = N.lib()
    assert L.gdn_chunk_upper_bound(1000, 5) == 20
    assert L.gdn_chunk_upper_bound(64, 1) == 1
    assert L.gdn_chunk_upper_bound(65, 1) == 2
    assert L.gdn_chunk_upper_bound(3, 8) == 3
    assert L.gdn_chunk_upper_bound(0, 4) == 0


def _decode_call(**over):
    args = dict(q=1 << 20, k=1 << 20, v=1 << 20, state=1 << 20, A_log=1 << 20, a=1 << 20,
                dt_bias=1 << 20, b=1 << 20, scale=0.0, out=1 << 20, new_state=1 << 21, B=1, Hq=4,
                Hk=4, Hv=8, D=128)
    args.update(over)
    L = N.lib()
    P = ctypes.c_void_p
    return L.gdn_decode(P(args["q"]), P(args["k"]), P(args["v"]), P(args["state"]),
                        P(args["A_log"]), P(args["a"]), P(args["dt_bias"]), P(args["b"]),
                        args["scale"], P(args["out"]), P(args["new_state"]), args["B"], args["Hq"],
                        args["Hk"], args["Hv"], args["D"], None)


@pytest.mark.parametrize("over,msg", [
    (dict(D=64), "head_size"),
    (dict(Hk=2), "num_k_heads"),
    (dict(Hv=6), "multiple"),
    (dict(B=-1), "non-negative"),
    (dict(q=0), "null"),
    (dict(q=(1 << 20) + 2), "aligned"),
    (dict(state=(1 << 20) + 4), "aligned"),
    (dict(state=1 << 21, new_state=(1 << 21) + 4096), "overlaps"),
])
def test_decode_validation_errors(over, msg):
    rc = _decode_call(**over)
    assert rc == N.GDN_ERR_VALUE
    assert msg in N.lib().gdn_last_error().decode()


def test_decode_zero_batch_is_a_noop():
    assert _decode_call(B=0, q=0, k=0) == N.GDN_OK


def test_prefill_needs_a_sequence():
    L = N.lib()
    P = ctypes.c_void_p
    rc = L.gdn_prefill(P(1 << 20), P(1 << 20), P(1 << 20), None, P(1 << 20), P(1 << 20),
                       P(1 << 20), P(1 << 20), P(1 << 20), 0.0, P(1 << 20), P(1 << 21), 10, 0,
                       4, 4, 8, 128, None, 0, None)
    assert rc == N.GDN_ERR_VALUE and b"at least one sequence" in L.gdn_last_error()


def test_python_entry_points_reject_cpu_tensors():
    from gdn_b200 import decode, prefill, workloads as W
    inp = W.make_decode_inputs(1, 4, 8, seed=0)
    with pytest.raises(ValueError, match="CUDA"):
        decode.run(*inp.args())
    pin = W.make_prefill_inputs([5], 4, 8, seed=0)
    with pytest.raises(ValueError, match="CUDA"):
        prefill.run(*pin.args())


def test_check_maps_codes_to_exceptions():
    with pytest.raises(ValueError):
        N.check(N.GDN_ERR_VALUE)
    with pytest.raises(TypeError):
        N.check(N.GDN_ERR_TYPE)
    with pytest.raises(RuntimeError):
        N.check(N.GDN_ERR_CUDA)
