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


def _peers_call(Hv_out=16, off=0, npeers=1, peers=(1 << 22,), out=1 << 20):
    L = N.lib()
    P = ctypes.c_void_p
    arr = (ctypes.c_void_p * max(len(peers), 1))(*peers)
    return L.gdn_prefill_chunked_peers(P(1 << 20), P(1 << 20), P(1 << 20), None, P(1 << 20),
                                       P(1 << 20), P(1 << 20), P(1 << 20), P(1 << 20), 0.0, P(out),
                                       P(1 << 21), 10, 1, 4, 4, 8, 128, Hv_out, off,
                                       ctypes.cast(arr, ctypes.c_void_p), npeers, 1, None, 0, None)


@pytest.mark.parametrize("over,msg", [
    (dict(npeers=8, peers=(1 << 22,) * 8), "num_peers"),
    (dict(off=9), "must lie in the output"),
    (dict(Hv_out=4), "must lie in the output"),
    (dict(peers=((1 << 22) + 2,)), "peer output 0"),
    (dict(peers=(0,)), "peer output 0"),
    (dict(out=(1 << 20) + 8), "16-byte aligned"),
])
def test_prefill_peers_validation_errors(over, msg):
    """The fused-gather prefill entry rejects bad routing before touching the GPU."""
    rc = _peers_call(**over)
    assert rc == N.GDN_ERR_VALUE
    assert msg in N.lib().gdn_last_error().decode()


def test_decode_pool_validation_errors():
    L = N.lib()
    P = ctypes.c_void_p
    base = [P(1 << 20)] * 7 + [0.0, P(1 << 21), 1, 4, P(1 << 22), None, None, 0, P(1 << 23),
                               2, 1, 4, 4, 8, 128, None]
    def call(**kw):
        a = list(base)
        for i, v in kw.items():
            a[int(i[1:])] = v
        return L.gdn_decode_pool(*a)
    assert call(a9=7) == N.GDN_ERR_TYPE                      # state dtype
    assert call(a17=0) == N.GDN_ERR_VALUE                    # seq_len 0
    assert call(a14=4) == N.GDN_ERR_VALUE                    # unknown flag
    assert call(a0=P((1 << 20) + 8)) == N.GDN_ERR_VALUE      # q alignment


def test_prefill_segment_choice():
    """Upper bound of the automatic piece count (148 SMs without a GPU; the device
    picks each sequence's count under it): a head shard of config 3 may be cut,
    the full 32-head call (more pairs than half the SMs) is not."""
    L = N.lib()
    assert L.gdn_prefill_segments(65536, 4, 32) == 1     # 128 pairs
    assert L.gdn_prefill_segments(65536, 4, 16) == 5     # 64 pairs: 64 x 4 <= 2 x 148
    assert L.gdn_prefill_segments(65536, 4, 8) == 10
    assert L.gdn_prefill_segments(65536, 4, 4) == 16
    assert L.gdn_prefill_segments(8192, 1, 8) == 16
    assert L.gdn_prefill_segments(4096, 1, 8) == 16      # 64 chunks = 4 x 16
    assert L.gdn_prefill_segments(700, 1, 8) == 1        # 10 chunks: fewer than 4 x 3
    # fewer chunks in all than the shortest sequence the job builder would cut (23)
    assert L.gdn_prefill_segments(1408, 1, 8) == 1       # 22 chunks
    assert L.gdn_prefill_segments(1472, 1, 8) == 5       # 23 chunks; 4 G <= 23
    assert L.gdn_prefill_segments(16, 1, 8) == 1         # the recurrent kernel's size
    assert L.gdn_prefill_workspace_bytes(65536, 4, 16, 32) == 0
    ws = L.gdn_prefill_workspace_bytes(65536, 4, 4, 4)
    assert ws == L.gdn_prefill_segmented_workspace_bytes(4, 4, 0)
    # the automatic form's state pool: 1.5 x 148 / Hv states of Hv x 64 KiB (the
    # device keeps every cut within it): 55 states for this shard
    assert 4 * 65536 * 55 <= ws < (16 << 20)
    # a forced count: N (2G - 3) states (start state of piece 1, F and P of the
    # middle pieces; the combine writes the later start states over F)
    assert L.gdn_prefill_segmented_workspace_bytes(4, 4, 6) >= 4 * 4 * 65536 * 9
    assert L.gdn_prefill_segmented_workspace_bytes(4, 4, 1) == 0


def test_prefill_segmented_validation_errors():
    L = N.lib()
    P = ctypes.c_void_p
    def call(segments, ws, ws_bytes, flags=0):
        return L.gdn_prefill_segmented(P(1 << 20), P(1 << 20), P(1 << 20), None, P(1 << 20),
                                       P(1 << 20), P(1 << 20), P(1 << 20), P(1 << 20), 0.0,
                                       P(1 << 20), P(1 << 21), 8192, 1, 4, 4, 8, 128, flags,
                                       segments, ws, ws_bytes, None)
    assert call(65, None, 0) == N.GDN_ERR_VALUE
    assert "segments" in L.gdn_last_error().decode()
    assert call(3, None, 0) == N.GDN_ERR_VALUE
    assert "workspace" in L.gdn_last_error().decode()
    assert call(3, P((1 << 24) + 16), 1 << 30) == N.GDN_ERR_VALUE
    assert "256-byte" in L.gdn_last_error().decode()
    assert call(3, P(1 << 24), 1 << 30, flags=8) == N.GDN_ERR_VALUE
    assert "flags" in L.gdn_last_error().decode()
