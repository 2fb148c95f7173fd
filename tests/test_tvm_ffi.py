"""The TVM-FFI module (gdn_b200/gdn_tvm_ffi.so): the binding the reference's
Solutions load with tvm_ffi.load_module.  CPU tests: the module loads, has every
export, and rejects bad tensors with the reference's exception kinds before any
launch.  GPU tests (-m gpu): decode and prefill through the module against the
oracle, and prep_meta_v2 against the oracle's metadata, bit for bit."""
import numpy as np
import pytest
import torch

import parity as PT
from oracle import c_oracle as C
from oracle import gdn_oracle as O
from gdn_b200 import tvm_ffi_module as TF, workloads as W


def test_module_loads_with_every_export():
    m = TF.load()
    for name in TF.EXPORTS:
        assert getattr(m, name) is not None, name


def test_workspace_bytes_matches_c_abi():
    from gdn_b200 import _native as N
    m = TF.load()
    for T, Nseq, Hq, Hv in [(65536, 4, 4, 8), (65536, 4, 16, 32), (100, 3, 4, 8), (8192, 1, 4, 8)]:
        assert m.gdn_prefill_workspace_bytes(T, Nseq, Hq, Hv) == \
            N.lib().gdn_prefill_workspace_bytes(T, Nseq, Hq, Hv)


def test_cpu_tensors_raise_value_error():
    m = TF.load()
    inp = W.make_decode_inputs(2, 4, 8, seed=1)
    out = torch.empty_like(inp.v)
    ns = torch.empty_like(inp.state)
    with pytest.raises(ValueError, match="CUDA tensor"):
        m.gdn_decode_small_batch(inp.q, inp.k, inp.v, inp.state, inp.A_log, inp.a, inp.dt_bias,
                                 inp.b, float(inp.scale), out, ns)


@pytest.mark.gpu
def test_decode_through_tvm_ffi():
    m = TF.load()
    cpu = W.make_decode_inputs(9, 4, 8, seed=31)
    o_ref, s_ref = O.decode(*PT.np_args(cpu))
    d = PT.to_device(cpu)
    out, ns = torch.empty_like(d.v), torch.empty_like(d.state)
    m.gdn_decode_small_batch(d.q, d.k, d.v, d.state, d.A_log, d.a, d.dt_bias, d.b, 0.0, out, ns)
    torch.cuda.synchronize()
    PT.assert_o_close(out, o_ref)
    PT.assert_state_close(ns, s_ref, PT.STATE_RTOL_FP32)
    # optional state: None = zero initial state
    z = W.make_decode_inputs(3, 16, 32, seed=32, with_state=False)
    zo_ref, zs_ref = O.decode(*PT.np_args(z))
    dz = PT.to_device(z)
    out, ns = torch.empty_like(dz.v), torch.empty((3, 32, 128, 128), device="cuda")
    m.gdn_decode(dz.q, dz.k, dz.v, None, dz.A_log, dz.a, dz.dt_bias, dz.b, 0.0, out, ns)
    torch.cuda.synchronize()
    PT.assert_o_close(out, zo_ref)
    PT.assert_state_close(ns, zs_ref, PT.STATE_RTOL_FP32)


@pytest.mark.gpu
@pytest.mark.parametrize("entry", ["gdn_prefill_recurrent_v1", "gdn_prefill_chunked", "gdn_prefill"])
def test_prefill_through_tvm_ffi(entry):
    m = TF.load()
    cpu = W.make_prefill_inputs([130, 1, 64, 700], 4, 8, seed=33)
    o_ref, s_ref = C.prefill(*cpu.args())
    d = PT.to_device(cpu)
    T, Nseq = d.q.shape[0], d.cu_seqlens.shape[0] - 1
    out = torch.empty_like(d.v)
    ns = torch.empty((Nseq, 8, 128, 128), device="cuda")
    args = [d.q, d.k, d.v, d.state, d.A_log, d.a, d.dt_bias, d.b, d.cu_seqlens, float(d.scale),
            out, ns]
    if entry == "gdn_prefill":
        args.append(None)  # no workspace
    getattr(m, entry)(*args)
    torch.cuda.synchronize()
    PT.assert_o_close(out, o_ref)
    PT.assert_state_close(ns, s_ref.numpy(),
                          PT.STATE_RTOL_FP32 if entry.endswith("_v1") else PT.STATE_REL)


@pytest.mark.gpu
def test_prefill_dtype_error_through_tvm_ffi():
    m = TF.load()
    d = PT.to_device(W.make_prefill_inputs([70], 4, 8, seed=34))
    out, ns = torch.empty_like(d.v), torch.empty((1, 8, 128, 128), device="cuda")
    with pytest.raises(TypeError, match="int64"):
        m.gdn_prefill(d.q, d.k, d.v, d.state, d.A_log, d.a, d.dt_bias, d.b,
                      d.cu_seqlens.to(torch.int32), 0.0, out, ns, None)


@pytest.mark.gpu
def test_prep_meta_v2_through_tvm_ffi():
    m = TF.load()
    lens = [1, 64, 65, 0, 300, 7]
    cu = torch.tensor(np.concatenate([[0], np.cumsum(lens)]), dtype=torch.int64)
    offs_ref, idx_ref = O.prep_meta(cu.numpy())
    Nseq = len(lens)
    ub = (Nseq - 1) + -(-(int(cu[-1]) - (Nseq - 1)) // 64)
    idx = torch.full((ub, 2), -7, dtype=torch.int32, device="cuda")
    offs = torch.empty(Nseq + 1, dtype=torch.int32, device="cuda")
    m.prep_meta_v2(cu.cuda(), idx, offs)
    torch.cuda.synchronize()
    assert offs.cpu().numpy().tolist() == list(offs_ref)
    n = int(offs_ref[-1])
    assert idx[:n].cpu().numpy().tolist() == np.asarray(idx_ref)[:n].tolist()
