"""GPU parity of the fused decode kernel against the CPU oracle and the golden
fixtures (reference outputs).  Every call goes through the C ABI."""
import numpy as np
import pytest
import torch

import golden_io as G
import parity as PT
from oracle import gdn_oracle as O
from gdn_b200 import decode, workloads as W

pytestmark = pytest.mark.gpu


def _check(inp, rel=PT.STATE_RTOL_FP32):
    o_ref, s_ref = O.decode(*PT.np_args(inp))
    dev = PT.to_device(inp)
    o, ns = decode.run(*dev.args())
    torch.cuda.synchronize()
    PT.assert_o_close(o, o_ref)
    PT.assert_state_close(ns, s_ref, rel)
    return o, ns


@pytest.mark.parametrize("name", G.names("decode"))
def test_decode_matches_reference_golden(name):
    meta, z = G.load(name)
    inp = G.regenerate_inputs(meta)
    assert G.sha_inputs(list(inp.args())) == str(z["input_sha"])
    o, ns = decode.run(*PT.to_device(inp).args())
    PT.assert_o_close(o, z["o"])
    G.check_state(O.to_numpy(ns), z, rtol=1e-4, atol=1e-5, sum_rtol=1e-5)


def test_decode_config0():
    # B=4, Hq=16, Hv=32
    _check(W.make_decode_inputs(4, 16, 32, seed=0))


@pytest.mark.parametrize("B", [1, 2, 3, 7, 8, 16, 33, 64])
@pytest.mark.parametrize("geom", [(4, 8), (16, 32)])
def test_decode_batch_sweep(B, geom):
    _check(W.make_decode_inputs(B, geom[0], geom[1], seed=B * 7 + geom[0]))


def test_decode_gva_ratio_4():
    _check(W.make_decode_inputs(5, 2, 8, seed=3))


def test_decode_state_none():
    inp = W.make_decode_inputs(6, 4, 8, seed=4, with_state=False)
    _check(inp)


def test_decode_scale_zero_means_default():
    inp = W.make_decode_inputs(2, 4, 8, seed=5)
    inp.scale = 0.0
    o0, s0 = decode.run(*PT.to_device(inp).args())
    inp.scale = 1.0 / np.sqrt(128.0)
    o1, s1 = decode.run(*inp.args())
    assert torch.equal(o0, o1) and torch.equal(s0, s1)


def test_decode_inplace_matches_out_of_place():
    inp = PT.to_device(W.make_decode_inputs(9, 16, 32, seed=6))
    o1, s1 = decode.run(*inp.args())
    st = inp.state.clone()
    args = list(inp.args())
    args[3] = st
    o2, s2 = decode.run_inplace(*args)
    assert s2.data_ptr() == st.data_ptr()
    assert torch.equal(o1, o2) and torch.equal(s1, s2)


def test_decode_deterministic():
    inp = PT.to_device(W.make_decode_inputs(3, 16, 32, seed=8))
    o1, s1 = decode.run(*inp.args())
    o2, s2 = decode.run(*inp.args())
    assert torch.equal(o1, o2) and torch.equal(s1, s2)


def test_decode_large_batch_all_sequences():
    """BASELINE config 1 (B=256, Hq=16, Hv=32): every one of the 256 x 32
    (sequence, v-head) updates against the C oracle (the reference decode
    recurrence on all host threads)."""
    from oracle import c_oracle as C
    cpu = W.make_decode_inputs(256, 16, 32, seed=11)
    o_ref, s_ref = C.decode(*cpu.args())
    inp = PT.to_device(cpu)
    o, ns = decode.run(*inp.args())
    torch.cuda.synchronize()
    PT.assert_o_close(o, o_ref)
    ns = ns.cpu()
    for b0 in range(0, 256, 32):  # 32 sequences at a time keeps the float64 copies small
        PT.assert_state_close(ns[b0:b0 + 32], s_ref[b0:b0 + 32].numpy(), PT.STATE_RTOL_FP32)


def test_decode_dtype_and_shape_errors():
    inp = PT.to_device(W.make_decode_inputs(2, 4, 8, seed=1))
    args = list(inp.args())
    bad = list(args)
    bad[0] = args[0].float()
    with pytest.raises(TypeError):
        decode.run(*bad)
    bad = list(args)
    bad[4] = args[4][:4].contiguous()
    with pytest.raises(ValueError):
        decode.run(*bad)
    bad = list(args)
    bad[0] = args[0].expand(2, 2, 4, 128)
    with pytest.raises(ValueError):
        decode.run(*bad)
