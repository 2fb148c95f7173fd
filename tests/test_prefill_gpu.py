"""GPU parity of the prefill kernels (token-recurrent path and the default
dispatch) and of the device chunk metadata, against the CPU oracle and the
golden fixtures."""
import numpy as np
import pytest
import torch

import golden_io as G
import parity as PT
from oracle import gdn_oracle as O
from gdn_b200 import _native as N, prefill, workloads as W

pytestmark = pytest.mark.gpu

CASES = [
    [1], [2, 3], [63], [64], [65], [130, 0, 7], [200, 64, 1], [0, 5], [129, 128, 127],
]


def _check(inp, fn, rel):
    o_ref, s_ref = O.prefill(*PT.np_args(inp))
    o, ns = fn(*PT.to_device(inp).args())
    torch.cuda.synchronize()
    PT.assert_o_close(o, o_ref)
    return PT.assert_state_close(ns, s_ref, rel)


@pytest.mark.parametrize("name", G.names("prefill"))
@pytest.mark.parametrize("path", ["recurrent", "default"])
def test_prefill_matches_reference_golden(name, path):
    meta, z = G.load(name)
    inp = G.regenerate_inputs(meta)
    assert G.sha_inputs(list(inp.args())) == str(z["input_sha"])
    fn = prefill.run_recurrent if path == "recurrent" else prefill.run
    o, ns = fn(*PT.to_device(inp).args())
    PT.assert_o_close(o, z["o"])
    tol = 1e-4 if path == "recurrent" else 2e-3
    G.check_state(O.to_numpy(ns), z, rtol=tol, atol=tol * 0.1, sum_rtol=tol)


@pytest.mark.parametrize("lengths", CASES)
@pytest.mark.parametrize("geom", [(4, 8), (16, 32)])
def test_prefill_recurrent_parity(lengths, geom):
    inp = W.make_prefill_inputs(lengths, geom[0], geom[1], seed=len(lengths) * 31 + sum(lengths))
    _check(inp, prefill.run_recurrent, PT.STATE_RTOL_FP32)


@pytest.mark.parametrize("lengths", CASES)
def test_prefill_default_parity(lengths):
    inp = W.make_prefill_inputs(lengths, 4, 8, seed=sum(lengths) + 5,
                                zero_state_every_other=True)
    _check(inp, prefill.run, PT.STATE_REL)


def test_prefill_state_none():
    inp = W.make_prefill_inputs([70, 9], 4, 8, seed=12, with_state=False)
    _check(inp, prefill.run, PT.STATE_REL)
    _check(inp, prefill.run_recurrent, PT.STATE_RTOL_FP32)


def test_prefill_int32_cu_seqlens():
    inp = W.make_prefill_inputs([33, 40], 4, 8, seed=13)
    inp32 = W.make_prefill_inputs([33, 40], 4, 8, seed=13, cu_dtype=torch.int32)
    o1, s1 = prefill.run(*PT.to_device(inp).args())
    o2, s2 = prefill.run(*PT.to_device(inp32).args())
    assert torch.equal(o1, o2) and torch.equal(s1, s2)


def test_prefill_even_and_uneven_generators():
    # the reference's load-balance rewrites (run_local_fast_even/uneven.py)
    for lens in (W.even_lengths(300, 4), W.uneven_lengths(300, 4)):
        inp = W.make_prefill_inputs(lens, 4, 8, seed=sum(lens))
        _check(inp, prefill.run, PT.STATE_REL)


@pytest.mark.parametrize("lengths", [[0], [1], [64, 64], [65, 0, 0, 300], [5] * 300,
                                     [0] * 7 + [129], list(range(0, 2000, 3))])
def test_prep_meta_bit_exact(lengths):
    cu = np.concatenate([[0], np.cumsum(lengths)]).astype(np.int64)
    T, Nseq = int(cu[-1]), len(lengths)
    off_ref, idx_ref = O.prep_meta(cu)
    ub = max(O.chunk_upper_bound(T, Nseq), 1)
    cu_d = torch.from_numpy(cu).cuda()
    off = torch.full((Nseq + 1,), -7, dtype=torch.int32, device="cuda")
    idx = torch.full((ub, 2), -7, dtype=torch.int32, device="cuda")
    L = N.lib()
    rc = L.gdn_prep_meta(N.ptr(cu_d), Nseq, N.ptr(off), N.ptr(idx), ub, N.stream_handle(cu_d.device))
    N.check(rc)
    torch.cuda.synchronize()
    assert off.cpu().numpy().tolist() == off_ref.tolist()
    total = int(off_ref[-1])
    assert idx[:total].cpu().numpy().tolist() == idx_ref.tolist()
