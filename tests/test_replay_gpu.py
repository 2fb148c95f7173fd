"""Contest-shape replay on the GPU: the public ``run`` entry points over seeded
synthetic shapes that span the contest workloads' axes (qk4_v8 geometry: Hq = Hk = 4,
Hv = 8; decode batch 1..64; prefill 6..8192 tokens over 1..57 sequences), each
checked against the C restatement of the reference definitions with the contract
tolerances (bf16 outputs atol = rtol = 1e-2, fp32 final state within 1e-3)."""
import pytest
import torch

import parity as PT
from oracle import c_oracle as C
from gdn_b200 import decode, prefill, workloads as W

pytestmark = pytest.mark.gpu

HQ, HV = W.CONTEST_HQ, W.CONTEST_HV
PREFILL_CASES = W.contest_prefill_cases()


@pytest.mark.parametrize("B", W.CONTEST_DECODE_BATCHES)
def test_replay_decode(B):
    inp = W.make_decode_inputs(B, HQ, HV, seed=500 + B)
    o_ref, s_ref = C.decode(*inp.args())
    o, ns = decode.run(*PT.to_device(inp).args())
    torch.cuda.synchronize()
    PT.assert_o_close(o, o_ref)
    PT.assert_state_close(ns, s_ref, PT.STATE_RTOL_FP32)


@pytest.mark.parametrize("i", range(len(PREFILL_CASES)))
def test_replay_prefill(i):
    lengths = PREFILL_CASES[i]
    inp = W.make_prefill_inputs(lengths, HQ, HV, seed=700 + i, zero_state_every_other=(i % 2 == 1))
    o_ref, s_ref = C.prefill(*inp.args())
    o, ns = prefill.run(*PT.to_device(inp).args())
    torch.cuda.synchronize()
    PT.assert_o_close(o, o_ref)
    PT.assert_state_close(ns, s_ref, PT.STATE_REL)
