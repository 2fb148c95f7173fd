"""Contest-record replay on the GPU: the public ``run`` entry points on every
workload record of the reference's workloads/gdn/*.md (qk4_v8 geometry: Hq = Hk =
4, Hv = 8), with seeded synthetic tensors of each record's shape: the 54 decode
records (batch_size) and the 100 prefill records (total_seq_len, num_seqs), each
prefill record under both of the reference's cu_seqlens rewrites, "even" and
"uneven" (gdn_prefill/scripts/run_local_fast_{even,uneven}.py).  Every case is
checked against the C restatement of the reference definitions with the contract
tolerances (bf16 outputs atol = rtol = 1e-2, fp32 final state within 1e-3)."""
import pytest
import torch

import parity as PT
from oracle import c_oracle as C
from gdn_b200 import decode, prefill, workloads as W

pytestmark = pytest.mark.gpu

HQ, HV = W.CONTEST_HQ, W.CONTEST_HV
DECODE_RECORDS = W.contest_decode_records()
PREFILL_RECORDS = W.contest_prefill_records()


def test_record_counts():
    assert len(DECODE_RECORDS) == 54 and len(PREFILL_RECORDS) == 200


@pytest.mark.parametrize("i", range(len(DECODE_RECORDS)))
def test_replay_decode_record(i):
    B = DECODE_RECORDS[i]
    inp = W.make_decode_inputs(B, HQ, HV, seed=500 + i)
    o_ref, s_ref = C.decode(*inp.args())
    o, ns = decode.run(*PT.to_device(inp).args())
    torch.cuda.synchronize()
    PT.assert_o_close(o, o_ref)
    PT.assert_state_close(ns, s_ref, PT.STATE_RTOL_FP32)


@pytest.mark.parametrize("j", range(len(PREFILL_RECORDS)))
def test_replay_prefill_record(j):
    rec, split, lengths = PREFILL_RECORDS[j]
    inp = W.make_prefill_inputs(lengths, HQ, HV, seed=700 + j, zero_state_every_other=(j % 4 == 1))
    o_ref, s_ref = C.prefill(*inp.args())
    o, ns = prefill.run(*PT.to_device(inp).args())
    torch.cuda.synchronize()
    PT.assert_o_close(o, o_ref)
    PT.assert_state_close(ns, s_ref, PT.STATE_REL)
