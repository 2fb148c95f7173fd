"""In-kernel q/k L2 normalisation of the prefill kernels (C ABI gdn_prefill_ex,
GDN_PREFILL_QK_L2NORM): un-normalised q, k against the oracle that normalises them
in fp32 first (x / sqrt(sum x^2 + 1e-6)) and then runs the definition's recurrence.
The chunked kernel folds 1/|k_t| and 1/|q_t| into per-token factors (A/P rows and
columns, K S columns, Vd rows, the output's Q S columns)."""
import pytest
import torch

import parity as PT
from oracle import gdn_oracle as O
from gdn_b200 import prefill, workloads as W

pytestmark = pytest.mark.gpu

CASES = [[1, 2], [65], [130, 0, 7], [200, 64, 1], [300]]
PATHS = {"recurrent": (prefill.run_recurrent, PT.STATE_RTOL_FP32),
         "chunked": (prefill.run_chunked, PT.STATE_REL),
         "auto": (prefill.run, PT.STATE_REL)}


@pytest.mark.parametrize("lengths", CASES)
@pytest.mark.parametrize("path", list(PATHS))
@pytest.mark.parametrize("geom", [(4, 8), (16, 32)])
def test_prefill_qk_l2norm(lengths, path, geom):
    inp = W.make_prefill_inputs(lengths, geom[0], geom[1], seed=sum(lengths) + len(path),
                                normalized_qk=False, zero_state_every_other=True)
    o_ref, s_ref = O.prefill(*PT.np_args(inp), qk_l2norm=True)
    fn, rel = PATHS[path]
    o, ns = fn(*PT.to_device(inp).args(), use_qk_l2norm=True)
    torch.cuda.synchronize()
    PT.assert_o_close(o, o_ref)
    PT.assert_state_close(ns, s_ref, rel)


def test_l2norm_of_normalised_inputs_changes_little():
    """Inputs already L2-normalised (then rounded to bf16): the option only
    re-normalises away the bf16 rounding of the norms."""
    inp = PT.to_device(W.make_prefill_inputs([200, 64], 4, 8, seed=3))
    o0, s0 = prefill.run_chunked(*inp.args())
    o1, s1 = prefill.run_chunked(*inp.args(), use_qk_l2norm=True)
    torch.cuda.synchronize()
    PT.assert_o_close(o1, o0)
    PT.assert_state_close(s1, O.to_numpy(s0), 1e-2)
