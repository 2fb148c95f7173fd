"""Decode steps replayed from CUDA graphs (gdn_b200.graphs.DecodeGraph) equal eager
steps bit for bit, in the ping-pong and the in-place forms, with fresh inputs
written into the captured buffers every step."""
import pytest
import torch

from gdn_b200 import decode, graphs, workloads as W

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("inplace", [False, True])
@pytest.mark.parametrize("B", [1, 37])
def test_decode_graph_matches_eager(B, inplace):
    steps = [W.make_decode_inputs(B, 4, 8, seed=100 + i, device="cuda") for i in range(4)]
    first = steps[0]
    st_eager = first.state.clone()
    g = graphs.DecodeGraph(first.q.clone(), first.k.clone(), first.v.clone(), first.state.clone(),
                           first.A_log, first.a.clone(), first.dt_bias, first.b.clone(), first.scale,
                           inplace=inplace)
    for inp in steps:
        for name in ("q", "k", "v", "a", "b"):
            getattr(g, name).copy_(getattr(inp, name))
        o_g = g.step()
        o_e, st_eager = decode.run(inp.q, inp.k, inp.v, st_eager, first.A_log, inp.a, first.dt_bias,
                                   inp.b, first.scale)
        torch.cuda.synchronize()
        assert torch.equal(o_g, o_e)
        assert torch.equal(g.state, st_eager)
