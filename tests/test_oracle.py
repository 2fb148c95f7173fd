"""CPU tests: pin the oracle to the reference's own outputs (golden fixtures),
check the chunked restatement and the metadata against the recurrence, and
cross-check the C restatement against the numpy one."""
import numpy as np
import pytest
import torch

import golden_io as G
from oracle import gdn_oracle as O
from oracle import c_oracle as C
from gdn_b200 import workloads as W


def _np_args(inp):
    return [O.to_numpy(x) if isinstance(x, torch.Tensor) else x for x in inp.args()]


def _o_close(o_bits, ref_bits):
    """bf16 outputs: equal bits almost everywhere, never more than 1 ulp apart in
    value terms (float32 accumulation order differs from torch's)."""
    a = O.bf16_to_f32(o_bits).astype(np.float64)
    r = O.bf16_to_f32(ref_bits).astype(np.float64)
    tol = np.abs(r) * 2.0 ** -7 + 1e-6  # one bf16 ulp
    assert np.all(np.abs(a - r) <= tol), float(np.abs(a - r).max())
    assert np.mean(o_bits != ref_bits) < 0.02


@pytest.mark.parametrize("name", G.names())
def test_oracle_matches_reference_golden(name):
    meta, z = G.load(name)
    inp = G.regenerate_inputs(meta)
    assert G.sha_inputs(list(inp.args())) == str(z["input_sha"]), "input generator drifted"
    args = _np_args(inp)
    if meta["kind"] == "decode":
        o, ns = O.decode(*args)
    else:
        o, ns = O.prefill(*args)
    _o_close(o, z["o"])
    G.check_state(ns, z)


@pytest.mark.parametrize("name", G.names())
def test_c_oracle_matches_reference_golden(name):
    meta, z = G.load(name)
    inp = G.regenerate_inputs(meta)
    if meta["kind"] == "decode":
        o, ns = C.decode(*inp.args(), nthreads=4)
    else:
        o, ns = C.prefill(*inp.args(), nthreads=4)
    _o_close(o.view(torch.int16).numpy().view(np.uint16), z["o"])
    G.check_state(ns.numpy(), z)


def test_prep_meta_known_answer():
    # Report.pdf p.5 App. A: N=2 sequences with 3 and 5 chunks -> offsets [0, 3, 8]
    off, idx = O.prep_meta([0, 150, 150 + 300])
    assert off.tolist() == [0, 3, 8]
    assert idx.tolist() == [[0, 0], [0, 1], [0, 2], [1, 0], [1, 1], [1, 2], [1, 3], [1, 4]]


def test_prep_meta_edges():
    off, idx = O.prep_meta([0, 0, 64, 65, 65, 200])
    assert off.tolist() == [0, 0, 1, 2, 2, 5]
    assert idx.tolist() == [[1, 0], [2, 0], [4, 0], [4, 1], [4, 2]]


def test_chunk_upper_bound_is_tight():
    rng = np.random.default_rng(0)
    for _ in range(300):
        N = int(rng.integers(1, 9))
        lens = rng.integers(0, 200, N)
        T = int(lens.sum())
        off, _ = O.prep_meta(np.concatenate([[0], np.cumsum(lens)]))
        assert off[-1] <= O.chunk_upper_bound(T, N)
    # tight for N-1 sequences of one token plus one long sequence
    for T, N in [(1000, 5), (64, 1), (65, 1), (7, 7), (130, 2)]:
        lens = W.uneven_lengths(T, N)
        off, _ = O.prep_meta(np.concatenate([[0], np.cumsum(lens)]))
        assert off[-1] == O.chunk_upper_bound(T, N)


def test_inverse_known_answer():
    # gdn_prefill/doc/newton-schulz-refinement.md:14-24
    M = np.array([[1, 0, 0], [0.5, 1, 0], [0.3, 0.4, 1]])
    np.testing.assert_allclose(np.linalg.inv(M), [[1, 0, 0], [-0.5, 1, 0], [-0.1, -0.4, 1]],
                               atol=1e-12)


@pytest.mark.parametrize("lengths", [[1], [63], [64], [65], [130, 0, 7], [200, 64]])
def test_chunked_matches_recurrence(lengths):
    inp = W.make_prefill_inputs(lengths, 2, 4, seed=sum(lengths) + len(lengths))
    args = _np_args(inp)
    o_ref, s_ref = O.prefill(*args)
    o, s = O.chunked_prefill(*args)
    assert O.rel_err(s, s_ref) < 1e-5
    assert O.rel_err(o, O.bf16_to_f32(o_ref)) < 5e-3  # the oracle rounds o to bf16
    assert O.rel_err(O.round_bf16(o), O.bf16_to_f32(o_ref)) < 5e-3


def test_state_none_equals_zero_state():
    inp = W.make_prefill_inputs([40, 3], 2, 4, seed=7, with_state=True)
    args = _np_args(inp)
    args[3] = np.zeros_like(args[3])
    o1, s1 = O.prefill(*args)
    args[3] = None
    o2, s2 = O.prefill(*args)
    assert np.array_equal(o1, o2) and np.array_equal(s1, s2)


def test_empty_sequence_gets_zero_state():
    inp = W.make_prefill_inputs([5, 0, 4], 2, 4, seed=9)
    o, s = O.prefill(*_np_args(inp))
    assert np.all(s[1] == 0)
    o2, s2 = C.prefill(*inp.args(), nthreads=2)
    assert torch.all(s2[1] == 0)


def test_c_oracle_threads_do_not_change_results():
    inp = W.make_decode_inputs(3, 2, 4, seed=5)
    o1, s1 = C.decode(*inp.args(), nthreads=1)
    o2, s2 = C.decode(*inp.args(), nthreads=3)
    assert torch.equal(o1, o2) and torch.equal(s1, s2)


@pytest.mark.parametrize("lengths,n,h,c", [([150], 0, 1, 1), ([40, 130], 1, 3, 2), ([64], 0, 0, 0)])
def test_chunk_intermediates_match_recurrence(lengths, n, h, c):
    inp = W.make_prefill_inputs(lengths, 2, 4, seed=sum(lengths) + n + h)
    args = _np_args(inp)
    ref = O.chunk_intermediates(*args[:9], n, h, c)
    # the state after the chunk equals the recurrence run up to the chunk end
    cu = np.asarray(args[8])
    end = min(int(cu[n]) + (c + 1) * O.CHUNK, int(cu[n + 1]))
    cut = list(args)
    cut[8] = np.array([0, end - int(cu[n])])
    sl = slice(int(cu[n]), end)
    for i in (0, 1, 2, 5, 7):
        cut[i] = args[i][sl]
    cut[3] = args[3][n:n + 1]
    _, s_rec = O.prefill(*cut)
    assert O.rel_err(ref["St"], s_rec[0, h]) < 1e-5
    # the chunk's outputs: scale (e^gamma QS + PV) equals the recurrence outputs
    o_rec, _ = O.prefill(*cut)
    t0 = c * O.CHUNK
    o_chunk = O.resolve_scale(None) * (np.exp(ref["gam"])[:, None] * ref["QS"] + ref["PV"])
    L = ref["L"]
    assert O.rel_err(o_chunk[:L], O.bf16_to_f32(o_rec[t0:t0 + L, h])) < 5e-3


def test_contest_shapes_span_the_axes():
    """The replay shapes are deterministic and cover the contest axis ranges."""
    cases = W.contest_prefill_cases()
    assert cases == W.contest_prefill_cases()
    totals = [sum(c) for c in cases]
    seqs = [len(c) for c in cases]
    assert min(totals) == W.CONTEST_MIN_TOKENS and max(totals) == W.CONTEST_MAX_TOKENS
    assert min(seqs) == 1 and max(seqs) == W.CONTEST_MAX_SEQS
    assert all(min(c) >= 1 for c in cases)
    assert sum(1 for n in seqs if n <= 4) >= len(cases) // 2
    assert W.CONTEST_DECODE_BATCHES[0] == 1 and W.CONTEST_DECODE_BATCHES[-1] == 64


def test_oracle_decode_pool_reduces_to_decode():
    """One token, identity slots, fp32: the pooled oracle is the definition's decode."""
    inp = W.make_decode_inputs(3, 4, 8, seed=4)
    a = O.to_numpy
    o_ref, s_ref = O.decode(*[a(x) if hasattr(x, "numpy") else x for x in inp.args()])
    o, pool, inter = O.decode_pool(a(inp.q), a(inp.k), a(inp.v), a(inp.A_log), a(inp.a),
                                   a(inp.dt_bias), a(inp.b), inp.scale, a(inp.state),
                                   np.arange(3), cache=True)
    assert (o == o_ref).all()
    assert np.array_equal(pool, s_ref) and np.array_equal(inter[:, 0], s_ref)


def test_oracle_decode_pool_slots_and_l2norm():
    """Slot -1 reads a zero state and is never written; T tokens equal T single steps."""
    inp = W.make_decode_pool_inputs(3, 2, 4, 8, 4, seed=5, normalized_qk=False)
    a = O.to_numpy
    args = (a(inp.q), a(inp.k), a(inp.v), a(inp.A_log), a(inp.a), a(inp.dt_bias), a(inp.b),
            inp.scale)
    o, pool, _ = O.decode_pool(*args, a(inp.pool), a(inp.in_slots), a(inp.out_slots),
                               qk_l2norm=True)
    written = set(int(x) for x in a(inp.out_slots) if x >= 0)
    for s in range(4):
        if s not in written:
            assert np.array_equal(pool[s], a(inp.pool)[s])
    qn = O.l2norm_heads(args[0])
    assert np.allclose(np.sum(qn * qn, axis=-1), 1.0, atol=1e-5)
