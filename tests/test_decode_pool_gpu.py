"""Pooled multi-token decode (C ABI gdn_decode_pool: state pool with read/write
slots, T tokens per sequence, fp32 or bf16 state, per-token state cache, in-kernel
q/k L2 norm) against the oracle's decode_pool, which applies the reference
definition's decode step token by token (oracle/gdn_oracle.py)."""
import numpy as np
import pytest
import torch

import parity as PT
from oracle import gdn_oracle as O
from gdn_b200 import decode, workloads as W

pytestmark = pytest.mark.gpu


def _np(t):
    return O.to_numpy(t)


def _oracle(inp, **kw):
    return O.decode_pool(_np(inp.q), _np(inp.k), _np(inp.v), _np(inp.A_log), _np(inp.a),
                         _np(inp.dt_bias), _np(inp.b), inp.scale, _np(inp.pool),
                         _np(inp.in_slots), _np(inp.out_slots), **kw)


def _state_close(gpu, ref, bf16):
    a = _np(gpu).astype(np.float64)
    r = np.asarray(ref, np.float64)
    if bf16:  # both round the same fp32 state once: at most one bf16 step apart
        assert np.all(np.abs(a - r) <= 2.0 ** -7 * np.abs(r) + 1e-7)
    else:
        PT.assert_state_close(torch.from_numpy(a.reshape(-1, 128, 128)), r.reshape(-1, 128, 128),
                              PT.STATE_RTOL_FP32)


def test_pool_t1_matches_dense_decode():
    """fp32 pool, identity slots, one token: the dense decode entry point."""
    inp = W.make_decode_inputs(6, 4, 8, seed=3, device="cuda")
    o_d, s_d = decode.run(*inp.args())
    pool = inp.state.clone()
    slots = torch.arange(6, dtype=torch.int32, device="cuda")
    o_p = decode.run_pool(inp.q, inp.k, inp.v, inp.A_log, inp.a, inp.dt_bias, inp.b, inp.scale,
                          pool, slots)
    torch.cuda.synchronize()
    PT.assert_o_close(o_p, o_d)
    PT.assert_state_close(pool, _np(s_d), PT.STATE_RTOL_FP32)


@pytest.mark.parametrize("T", [1, 3])
@pytest.mark.parametrize("bf16", [False, True])
@pytest.mark.parametrize("l2", [False, True])
@pytest.mark.parametrize("geom", [(5, 4, 8, 7), (40, 16, 32, 45)])
def test_pool_matches_oracle(T, bf16, l2, geom):
    B, Hq, Hv, P = geom
    inp = W.make_decode_pool_inputs(B, T, Hq, Hv, P, seed=B + 10 * T + bf16 + 2 * l2,
                                    device="cuda", state_bf16=bf16, normalized_qk=not l2)
    o_ref, pool_ref, inter_ref = _oracle(inp, state_bf16=bf16, qk_l2norm=l2, cache=True)
    inter = torch.empty((B, T, Hv, 128, 128), dtype=inp.pool.dtype, device="cuda")
    pool = inp.pool.clone()
    o = decode.run_pool(inp.q, inp.k, inp.v, inp.A_log, inp.a, inp.dt_bias, inp.b, inp.scale,
                        pool, inp.in_slots, inp.out_slots, intermediate=inter, qk_l2norm=l2)
    torch.cuda.synchronize()
    PT.assert_o_close(o, o_ref)
    _state_close(pool, pool_ref, bf16)
    _state_close(inter, inter_ref, bf16)


@pytest.mark.parametrize("T", [2, 4, 7, 8, 9, 16, 17, 24, 25, 32])
@pytest.mark.parametrize("l2", [False, True])
@pytest.mark.parametrize("geom", [(5, 4, 8, 7), (40, 16, 32, 45)])
def test_pool_bf16_multi_token_tensor_core(T, l2, geom):
    """bf16 pools without a per-token cache: 3..16 tokens take the tensor-core
    closed form (gdn_decode_pool_tc.cu, token bounds TP = 8 and 16), fewer and more
    tokens the token-by-token kernel; zero-state and no-write slots, in-kernel L2
    norm, against the token-by-token oracle."""
    B, Hq, Hv, P = geom
    inp = W.make_decode_pool_inputs(B, T, Hq, Hv, P, seed=1000 + 7 * T + l2 + B, device="cuda",
                                    state_bf16=True, normalized_qk=not l2)
    o_ref, pool_ref, _ = _oracle(inp, state_bf16=True, qk_l2norm=l2)
    pool = inp.pool.clone()
    o = decode.run_pool(inp.q, inp.k, inp.v, inp.A_log, inp.a, inp.dt_bias, inp.b, inp.scale,
                        pool, inp.in_slots, inp.out_slots, qk_l2norm=l2)
    torch.cuda.synchronize()
    PT.assert_o_close(o, o_ref)
    _state_close(pool, pool_ref, True)


@pytest.mark.parametrize("dt_bias", [-6.0, 4.0])
def test_pool_bf16_multi_token_decay_extremes(dt_bias):
    """Slow decay (the state and every delta carry across the tokens) and fast
    decay (the decay products underflow) through the closed form."""
    inp = W.make_decode_pool_inputs(6, 8, 4, 8, 8, seed=77, device="cuda", state_bf16=True)
    inp.dt_bias[:] = dt_bias
    o_ref, pool_ref, _ = _oracle(inp, state_bf16=True)
    pool = inp.pool.clone()
    o = decode.run_pool(inp.q, inp.k, inp.v, inp.A_log, inp.a, inp.dt_bias, inp.b, inp.scale,
                        pool, inp.in_slots, inp.out_slots)
    torch.cuda.synchronize()
    PT.assert_o_close(o, o_ref)
    _state_close(pool, pool_ref, True)


@pytest.mark.parametrize("T", [12, 32])
def test_pool_bf16_many_tokens(T):
    """bf16 multi-token steps stage T tokens in shared memory: above T = 11 that is
    more than the 48 KiB default (T = 32, the largest staged count: 49,408 B)."""
    B, Hq, Hv, P = 3, 4, 8, 4
    inp = W.make_decode_pool_inputs(B, T, Hq, Hv, P, seed=300 + T, device="cuda", state_bf16=True)
    o_ref, pool_ref, _ = _oracle(inp, state_bf16=True)
    pool = inp.pool.clone()
    o = decode.run_pool(inp.q, inp.k, inp.v, inp.A_log, inp.a, inp.dt_bias, inp.b, inp.scale,
                        pool, inp.in_slots, inp.out_slots)
    torch.cuda.synchronize()
    PT.assert_o_close(o, o_ref)
    _state_close(pool, pool_ref, True)


@pytest.mark.parametrize("T", [2, 4, 8, 17, 32])
@pytest.mark.parametrize("l2", [False, True])
@pytest.mark.parametrize("geom", [(5, 4, 8, 7), (40, 16, 32, 45)])
def test_pool_f32_multi_token(T, l2, geom):
    """fp32 pools, 2..32 tokens without a per-token cache (the 64-row kernel: tokens
    staged in shared memory, more than the 48 KiB default above T = 11); zero-state
    and no-write slots, in-kernel L2 norm, against the token-by-token oracle."""
    B, Hq, Hv, P = geom
    inp = W.make_decode_pool_inputs(B, T, Hq, Hv, P, seed=2000 + 7 * T + l2 + B, device="cuda",
                                    state_bf16=False, normalized_qk=not l2)
    o_ref, pool_ref, _ = _oracle(inp, state_bf16=False, qk_l2norm=l2)
    pool = inp.pool.clone()
    o = decode.run_pool(inp.q, inp.k, inp.v, inp.A_log, inp.a, inp.dt_bias, inp.b, inp.scale,
                        pool, inp.in_slots, inp.out_slots, qk_l2norm=l2)
    torch.cuda.synchronize()
    PT.assert_o_close(o, o_ref)
    _state_close(pool, pool_ref, False)


@pytest.mark.parametrize("dt_bias", [-6.0, 4.0])
def test_pool_f32_multi_token_decay_extremes(dt_bias):
    inp = W.make_decode_pool_inputs(6, 8, 4, 8, 8, seed=78, device="cuda", state_bf16=False)
    inp.dt_bias[:] = dt_bias
    o_ref, pool_ref, _ = _oracle(inp, state_bf16=False)
    pool = inp.pool.clone()
    o = decode.run_pool(inp.q, inp.k, inp.v, inp.A_log, inp.a, inp.dt_bias, inp.b, inp.scale,
                        pool, inp.in_slots, inp.out_slots)
    torch.cuda.synchronize()
    PT.assert_o_close(o, o_ref)
    _state_close(pool, pool_ref, False)


def test_pool_f32_no_state_update_leaves_pool():
    inp = W.make_decode_pool_inputs(4, 4, 4, 8, 6, seed=10, device="cuda", state_bf16=False)
    o_ref, _, _ = _oracle(inp, state_bf16=False, no_state_update=True)
    pool = inp.pool.clone()
    o = decode.run_pool(inp.q, inp.k, inp.v, inp.A_log, inp.a, inp.dt_bias, inp.b, inp.scale,
                        pool, inp.in_slots, inp.out_slots, no_state_update=True)
    torch.cuda.synchronize()
    PT.assert_o_close(o, o_ref)
    assert torch.equal(pool, inp.pool)


def test_pool_no_state_update_leaves_pool():
    inp = W.make_decode_pool_inputs(4, 2, 4, 8, 6, seed=9, device="cuda", state_bf16=True)
    o_ref, _, _ = _oracle(inp, state_bf16=True, no_state_update=True)
    pool = inp.pool.clone()
    o = decode.run_pool(inp.q, inp.k, inp.v, inp.A_log, inp.a, inp.dt_bias, inp.b, inp.scale,
                        pool, inp.in_slots, inp.out_slots, no_state_update=True)
    torch.cuda.synchronize()
    PT.assert_o_close(o, o_ref)
    assert torch.equal(pool, inp.pool)


def test_pool_argument_errors():
    inp = W.make_decode_pool_inputs(3, 1, 4, 8, 4, seed=2, device="cuda")
    with pytest.raises(TypeError):
        decode.run_pool(inp.q, inp.k, inp.v, inp.A_log, inp.a, inp.dt_bias, inp.b, inp.scale,
                        inp.pool, inp.in_slots.long())
    with pytest.raises(ValueError):
        decode.run_pool(inp.q, inp.k, inp.v, inp.A_log, inp.a, inp.dt_bias, inp.b, inp.scale,
                        inp.pool, inp.in_slots[:2].contiguous())
