"""CPU oracle for the Gated DeltaNet (GDN) decode and prefill path.

TEST INFRASTRUCTURE ONLY.  Only ``tests/``, ``__graft_entry__.smoke()`` and the
``cpu_baseline`` / ``--impl reference`` legs of ``bench.py`` may import this module,
and only as the checker or the timed CPU baseline.  The product path
(``gdn_b200``) never calls it and fails loudly when its CUDA library is missing.

What it restates (numpy, fp32 unless noted):

* ``gates``            -- definitions/gdn/gdn_decode_qk4_v8_d128_k_last.md:91-94
                          (g = exp(-exp(A_log) * softplus(a + dt_bias)), beta = sigmoid(b));
                          torch's softplus switches to the identity above 20.
* ``decode``           -- definitions/gdn/gdn_decode_qk4_v8_d128_k_last.md:61-133,
                          the per-(sequence, v-head) recurrence, vectorised over (B, Hv);
                          head-count asserts lifted (any Hv with Hv % Hq == 0).
* ``prefill``          -- definitions/gdn/gdn_prefill_qk4_v8_d128_k_last.md:62-142,
                          the per-token loop over each packed sequence, vectorised over
                          heads; ``state=None`` means a zero initial state.
* ``prep_meta``        -- gdn_prefill/solution/python/cuda_prep_meta_v2.cu:11-70
                          (chunk_offsets[N+1], chunk_indices[C, 2] for chunk size 64).
* ``chunked_prefill``  -- the chunk-64 WY/UT form that the tensor-core kernels compute
                          (gdn_prefill/solution/python/cuda_kkt_inv_uw_v1.cu:1-20 for
                          the per-chunk quantities, cuda_h_v2b.cu / cuda_o_v1.cu for
                          the state scan and the output), in fp64 by default, with an
                          optional emulation of the bf16 rounding points of the GPU path.

Pinning: ``tests/golden/make_golden.py`` executes the reference's own definition
code (extracted from the definition markdown) on seeded inputs and stores the
outputs under ``tests/golden``; ``tests/test_oracle.py`` checks this module against
them.
"""
from __future__ import annotations

import math
from typing import Optional, Sequence

import numpy as np

HEAD = 128
CHUNK = 64


# ---------------------------------------------------------------- bf16 helpers
def bf16_to_f32(bits: np.ndarray) -> np.ndarray:
    """bf16 bit patterns (uint16/int16) -> float32 values."""
    u = np.asarray(bits).astype(np.uint16).astype(np.uint32) << 16
    return u.view(np.float32)


def f32_to_bf16(x: np.ndarray) -> np.ndarray:
    """float32 -> bf16 bit patterns, round-to-nearest-even (finite inputs)."""
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32).astype(np.uint64)
    u = u + 0x7FFF + ((u >> 16) & 1)
    return (u >> 16).astype(np.uint16)


def round_bf16(x: np.ndarray) -> np.ndarray:
    """Round to the nearest bf16 value, returned as float32."""
    return bf16_to_f32(f32_to_bf16(np.asarray(x, dtype=np.float32)))


def to_numpy(t):
    """torch tensor (any device) -> numpy; bf16 becomes float32 values."""
    import torch
    if t is None:
        return None
    if isinstance(t, np.ndarray):
        return t
    t = t.detach().cpu()
    if t.dtype == torch.bfloat16:
        return bf16_to_f32(t.view(torch.int16).numpy().view(np.uint16))
    return t.numpy()


# ---------------------------------------------------------------- gates
def softplus(x: np.ndarray) -> np.ndarray:
    x = np.asarray(x, dtype=np.float32)
    safe = np.minimum(x, np.float32(20.0))
    return np.where(x > 20.0, x, np.log1p(np.exp(safe))).astype(np.float32)


def sigmoid(x: np.ndarray) -> np.ndarray:
    x = np.asarray(x, dtype=np.float32)
    return (np.float32(1.0) / (np.float32(1.0) + np.exp(-x))).astype(np.float32)


def gates(A_log, a, dt_bias, b):
    """Multiplicative decay g and update gate beta, broadcast over a's shape
    (decode def :91-94, prefill def :91-94)."""
    x = np.asarray(a, np.float32) + np.asarray(dt_bias, np.float32)
    g = np.exp(-np.exp(np.asarray(A_log, np.float32)) * softplus(x)).astype(np.float32)
    beta = sigmoid(b)
    return g, beta


def log_gates(A_log, a, dt_bias, b):
    """Log-space decay log(g) = -exp(A_log) * softplus(a + dt_bias) and beta."""
    x = np.asarray(a, np.float32) + np.asarray(dt_bias, np.float32)
    lg = (-np.exp(np.asarray(A_log, np.float32)) * softplus(x)).astype(np.float32)
    return lg, sigmoid(b)


def resolve_scale(scale, head=HEAD) -> float:
    if scale is None or float(scale) == 0.0:
        return 1.0 / math.sqrt(head)
    return float(scale)


# ---------------------------------------------------------------- decode
def decode(q, k, v, state, A_log, a, dt_bias, b, scale):
    """GDN decode (T=1).  Inputs are float32 arrays holding the bf16 values:
    q, k [B,1,Hq,128]; v [B,1,Hv,128]; state [B,Hv,V,K] or None; A_log, dt_bias [Hv];
    a, b [B,1,Hv].  Returns (o as bf16 bits [B,1,Hv,128], new_state fp32 [B,Hv,V,K]).

    Follows definitions/gdn/gdn_decode_qk4_v8_d128_k_last.md:96-132:
    old_state = g*S (S in [K,V] form), old_v = k @ old_state,
    new_v = beta*v + (1-beta)*old_v, S' = old_state - k^T old_v + k^T new_v,
    o = scale * q @ S'.
    """
    q = np.asarray(q, np.float32)
    B, T, Hq, K = q.shape
    Hv = v.shape[2]
    assert T == 1 and K == HEAD and v.shape[3] == HEAD and Hv % Hq == 0
    scale = np.float32(resolve_scale(scale, K))
    g, beta = gates(A_log, a, dt_bias, b)          # [B,1,Hv]
    g = g[:, 0]
    beta = beta[:, 0]
    rep = Hv // Hq
    qe = np.repeat(q[:, 0], rep, axis=1)            # [B,Hv,K]
    ke = np.repeat(np.asarray(k, np.float32)[:, 0], rep, axis=1)
    ve = np.asarray(v, np.float32)[:, 0]           # [B,Hv,V]
    if state is None:
        S = np.zeros((B, Hv, K, HEAD), np.float32)
    else:
        S = np.asarray(state, np.float32).transpose(0, 1, 3, 2)  # [B,Hv,K,V]
    old_state = g[:, :, None, None] * S
    old_v = np.einsum("bhk,bhkv->bhv", ke, old_state)
    new_v = beta[..., None] * ve + (np.float32(1.0) - beta[..., None]) * old_v
    remove = ke[..., :, None] * old_v[..., None, :]
    update = ke[..., :, None] * new_v[..., None, :]
    S = old_state - remove + update
    o = scale * np.einsum("bhk,bhkv->bhv", qe, S)
    new_state = np.ascontiguousarray(S.transpose(0, 1, 3, 2)).astype(np.float32)
    return f32_to_bf16(o[:, None].astype(np.float32)), new_state


def l2norm_heads(x):
    """x / sqrt(sum x^2 + 1e-6) over the last axis, in fp32 (the in-kernel q/k
    normalisation of the pooled decode)."""
    x = np.asarray(x, np.float32)
    return x / np.sqrt(np.sum(x * x, axis=-1, keepdims=True, dtype=np.float32) + np.float32(1e-6))


def decode_pool(q, k, v, A_log, a, dt_bias, b, scale, pool, in_slots, out_slots=None,
                state_bf16=False, qk_l2norm=False, no_state_update=False, cache=False):
    """Pooled multi-token decode (the serving form; no reference counterpart).

    q, k [B,T,Hq,128]; v [B,T,Hv,128]; a, b [B,T,Hv] (float32 arrays holding the
    bf16 values); pool [P,Hv,V,K] (fp32 values; with state_bf16 they are bf16
    values and every stored state is rounded to bf16).  Sequence i starts from
    pool[in_slots[i]] (zero if the slot is negative or >= P), applies its T tokens
    in order with the decode step of definitions/gdn/gdn_decode_qk4_v8_d128_k_last.md:96-132
    (the ``decode`` above, one token at a time), and writes its final state to
    pool[out_slots[i]] (default in_slots; skipped if negative, >= P or
    no_state_update).  Returns (o as bf16 bits [B,T,Hv,128], new pool,
    per-token states [B,T,Hv,V,K] or None)."""
    q = np.asarray(q, np.float32)
    k = np.asarray(k, np.float32)
    B, T, Hq, _ = q.shape
    Hv = v.shape[2]
    P = pool.shape[0]
    if qk_l2norm:
        q, k = l2norm_heads(q), l2norm_heads(k)
    rnd = round_bf16 if state_bf16 else (lambda x: np.asarray(x, np.float32))
    new_pool = np.array(pool, np.float32, copy=True)
    o = np.zeros((B, T, Hv, HEAD), np.uint16)
    inter = np.zeros((B, T, Hv, HEAD, HEAD), np.float32) if cache else None
    ins = [int(x) for x in np.asarray(in_slots).reshape(-1)]
    outs = ins if out_slots is None else [int(x) for x in np.asarray(out_slots).reshape(-1)]
    finals = []
    for i in range(B):
        S = pool[ins[i]][None] if 0 <= ins[i] < P else None
        for t in range(T):
            ob, S = decode(q[i:i + 1, t:t + 1], k[i:i + 1, t:t + 1], v[i:i + 1, t:t + 1], S, A_log,
                           a[i:i + 1, t:t + 1], dt_bias, b[i:i + 1, t:t + 1], scale)
            o[i, t] = ob[0, 0]
            if cache:
                inter[i, t] = rnd(S[0])
        finals.append(S[0])
    if not no_state_update:
        for i in range(B):
            if 0 <= outs[i] < P:
                new_pool[outs[i]] = rnd(finals[i])
    return o, new_pool, inter


# ---------------------------------------------------------------- prefill
def prefill(q, k, v, state, A_log, a, dt_bias, b, cu_seqlens, scale, qk_l2norm=False):
    """GDN prefill over packed variable-length sequences.  q, k [T,Hq,128];
    v [T,Hv,128]; state [N,Hv,V,K] or None; a, b [T,Hv]; cu_seqlens [N+1].
    Returns (o bf16 bits [T,Hv,128], new_state fp32 [N,Hv,V,K]).

    Follows definitions/gdn/gdn_prefill_qk4_v8_d128_k_last.md:108-142 token by
    token; sequences of length <= 0 keep a zero final state (def :113-114 skips
    them and new_state starts at zero).  ``qk_l2norm`` first normalises q and k
    per head in fp32 (``l2norm_heads``), the in-kernel option of the GPU path."""
    if qk_l2norm:
        q, k = l2norm_heads(q), l2norm_heads(k)
    q = np.asarray(q, np.float32)
    T, Hq, K = q.shape
    Hv = v.shape[1]
    assert K == HEAD and Hv % Hq == 0
    cu = [int(x) for x in np.asarray(cu_seqlens).reshape(-1)]
    N = len(cu) - 1
    scale = np.float32(resolve_scale(scale, K))
    g, beta = gates(A_log, a, dt_bias, b)          # [T,Hv]
    rep = Hv // Hq
    qe = np.repeat(q, rep, axis=1)
    ke = np.repeat(np.asarray(k, np.float32), rep, axis=1)
    vv = np.asarray(v, np.float32)
    out = np.zeros((T, Hv, HEAD), np.float32)
    new_state = np.zeros((N, Hv, HEAD, K), np.float32)
    one = np.float32(1.0)
    for n in range(N):
        s, e = cu[n], cu[n + 1]
        if e - s <= 0:
            continue
        if state is not None:
            S = np.asarray(state[n], np.float32).transpose(0, 2, 1).copy()  # [H,K,V]
        else:
            S = np.zeros((Hv, K, HEAD), np.float32)
        for t in range(s, e):
            old_state = g[t][:, None, None] * S
            old_v = np.einsum("hk,hkv->hv", ke[t], old_state)
            new_v = beta[t][:, None] * vv[t] + (one - beta[t][:, None]) * old_v
            S = old_state - ke[t][:, :, None] * old_v[:, None, :] \
                + ke[t][:, :, None] * new_v[:, None, :]
            out[t] = scale * np.einsum("hk,hkv->hv", qe[t], S)
        new_state[n] = S.transpose(0, 2, 1)
    return f32_to_bf16(out), new_state


# ---------------------------------------------------------------- chunk metadata
def prep_meta(cu_seqlens, chunk=CHUNK):
    """(chunk_offsets int32 [N+1], chunk_indices int32 [C,2]) for packed sequences,
    as cuda_prep_meta_v2.cu:11-70 produces them: chunk_offsets[n] is the number of
    64-token chunks before sequence n, chunk_indices lists (seq, chunk-in-seq)."""
    cu = np.asarray(cu_seqlens, dtype=np.int64).reshape(-1)
    lens = np.diff(cu)
    nch = np.maximum((lens + chunk - 1) // chunk, 0)
    offsets = np.zeros(len(cu), np.int32)
    offsets[1:] = np.cumsum(nch)
    idx = [(n, c) for n in range(len(nch)) for c in range(int(nch[n]))]
    indices = np.array(idx, np.int32).reshape(-1, 2)
    return offsets, indices


def chunk_upper_bound(T: int, N: int, chunk=CHUNK) -> int:
    """Upper bound on the number of chunks of any packing of T tokens into N
    sequences (gdn_prefill/solution/python/chunk_v12.py:53)."""
    # sum_n ceil(L_n / C) <= N + floor((T - N) / C) when every L_n >= 1, and a
    # sequence with L_n = 0 has no chunk, so at most T sequences carry chunks.
    if T <= 0:
        return 0
    if T < N:
        return T
    return N + (T - N) // chunk


# ---------------------------------------------------------------- chunked form
def chunked_prefill(q, k, v, state, A_log, a, dt_bias, b, cu_seqlens, scale,
                    chunk=CHUNK, dtype=np.float64, bf16_points: Sequence[str] = ()):
    """Chunk-wise WY/UT restatement of ``prefill``.

    Per sequence, per v-head, per chunk of C tokens with gamma = within-chunk
    cumulative log-decay, and S the [K,V] state at the chunk start:

        A[i,j]  = beta_i (k_i . k_j) exp(gamma_i - gamma_j)     (i > j)
        Tm      = (I + A)^-1
        U       = Tm diag(beta) V
        W       = Tm diag(beta exp(gamma)) K
        Vn      = U - W S                                          (the delta rows)
        O       = scale (diag(exp(gamma)) Q S + (tril(Q K^T) * exp(gamma_i - gamma_j)) Vn)
        S_next  = exp(gamma_C) S + (K * exp(gamma_C - gamma))^T Vn

    ``bf16_points`` names intermediates rounded to bf16 before use, emulating the
    GPU kernels' operand precision: any of "T", "UW", "Vn", "S", "Kd", "QKmask".
    Returns float arrays (o [T,Hv,128] unrounded, new_state [N,Hv,V,K])."""
    q = np.asarray(q, dtype)
    T, Hq, K = q.shape
    Hv = v.shape[1]
    rep = Hv // Hq
    cu = [int(x) for x in np.asarray(cu_seqlens).reshape(-1)]
    N = len(cu) - 1
    scale = resolve_scale(scale, K)
    lg, beta = log_gates(A_log, a, dt_bias, b)
    lg = lg.astype(dtype)
    beta = beta.astype(dtype)
    ke = np.repeat(np.asarray(k, dtype), rep, axis=1)
    qe = np.repeat(q, rep, axis=1)
    vv = np.asarray(v, dtype)
    out = np.zeros((T, Hv, HEAD), dtype)
    new_state = np.zeros((N, Hv, HEAD, K), dtype)

    def rb(name, x):
        return round_bf16(x).astype(dtype) if name in bf16_points else x

    for n in range(N):
        s0, e0 = cu[n], cu[n + 1]
        if e0 - s0 <= 0:
            continue
        for h in range(Hv):
            if state is not None:
                S = np.asarray(state[n, h], dtype).T.copy()          # [K,V]
            else:
                S = np.zeros((K, HEAD), dtype)
            for cs in range(s0, e0, chunk):
                ce = min(cs + chunk, e0)
                Kc, Qc, Vc = ke[cs:ce, h], qe[cs:ce, h], vv[cs:ce, h]
                gam = np.cumsum(lg[cs:ce, h])
                bc = beta[cs:ce, h]
                diff = gam[:, None] - gam[None, :]
                low = np.tril(np.ones((ce - cs, ce - cs), bool), -1)
                E = np.where(low | np.eye(ce - cs, dtype=bool), np.exp(np.minimum(diff, 0)), 0)
                A = np.where(low, bc[:, None] * (Kc @ Kc.T) * E, 0)
                Tm = rb("T", np.linalg.inv(np.eye(ce - cs) + A))
                U = rb("UW", Tm @ (bc[:, None] * Vc))
                W = rb("UW", Tm @ ((bc * np.exp(gam))[:, None] * Kc))
                Sb = rb("S", S)
                Vn = rb("Vn", U - W @ Sb)
                QK = rb("QKmask", np.tril(Qc @ Kc.T) * E)
                out[cs:ce, h] = scale * (np.exp(gam)[:, None] * (Qc @ Sb) + QK @ Vn)
                Kd = rb("Kd", Kc * np.exp(gam[-1] - gam)[:, None])
                S = np.exp(gam[-1]) * S + Kd.T @ Vn
            new_state[n, h] = S.T
    return out, new_state


# ---------------------------------------------------------------- comparisons
def rel_err(x, ref) -> float:
    """Norm-wise relative error ||x - ref||_F / max(||ref||_F, tiny)."""
    x = np.asarray(x, np.float64)
    ref = np.asarray(ref, np.float64)
    den = max(np.linalg.norm(ref), 1e-30)
    return float(np.linalg.norm(x - ref) / den)


def chunk_intermediates(q, k, v, state, A_log, a, dt_bias, b, cu_seqlens, n, h, c, chunk=CHUNK):
    """fp64 intermediates of chunk ``c`` of sequence ``n``, v-head ``h``, in the
    definitions the fused tensor-core kernel uses (it dumps the same names):
    gam, bet (zero log-decay and beta past the sequence end), A, P, T, U, W, KS
    (K times the chunk-start state, the kernel's form of W S = T^ (K S)), Vn, QS,
    PV and the k-last state after the chunk.  Rows past the sequence end hold
    the packed neighbours' data (or zeros past T), as the kernel's tile loads do.
    The state at the chunk start comes from the token recurrence in fp64."""
    T_, Hq, K = np.asarray(q).shape
    Hv = np.asarray(v).shape[1]
    qh = h // (Hv // Hq)
    cu = [int(x) for x in np.asarray(cu_seqlens).reshape(-1)]
    s0, e0 = cu[n], cu[n + 1]
    lg_all, beta_all = log_gates(A_log, a, dt_bias, b)
    S = (np.asarray(state[n, h], np.float64).T.copy() if state is not None
         else np.zeros((K, HEAD)))
    kk = np.asarray(k, np.float64)[:, qh]
    qq = np.asarray(q, np.float64)[:, qh]
    vv = np.asarray(v, np.float64)[:, h]
    t0 = s0 + c * chunk
    for t in range(s0, t0):                       # recurrence up to the chunk start
        g = np.exp(float(lg_all[t, h]))
        S = g * S
        S = S + np.outer(kk[t], float(beta_all[t, h]) * (vv[t] - kk[t] @ S))
    L = min(chunk, e0 - t0)
    rows = np.arange(t0, t0 + chunk)
    inb = rows < T_
    Kc = np.where(inb[:, None], kk[np.minimum(rows, T_ - 1)], 0.0)
    Qc = np.where(inb[:, None], qq[np.minimum(rows, T_ - 1)], 0.0)
    Vc = np.where(inb[:, None], vv[np.minimum(rows, T_ - 1)], 0.0)
    valid = np.arange(chunk) < L
    lg = np.where(valid, lg_all[np.minimum(rows, T_ - 1), h].astype(np.float64), 0.0)
    bet = np.where(valid, beta_all[np.minimum(rows, T_ - 1), h].astype(np.float64), 0.0)
    gam = np.cumsum(lg)
    diff = np.minimum(gam[:, None] - gam[None, :], 0.0)
    low = np.tril(np.ones((chunk, chunk), bool), -1)
    E = np.exp(diff)
    A = np.where(low, bet[:, None] * (Kc @ Kc.T) * E, 0.0)
    P = np.where(low | np.eye(chunk, dtype=bool), (Qc @ Kc.T) * E, 0.0)
    Tm = np.linalg.inv(np.eye(chunk) + A)
    U = Tm @ (bet[:, None] * Vc)
    W = Tm @ ((bet * np.exp(gam))[:, None] * Kc)
    Vn = U - W @ S
    Vn[~valid] = 0.0
    QS = Qc @ S
    KS = Kc @ S
    PV = P @ Vn
    S_after = np.exp(gam[-1]) * S + Kc.T @ (np.exp(gam[-1] - gam)[:, None] * Vn)
    return dict(gam=gam, bet=bet, A=A, P=P, T=Tm, U=U, W=W, KS=KS, Vn=Vn, QS=QS, PV=PV,
                St=S_after.T, L=L, valid=valid)
