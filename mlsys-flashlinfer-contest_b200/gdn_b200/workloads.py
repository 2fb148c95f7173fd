"""Seeded synthetic GDN inputs.

The contest's workload tensors (safetensors blobs of the HF dataset
``flashinfer-ai/mlsys26-contest``) are not available offline, so every test and
benchmark uses seeded synthetic tensors with the shapes and value distributions of
the contest definitions ``definitions/gdn/gdn_decode_qk4_v8_d128_k_last.md:27-39``
and ``definitions/gdn/gdn_prefill_qk4_v8_d128_k_last.md:28-41``:

* q, k, v ~ N(0, 1) in bf16; q and k L2-normalised per head (in fp32, then rounded);
* A_log = log(U(1, 16)) fp32, dt_bias ~ U(-1, 1) fp32;
* a, b ~ N(0, 1) bf16 (decode shape [B, 1, Hv], prefill shape [T, Hv]);
* initial state fp32 ~ N(0, 0.05^2) in the k-last layout [B or N, Hv, V, K].

Generation runs on the device named by ``device`` with a ``torch.Generator``
seeded per call; on CPU the result is bit-identical across machines that run the
same torch build, which is what the committed golden fixtures rely on.
"""
from __future__ import annotations

import math
from dataclasses import dataclass
from pathlib import Path
from typing import Optional, Sequence

import torch

HEAD_SIZE = 128


def _gen(device, seed: int) -> torch.Generator:
    g = torch.Generator(device=device)
    g.manual_seed(int(seed))
    return g


def _normal(shape, gen, device, std=1.0):
    return torch.randn(shape, generator=gen, device=device, dtype=torch.float32) * std


def _uniform(shape, gen, device, lo, hi):
    return torch.rand(shape, generator=gen, device=device, dtype=torch.float32) * (hi - lo) + lo


def _l2norm_bf16(x: torch.Tensor) -> torch.Tensor:
    x = x / x.norm(dim=-1, keepdim=True).clamp_min(1e-6)
    return x.to(torch.bfloat16)


@dataclass
class DecodeInputs:
    q: torch.Tensor
    k: torch.Tensor
    v: torch.Tensor
    state: Optional[torch.Tensor]
    A_log: torch.Tensor
    a: torch.Tensor
    dt_bias: torch.Tensor
    b: torch.Tensor
    scale: float

    def args(self):
        """Positional arguments in the definition's input order."""
        return (self.q, self.k, self.v, self.state, self.A_log, self.a, self.dt_bias,
                self.b, self.scale)


@dataclass
class PrefillInputs:
    q: torch.Tensor
    k: torch.Tensor
    v: torch.Tensor
    state: Optional[torch.Tensor]
    A_log: torch.Tensor
    a: torch.Tensor
    dt_bias: torch.Tensor
    b: torch.Tensor
    cu_seqlens: torch.Tensor
    scale: float

    def args(self):
        return (self.q, self.k, self.v, self.state, self.A_log, self.a, self.dt_bias,
                self.b, self.cu_seqlens, self.scale)


def head_params(Hv: int, gen, device):
    A_log = torch.log(_uniform((Hv,), gen, device, 1.0, 16.0))
    dt_bias = _uniform((Hv,), gen, device, -1.0, 1.0)
    return A_log, dt_bias


def make_decode_inputs(B: int, Hq: int = 16, Hv: int = 32, seed: int = 0,
                       device="cpu", with_state: bool = True,
                       state_std: float = 0.05) -> DecodeInputs:
    """Decode inputs of BASELINE configs 0/1/4 (T=1)."""
    gen = _gen(device, seed)
    d = HEAD_SIZE
    q = _l2norm_bf16(_normal((B, 1, Hq, d), gen, device))
    k = _l2norm_bf16(_normal((B, 1, Hq, d), gen, device))
    v = _normal((B, 1, Hv, d), gen, device).to(torch.bfloat16)
    A_log, dt_bias = head_params(Hv, gen, device)
    a = _normal((B, 1, Hv), gen, device).to(torch.bfloat16)
    b = _normal((B, 1, Hv), gen, device).to(torch.bfloat16)
    state = _normal((B, Hv, d, d), gen, device, state_std) if with_state else None
    return DecodeInputs(q, k, v, state, A_log, a, dt_bias, b, 1.0 / math.sqrt(d))


@dataclass
class DecodePoolInputs:
    q: torch.Tensor       # [B,T,Hq,128] bf16
    k: torch.Tensor
    v: torch.Tensor       # [B,T,Hv,128] bf16
    A_log: torch.Tensor
    a: torch.Tensor       # [B,T,Hv] bf16
    dt_bias: torch.Tensor
    b: torch.Tensor
    scale: float
    pool: torch.Tensor    # [P,Hv,128,128] fp32 or bf16
    in_slots: torch.Tensor   # [B] int32
    out_slots: torch.Tensor  # [B] int32


def make_decode_pool_inputs(B: int, T: int, Hq: int, Hv: int, pool_size: int, seed: int = 0,
                            device="cpu", state_bf16: bool = False, normalized_qk: bool = True,
                            state_std: float = 0.05) -> DecodePoolInputs:
    """Pooled multi-token decode inputs: T tokens per sequence, a state pool of
    ``pool_size`` slots, read slots a seeded choice of distinct slots (the first
    sequence reads slot -1: zero state).  Sequences write back in place, except
    that every third one writes to a slot nobody reads (while free slots last) and
    the last one writes slot -1 (no write-back): no slot is both read and written
    by different sequences, which would race.  ``normalized_qk=False`` leaves q, k
    un-normalised (for the in-kernel L2 norm)."""
    assert pool_size >= B
    gen = _gen(device, seed)
    d = HEAD_SIZE
    q = _normal((B, T, Hq, d), gen, device)
    k = _normal((B, T, Hq, d), gen, device)
    q = _l2norm_bf16(q) if normalized_qk else q.to(torch.bfloat16)
    k = _l2norm_bf16(k) if normalized_qk else k.to(torch.bfloat16)
    v = _normal((B, T, Hv, d), gen, device).to(torch.bfloat16)
    A_log, dt_bias = head_params(Hv, gen, device)
    a = _normal((B, T, Hv), gen, device).to(torch.bfloat16)
    b = _normal((B, T, Hv), gen, device).to(torch.bfloat16)
    pool = _normal((pool_size, Hv, d, d), gen, device, state_std)
    if state_bf16:
        pool = pool.to(torch.bfloat16)
    cpu_gen = _gen("cpu", seed + 1)
    perm = torch.randperm(pool_size, generator=cpu_gen).to(torch.int32)
    ins, free = perm[:B].clone(), [int(x) for x in perm[B:]]
    outs = ins.clone()
    for i in range(0, B, 3):
        if free:
            outs[i] = free.pop()
    ins[0] = -1
    outs[-1] = -1
    return DecodePoolInputs(q, k, v, A_log, a, dt_bias, b, 1.0 / math.sqrt(d), pool,
                            ins.to(device), outs.to(device))


def varlen_lengths(n: int, lo: int, hi: int, seed: int) -> list:
    """n sequence lengths ~ U[lo, hi] (inclusive), seeded."""
    gen = _gen("cpu", seed)
    return [int(x) for x in torch.randint(lo, hi + 1, (n,), generator=gen)]


def even_lengths(total: int, n: int) -> list:
    """Equal-length rewrite of a varlen batch (the reference's even generator,
    gdn_prefill/scripts/run_local_fast_even.py:32-44): same total, n sequences."""
    base, rem = divmod(total, n)
    return [base + (1 if i < rem else 0) for i in range(n)]


def uneven_lengths(total: int, n: int) -> list:
    """n-1 sequences of length 1 plus one long sequence with the same total
    (gdn_prefill/scripts/run_local_fast_uneven.py)."""
    if n <= 1:
        return [total]
    return [1] * (n - 1) + [total - (n - 1)]


def make_prefill_inputs(lengths: Sequence[int], Hq: int = 16, Hv: int = 32, seed: int = 0,
                        device="cpu", with_state=True, state_std: float = 0.05,
                        zero_state_every_other: bool = False,
                        cu_dtype=torch.int64, normalized_qk: bool = True) -> PrefillInputs:
    """Packed varlen prefill inputs (BASELINE configs 2/3).

    ``zero_state_every_other`` zeroes the initial state of every second sequence
    (config 2: "initial state is zero for half the sequences");
    ``normalized_qk=False`` leaves q, k un-normalised (for the in-kernel L2 norm)."""
    gen = _gen(device, seed)
    d = HEAD_SIZE
    N = len(lengths)
    T = int(sum(lengths))
    q = _normal((T, Hq, d), gen, device)
    k = _normal((T, Hq, d), gen, device)
    q = _l2norm_bf16(q) if normalized_qk else q.to(torch.bfloat16)
    k = _l2norm_bf16(k) if normalized_qk else k.to(torch.bfloat16)
    v = _normal((T, Hv, d), gen, device).to(torch.bfloat16)
    A_log, dt_bias = head_params(Hv, gen, device)
    a = _normal((T, Hv), gen, device).to(torch.bfloat16)
    b = _normal((T, Hv), gen, device).to(torch.bfloat16)
    state = None
    if with_state:
        state = _normal((N, Hv, d, d), gen, device, state_std)
        if zero_state_every_other:
            state[0::2] = 0.0
    cu = [0]
    for L in lengths:
        cu.append(cu[-1] + int(L))
    cu_seqlens = torch.tensor(cu, dtype=cu_dtype, device=device)
    return PrefillInputs(q, k, v, state, A_log, a, dt_bias, b, cu_seqlens, 1.0 / math.sqrt(d))


# Named BASELINE.json configurations.
def config_lengths(name: str) -> list:
    if name == "prefill_varlen":      # config 2: 16 seqs, len ~ U[64, 1024]
        return varlen_lengths(16, 64, 1024, seed=2)
    if name == "prefill_long":        # config 3: 4 x 16384
        return [16384] * 4
    raise KeyError(name)


# ---- contest-shape replay ---------------------------------------------------
# The contest scores solutions on workloads of the qk4_v8 definitions (Hq = Hk = 4,
# Hv = 8).  Their axes, as listed in the reference's workloads/gdn/*.md, span:
# decode batch_size 1..64 (values 1, 4, 8, 16, 32, 48, 64); prefill total_seq_len
# 6..8192 over num_seqs 1..57, most batches holding 1-4 sequences.  The tensors
# themselves are not available, so the replay draws seeded synthetic shapes over
# the same ranges (both extremes included) and feeds them the usual distributions.
CONTEST_HQ, CONTEST_HV = 4, 8
CONTEST_DECODE_BATCHES = (1, 4, 8, 16, 32, 48, 64)
CONTEST_MAX_TOKENS, CONTEST_MAX_SEQS, CONTEST_MIN_TOKENS = 8192, 57, 6


def split_lengths(total: int, n: int, gen: torch.Generator) -> list:
    """Ragged split of ``total`` tokens into ``n`` sequences of length >= 1."""
    if n <= 1:
        return [int(total)]
    cuts = torch.randperm(total - 1, generator=gen)[: n - 1] + 1
    cuts = sorted(int(c) for c in cuts)
    edges = [0] + cuts + [int(total)]
    return [edges[i + 1] - edges[i] for i in range(n)]


def contest_prefill_cases(n_random: int = 20, seed: int = 26) -> list:
    """Seeded lists of sequence lengths spanning the contest prefill axes: the
    four corners (fewest/most tokens with one sequence and with the most
    sequences), then ``n_random`` draws with num_seqs mostly in 1..4 (a tail up
    to 57) and total_seq_len log-uniform over [max(6, num_seqs), 8192]."""
    gen = _gen("cpu", seed)
    cases = [[CONTEST_MIN_TOKENS], [CONTEST_MAX_TOKENS],
             split_lengths(CONTEST_MAX_SEQS * 2, CONTEST_MAX_SEQS, gen),
             split_lengths(CONTEST_MAX_TOKENS, CONTEST_MAX_SEQS, gen)]
    for _ in range(n_random):
        u = float(torch.rand((), generator=gen))
        if u < 0.65:
            n = 1 + int(torch.randint(0, 4, (), generator=gen))
        else:
            n = int(round(math.exp(math.log(5) + float(torch.rand((), generator=gen))
                                   * (math.log(CONTEST_MAX_SEQS) - math.log(5)))))
        lo = math.log(max(CONTEST_MIN_TOKENS, n))
        hi = math.log(CONTEST_MAX_TOKENS)
        total = int(round(math.exp(lo + float(torch.rand((), generator=gen)) * (hi - lo))))
        cases.append(split_lengths(max(total, n), n, gen))
    return cases



# ---- contest records (exact axes) --------------------------------------------
# data/contest_axes.json holds the axes of every contest workload record in the
# reference's workloads/gdn/*.md, in record order (made by data/make_contest_axes.py):
# 100 prefill records (total_seq_len, num_seqs) and 54 decode batch sizes.  The
# per-sequence lengths live in the (unavailable) safetensors blobs, so each prefill
# record is replayed with the two rewrites the reference's own scripts apply:
# "even" (total split as evenly as possible, the first total % num_seqs sequences
# one token longer: gdn_prefill/scripts/run_local_fast_even.py:31-43) and "uneven"
# (num_seqs - 1 one-token sequences, then one long sequence:
# gdn_prefill/scripts/run_local_fast_uneven.py:32-46).
_AXES_PATH = Path(__file__).resolve().parent / "data" / "contest_axes.json"


def contest_axes() -> dict:
    import json
    return json.loads(_AXES_PATH.read_text())


def even_lengths(total: int, n: int) -> list:
    base, rem = divmod(int(total), int(n))
    return [base + 1 if i < rem else base for i in range(int(n))]


def uneven_lengths(total: int, n: int) -> list:
    if total < n:
        raise ValueError(f"uneven layout needs total_seq_len >= num_seqs ({total} < {n})")
    return [1] * (int(n) - 1) + [int(total) - (int(n) - 1)]


def contest_prefill_records() -> list:
    """[(record index, split name, lengths)] for every prefill record, even then
    uneven."""
    out = []
    for i, (total, n) in enumerate(contest_axes()["prefill"]):
        out.append((i, "even", even_lengths(total, n)))
        out.append((i, "uneven", uneven_lengths(total, n)))
    return out


def contest_decode_records() -> list:
    return list(contest_axes()["decode_batch"])
