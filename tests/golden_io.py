"""Loading helpers for the golden fixtures in tests/golden (written by
tests/golden/make_golden.py from the reference's own definition code)."""
import json
from pathlib import Path

import numpy as np

from gdn_b200 import workloads as W

GOLDEN = Path(__file__).resolve().parent / "golden"


def names(kind=None):
    out = []
    for p in sorted(GOLDEN.glob("*.npz")):
        meta = json.loads(str(np.load(p)["meta"]))
        if kind is None or meta["kind"] == kind:
            out.append(p.stem)
    return out


def load(name):
    z = np.load(GOLDEN / f"{name}.npz")
    meta = json.loads(str(z["meta"]))
    return meta, z


def regenerate_inputs(meta, device="cpu"):
    p = meta["params"]
    if meta["kind"] == "decode":
        return W.make_decode_inputs(p["B"], meta["Hq"], meta["Hv"], seed=p["seed"],
                                    with_state=p["with_state"], device=device)
    return W.make_prefill_inputs(p["lengths"], meta["Hq"], meta["Hv"], seed=p["seed"],
                                 with_state=p["with_state"], device=device,
                                 zero_state_every_other=p.get("zero_state_every_other", False))


def check_state(new_state, z, rtol=1e-5, atol=1e-6, sum_rtol=1e-5):
    """Compare a full new_state (numpy fp32) with the fixture's rows + checksums.
    Returns the max abs row difference."""
    ns = np.asarray(new_state, np.float32)
    assert tuple(ns.shape) == tuple(z["state_shape"])
    rows = ns.reshape(-1, ns.shape[-1])[z["row_ids"]]
    np.testing.assert_allclose(rows, z["state_rows"], rtol=rtol, atol=atol)
    s = ns.astype(np.float64)
    ref_sumsq = float(z["state_sumsq"])
    assert abs(float((s ** 2).sum()) - ref_sumsq) <= sum_rtol * max(ref_sumsq, 1e-30) + 1e-9
    # the plain sum can cancel; compare it against the scale of the tensor
    assert abs(float(s.sum()) - float(z["state_sum"])) <= sum_rtol * (np.sqrt(ref_sumsq) * np.sqrt(s.size)) + 1e-9
    return float(np.abs(rows - z["state_rows"]).max()) if rows.size else 0.0


def sha_inputs(tensors) -> str:
    """sha256 over the definition-order inputs (bf16 hashed as raw bits)."""
    import hashlib
    import torch
    h = hashlib.sha256()
    for t in tensors:
        if t is None:
            h.update(b"none")
            continue
        if isinstance(t, float):
            h.update(repr(t).encode())
            continue
        t = t.detach().cpu().contiguous()
        if t.dtype == torch.bfloat16:
            t = t.view(torch.int16)
        h.update(t.numpy().tobytes())
    return h.hexdigest()
