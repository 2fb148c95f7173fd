"""Generate the golden fixtures that pin the CPU oracle to the reference.

Run in a container where the reference workspace is mounted; its root
directory is the one required argument:

    python tests/golden/make_golden.py [REFERENCE_ROOT]

It extracts the PyTorch ``run`` function from the two GDN definition files
(``definitions/gdn/gdn_decode_qk4_v8_d128_k_last.md`` and
``definitions/gdn/gdn_prefill_qk4_v8_d128_k_last.md``), executes it unmodified at
the definition geometry (Hq=Hk=4, Hv=8) and with its four head-count asserts
removed at the TP=1 geometry (Hq=Hk=16, Hv=32), on seeded CPU inputs from
``gdn_b200.workloads``, and writes one compressed ``.npz`` per case.

Each fixture holds:
* ``o``: the full bf16 output (as uint16 bit patterns);
* ``state_rows`` / ``row_ids``: new_state rows [128 fp32] at seeded (n, h, v)
  positions (all rows when the tensor is at most 512 KiB);
* ``state_sum`` / ``state_sumsq``: float64 checksums of the whole new_state;
* ``input_sha``: sha256 of the generated inputs, so a drift of the generator is
  caught instead of silently comparing different problems;
* ``meta``: a JSON string with the case parameters.

Nothing on the GPU box reads the reference: the fixtures travel, this script
does not need to.
"""
from __future__ import annotations

import json
import math
import os
import re
import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
REPO = HERE.parent.parent
sys.path.insert(0, str(REPO / "mlsys-flashlinfer-contest_b200"))

from gdn_b200 import workloads as W  # noqa: E402

sys.path.insert(0, str(REPO / "tests"))
from golden_io import sha_inputs  # noqa: E402

FULL_STATE_LIMIT = 512 * 1024
SUBSET_ROWS = 256

# Cases: (name, kind, geometry (Hq, Hv), params)
CASES = [
    ("decode_def_b2", "decode", (4, 8), dict(B=2, seed=101, with_state=True)),
    ("decode_def_b1_nostate", "decode", (4, 8), dict(B=1, seed=102, with_state=False)),
    ("decode_tp1_b2", "decode", (16, 32), dict(B=2, seed=103, with_state=True)),
    ("prefill_def_varlen", "prefill", (4, 8),
     dict(lengths=[37, 0, 93, 65], seed=201, with_state=True, zero_state_every_other=True)),
    ("prefill_def_nostate", "prefill", (4, 8),
     dict(lengths=[64, 1, 130], seed=202, with_state=False)),
    ("prefill_tp1", "prefill", (16, 32),
     dict(lengths=[70, 5], seed=203, with_state=True)),
]


def extract_run(md_path: Path, lift_asserts: bool):
    text = md_path.read_text()
    m = re.search(r"```python\n(.*?)```", text, re.S)
    if m is None:
        raise RuntimeError(f"no python block in {md_path}")
    src = m.group(1)
    if lift_asserts:
        src2 = re.sub(r"^\s*assert num_(q|k|v)_heads == \d+\s*$", "", src, flags=re.M)
        assert src2.count("assert num_") == 0, "head asserts not all lifted"
        src = src2
    ns: dict = {}
    exec(compile(src, str(md_path), "exec"), ns)
    return ns["run"]


def make_inputs(kind, geom, p):
    Hq, Hv = geom
    if kind == "decode":
        return W.make_decode_inputs(p["B"], Hq, Hv, seed=p["seed"], with_state=p["with_state"])
    return W.make_prefill_inputs(p["lengths"], Hq, Hv, seed=p["seed"], with_state=p["with_state"],
                                 zero_state_every_other=p.get("zero_state_every_other", False))


def state_subset(new_state: np.ndarray, seed: int):
    rows = new_state.reshape(-1, new_state.shape[-1])
    if new_state.nbytes <= FULL_STATE_LIMIT:
        ids = np.arange(rows.shape[0], dtype=np.int64)
    else:
        rng = np.random.default_rng(seed)
        ids = np.sort(rng.choice(rows.shape[0], SUBSET_ROWS, replace=False)).astype(np.int64)
    return ids, rows[ids].astype(np.float32)


def main():
    if len(sys.argv) != 2:
        sys.exit("usage: make_golden.py REFERENCE_ROOT")
    ref_root = Path(sys.argv[1])
    dec_md = ref_root / "definitions/gdn/gdn_decode_qk4_v8_d128_k_last.md"
    pre_md = ref_root / "definitions/gdn/gdn_prefill_qk4_v8_d128_k_last.md"
    torch.set_num_threads(os.cpu_count() or 1)
    for name, kind, geom, p in CASES:
        lift = geom != (4, 8)
        run = extract_run(dec_md if kind == "decode" else pre_md, lift)
        inp = make_inputs(kind, geom, p)
        args = inp.args()
        o, new_state = run(*args)
        o_bits = o.contiguous().view(torch.int16).numpy().view(np.uint16)
        ns = new_state.numpy().astype(np.float32)
        ids, rows = state_subset(ns, p["seed"])
        meta = dict(name=name, kind=kind, Hq=geom[0], Hv=geom[1], params=p,
                    reference_file=str((dec_md if kind == "decode" else pre_md).relative_to(ref_root)),
                    asserts_lifted=lift, torch=torch.__version__)
        np.savez_compressed(
            HERE / f"{name}.npz", o=o_bits, row_ids=ids, state_rows=rows,
            state_shape=np.array(ns.shape, np.int64),
            state_sum=np.float64(ns.astype(np.float64).sum()),
            state_sumsq=np.float64((ns.astype(np.float64) ** 2).sum()),
            input_sha=np.array(sha_inputs(list(args))), meta=np.array(json.dumps(meta)))
        print(f"{name}: o{tuple(o.shape)} state{ns.shape} rows={len(ids)}")


if __name__ == "__main__":
    main()
