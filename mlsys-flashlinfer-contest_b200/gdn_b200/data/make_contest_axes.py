"""Extract the shape axes of the contest workloads into contest_axes.json.

The reference lists the contest's GDN workloads in
``workloads/gdn/gdn_prefill_qk4_v8_d128_k_last.md`` (100 records) and
``workloads/gdn/gdn_decode_qk4_v8_d128_k_last.md`` (54 records).  Each record
names a safetensors blob (not available offline) and its axes.  Only the axes
are kept here, in record order: (total_seq_len, num_seqs) per prefill record and
batch_size per decode record; the replay feeds seeded synthetic tensors of those
shapes to the kernels.  Run where the reference tree is mounted:

    python mlsys-flashlinfer-contest_b200/gdn_b200/data/make_contest_axes.py REFERENCE_ROOT
"""
import json
import re
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent


def axes(md: Path, names):
    text = md.read_text()
    records = re.split(r"^## Record \d+:", text, flags=re.M)[1:]
    out = []
    for rec in records:
        vals = {}
        for name in names:
            m = re.search(r"\|\s*`%s`\s*\|\s*`(\d+)`\s*\|" % name, rec)
            if m is None:
                raise ValueError(f"axis {name} missing in a record of {md.name}")
            vals[name] = int(m.group(1))
        out.append(vals)
    return out


def main():
    if len(sys.argv) != 2:
        sys.exit("usage: make_contest_axes.py REFERENCE_ROOT")
    root = Path(sys.argv[1])
    pre = axes(root / "workloads/gdn/gdn_prefill_qk4_v8_d128_k_last.md", ("total_seq_len", "num_seqs"))
    dec = axes(root / "workloads/gdn/gdn_decode_qk4_v8_d128_k_last.md", ("batch_size",))
    data = {
        "source": "workloads/gdn/gdn_{prefill,decode}_qk4_v8_d128_k_last.md (axes only, record order)",
        "geometry": {"num_q_heads": 4, "num_k_heads": 4, "num_v_heads": 8, "head_size": 128},
        "prefill": [[r["total_seq_len"], r["num_seqs"]] for r in pre],
        "decode_batch": [r["batch_size"] for r in dec],
    }
    (HERE / "contest_axes.json").write_text(json.dumps(data, indent=0) + "\n")
    print(f"{len(pre)} prefill and {len(dec)} decode records")


if __name__ == "__main__":
    main()
