"""Solution entry point for gdn_prefill_qk4_v8_d128_k_last: the harness imports this
module and calls run(q, k, v, state, A_log, a, dt_bias, b, cu_seqlens, scale) in
definition input order, expecting (output, new_state).  The gdn_b200 package sits
two levels up (mlsys-flashlinfer-contest_b200/); its CUDA library must be built
(mlsys-flashlinfer-contest_b200/build.py)."""
import sys
from pathlib import Path

_PKG_ROOT = str(Path(__file__).resolve().parents[2])
if _PKG_ROOT not in sys.path:
    sys.path.insert(0, _PKG_ROOT)

from gdn_b200.prefill import run  # noqa: E402,F401
