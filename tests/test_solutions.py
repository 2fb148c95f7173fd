"""The flashinfer-bench Solution packs under mlsys-flashlinfer-contest_b200/solutions/:
each directory holds a config.toml with the reference's keys (gdn_decode/config.toml,
gdn_prefill/config.toml: [solution] name / definition, [build] language = "python",
entry_point = "<file>.py::run", destination_passing_style = false) and the entry
module it names, which the harness imports by path and calls with the definition's
inputs in order.  CPU: the configs, the entry files and run's parameter order.  GPU:
one small call through each entry module against the C oracle."""
import importlib.util
import inspect
import tomllib
from pathlib import Path

import pytest
import torch

import parity as PT
from oracle import c_oracle as C
from gdn_b200 import workloads as W

SOL = Path(__file__).resolve().parents[1] / "mlsys-flashlinfer-contest_b200" / "solutions"
PACKS = {
    "gdn_decode": ("gdn_decode_qk4_v8_d128_k_last",
                   ["q", "k", "v", "state", "A_log", "a", "dt_bias", "b", "scale"]),
    "gdn_prefill": ("gdn_prefill_qk4_v8_d128_k_last",
                    ["q", "k", "v", "state", "A_log", "a", "dt_bias", "b", "cu_seqlens", "scale"]),
}


def _load(pack):
    cfg = tomllib.loads((SOL / pack / "config.toml").read_text())
    fname, fn = cfg["build"]["entry_point"].split("::")
    spec = importlib.util.spec_from_file_location(f"_solution_{pack}", SOL / pack / fname)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return cfg, getattr(mod, fn)


@pytest.mark.parametrize("pack", sorted(PACKS))
def test_solution_config_and_entry(pack):
    cfg, run = _load(pack)
    definition, inputs = PACKS[pack]
    assert cfg["solution"]["definition"] == definition
    assert cfg["build"]["language"] == "python"
    assert cfg["build"]["destination_passing_style"] is False
    params = [p.name for p in inspect.signature(run).parameters.values()
              if p.default is inspect.Parameter.empty]
    assert params == inputs


@pytest.mark.gpu
def test_decode_solution_runs():
    _, run = _load("gdn_decode")
    inp = W.make_decode_inputs(4, 4, 8, seed=3)
    o_ref, s_ref = C.decode(*inp.args())
    o, ns = run(*PT.to_device(inp).args())
    torch.cuda.synchronize()
    PT.assert_o_close(o, o_ref)
    PT.assert_state_close(ns, s_ref, PT.STATE_RTOL_FP32)


@pytest.mark.gpu
def test_prefill_solution_runs():
    _, run = _load("gdn_prefill")
    inp = W.make_prefill_inputs([300, 77], 4, 8, seed=4)
    o_ref, s_ref = C.prefill(*inp.args())
    o, ns = run(*PT.to_device(inp).args())
    torch.cuda.synchronize()
    PT.assert_o_close(o, o_ref)
    PT.assert_state_close(ns, s_ref, PT.STATE_REL)
