"""Multi-kernel problems on CPU: chain validation, per-kernel meta selection, and the chained
computation evaluated by the oracle's IR interpreter."""

import numpy as np
import pytest

from emmyptx import problem, workloads
from emmyptx.meta import EmmyIRParser


def test_chain_check_accepts_meta_order_and_rejects_the_reverse():
    _, meta = workloads.chain_add_sum(1024)
    problem.check_chain(meta)
    meta["kernels"].reverse()
    with pytest.raises(ValueError, match="needs add from an earlier kernel"):
        problem.check_chain(meta)


def test_each_kernel_file_selects_its_own_meta_record(tmp_path):
    payloads, meta = workloads.chain_add_sum(1024)
    d = workloads.write_problem(tmp_path, payloads, meta)
    for k in meta["kernels"]:
        kern = EmmyIRParser(d / f"{k['entry']}.ir.json").parse()
        assert kern.name == k["entry"] and list(kern.arg_order) == k["arg_order"]


def test_chain_through_the_interpreter_matches_fp64(tmp_path):
    from oracle.expressions import seeded_input
    from oracle.ir_eval import run_kernel
    payloads, meta = workloads.chain_add_sum(4096)
    d = workloads.write_problem(tmp_path, payloads, meta)
    values = {}
    for k in meta["kernels"]:
        kern = EmmyIRParser(d / f"{k['entry']}.ir.json").parse()
        inputs = {a["name"]: values[a["name"]] if a.get("intermediate") else seeded_input(a)
                  for a in k["args"] if not a.get("output")}
        values.update(run_kernel(kern, k, inputs))
    x0 = seeded_input(meta["kernels"][0]["args"][0]).astype(np.float64)
    x1 = seeded_input(meta["kernels"][0]["args"][1]).astype(np.float64)
    want = (x0 + x1).sum()
    assert abs(float(values["sum_1"].reshape(-1)[0]) - want) <= 1e-5 * abs(want) + 1e-5
