"""Whole problems through emmyptx.problem.run_problem on a B200: a two-kernel chain whose
intermediate stays in device memory, and every fixture folder against its expected.npz."""

import json

import numpy as np
import pytest

from conftest import problem_dirs

pytestmark = pytest.mark.gpu


def test_two_kernel_chain_on_the_gpu(tmp_path, gpu_runtime):
    from emmyptx import problem, workloads
    from emmyptx.inputs import seeded_input
    payloads, meta = workloads.chain_add_sum(1 << 20)
    d = workloads.write_problem(tmp_path, payloads, meta)
    out = problem.run_problem(d)
    assert all(v == 0 for v in out["_error_words"].values())
    x0 = seeded_input(meta["kernels"][0]["args"][0]).astype(np.float64)
    x1 = seeded_input(meta["kernels"][0]["args"][1]).astype(np.float64)
    want = (x0 + x1).sum()
    got = float(out["sum_1"].reshape(-1)[0])
    assert abs(got - want) <= 1e-5 * abs(want) + 1e-5


@pytest.mark.parametrize("pdir", problem_dirs(), ids=lambda p: p.name)
def test_fixture_problem_runner(pdir, gpu_runtime):
    from emmyptx import problem
    meta = json.loads((pdir / "meta.json").read_text())
    out = problem.run_problem(pdir)
    expected = np.load(pdir / "expected.npz")
    for name in meta["graph_outputs"]:
        want = expected[name]
        got = out[name].reshape(want.shape)
        assert np.allclose(got, want, rtol=meta["rtol"], atol=meta["atol"]), name
