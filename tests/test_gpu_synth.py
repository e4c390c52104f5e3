"""Synthesized IR (emmyptx/synth.py) on a B200 against the oracle.

Tolerances (written here): pointwise DAGs of correctly rounded ops bit-exact against the
interpreter (numpy float32); DAGs with approximate ops (ex2/lg2/rsqrt/tanh) within
1e-4 * |ref| + 1e-5 * max|ref| with identical non-finite positions; rows and reductions
every element within 1e-5 relative of fp64 (RMSNorm and L2 with an absolute floor of 1e-5 *
1e-6 * max|ref| below 1e-6 * max|ref|); matmul and attention within 1e-4 * (|ref| + row
max|ref|) of fp64 (template and walker cases alike). The bounds are in tolerance.py.
"""

import numpy as np
import pytest

import tolerance as tol
from test_synth import _fp64

pytestmark = pytest.mark.gpu

# seeds per test by default; ``pytest --synth-seeds N`` runs N seeds of every family
DEFAULT_SEEDS = {"test_pointwise": 40, "test_rows_and_reductions": 40, "test_contraction": 40,
                 "test_contraction_template": 32, "test_contraction_ragged_edges": 24,
                 "test_attention": 24}


def pytest_generate_tests(metafunc):
    if "seed" in metafunc.fixturenames:
        n = metafunc.config.getoption("synth_seeds") or DEFAULT_SEEDS[metafunc.function.__name__]
        metafunc.parametrize("seed", range(n))


def _close(got, ref, rel, label=None):
    return tol.rowscaled(got, ref, rel, label=label)[0]


def _close_rows(info, got, ref):
    kind = info.get("kind", info.get("op"))
    floor = 1e-6 if kind in ("rmsnorm", "l2norm") else None
    return tol.elementwise(got, ref, 1e-5, floor=floor, label=f"synth {kind}")[0]


def test_pointwise(seed, gpu_runtime):
    from emmyptx import synth
    from emmyptx.emit import compile_payload
    from oracle.expressions import kernel_inputs
    from oracle.ir_eval import run_kernel
    payload, meta, info = synth.pointwise(seed)
    k = meta["kernels"][0]
    ptx, template, kernel = compile_payload(payload, meta)
    assert template == "pointwise"
    inputs = kernel_inputs(k)
    got = gpu_runtime.run_kernel(ptx, k, inputs)[0]["out"]
    want = run_kernel(kernel, k, inputs)["out"]
    if info["exact"]:
        assert np.array_equal(got, want, equal_nan=True), info
        return
    fin = np.isfinite(want)
    assert np.array_equal(np.isfinite(got), fin), info
    assert np.array_equal(got[~fin], want[~fin], equal_nan=True), info
    g, w = got[fin].astype(np.float64), want[fin].astype(np.float64)
    scale = float(np.max(np.abs(w))) if w.size else 0.0
    assert np.all(np.abs(g - w) <= 1e-4 * np.abs(w) + 1e-5 * scale), info


def test_rows_and_reductions(seed, gpu_runtime):
    from emmyptx import synth
    from emmyptx.emit import compile_payload
    from oracle.expressions import kernel_inputs
    for payload, meta, info in (synth.rows(seed), synth.reduction(seed)):
        k = meta["kernels"][0]
        ptx, template, _ = compile_payload(payload, meta)
        inputs = kernel_inputs(k)
        (out,) = meta["graph_outputs"]
        got = gpu_runtime.run_kernel(ptx, k, inputs)[0][out]
        assert _close_rows(info, got, _fp64(info, inputs)), (template, info)


def test_contraction(seed, gpu_runtime):
    from emmyptx import synth
    from emmyptx.emit import compile_payload
    from oracle.expressions import kernel_inputs
    payload, meta, info = synth.contraction(seed)
    k = meta["kernels"][0]
    ptx, template, _ = compile_payload(payload, meta)
    inputs = kernel_inputs(k)
    got = gpu_runtime.run_kernel(ptx, k, inputs)[0]["matmul"]
    want = inputs["x0"].astype(np.float64) @ inputs["x1"].astype(np.float64)
    assert _close(got, want, 1e-4, label=f"synth matmul {template}"), (template, info)


def test_contraction_template(seed, gpu_runtime):
    """Random shapes inside the tcgen05 template's conditions with the template forced: CTA
    pairs, single CTAs, several tiles per CTA or cluster, half-width units; error word 0
    (run_kernel raises otherwise) and within 1e-4 of fp64."""
    from emmyptx import synth
    from emmyptx.emit import compile_payload
    from oracle.expressions import kernel_inputs
    payload, meta, info = synth.contraction_tc(seed)
    k = meta["kernels"][0]
    ptx, template, _ = compile_payload(payload, meta, template="contraction")
    inputs = kernel_inputs(k)
    got = gpu_runtime.run_kernel(ptx, k, inputs)[0]["matmul"]
    want = inputs["x0"].astype(np.float64) @ inputs["x1"].astype(np.float64)
    assert _close(got, want, 1e-4, label="synth matmul tcgen05 forced"), info


def test_contraction_ragged_edges(seed, gpu_runtime):
    """Shapes that are not multiples of the tcgen05 tile (M of 128, N of the tile width, K of
    32) on the template, with the edge tiles masked: zero-filled loads past the matrix, no
    stores past it; every seed is also run twice in a row (stale shared memory from the
    previous tile would show). Within 1e-4 of fp64, error word 0."""
    from emmyptx import synth
    from emmyptx.emit import compile_payload
    from oracle.expressions import kernel_inputs
    payload, meta, info = synth.contraction_ragged(seed)
    k = meta["kernels"][0]
    ptx, template, _ = compile_payload(payload, meta, template="contraction")
    assert template == "contraction"
    inputs = kernel_inputs(k)
    got = gpu_runtime.run_kernel(ptx, k, inputs, iters=2)[0]["matmul"]
    want = inputs["x0"].astype(np.float64) @ inputs["x1"].astype(np.float64)
    assert _close(got, want, 1e-4, label="synth matmul ragged tcgen05"), info


def test_attention(seed, gpu_runtime):
    from emmyptx import synth
    from emmyptx.emit import compile_payload
    from oracle.expressions import _attention, kernel_inputs
    payload, meta, info = synth.attention(seed)
    k = meta["kernels"][0]
    ptx, template, _ = compile_payload(payload, meta)
    inputs = kernel_inputs(k)
    got = gpu_runtime.run_kernel(ptx, k, inputs)[0]["matmul_1"]
    want = _attention(inputs["q"], inputs["kt"], inputs["v"], float(inputs["div_c1"][0]))
    assert _close(got, want, 1e-4, label=f"synth attention {template}"), (template, info)
