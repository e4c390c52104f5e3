"""Our PTX against the reference compiler's own PTX, both JIT-run on the same B200 through
the C ABI, on the same seeded inputs.

The reference PTX (``.target sm_89``, JIT-compiled by the driver for sm_100a) comes from the
reference ``compile.py`` itself (``tests/golden/make_ref_ptx.py``), for every fixture and for
each benchmark configuration in the form the reference's lowerers accept (grid 1 for the
scalar sum, 128-thread row kernels, the rank-2 attention slice).

Tolerances (written here): pointwise bit-exact; reductions and row operations
|ours - ref| <= 1e-5 * |ref| + 1e-5 * max|ref|; matmul and attention the same with 1e-4. The
reference output is itself checked against the fp64 oracle with the same bound, so a
disagreement points at one side. Both compilers' outputs carry their own f32 rounding (the
reference's grid-1 sum adds 2^18 terms per thread in sequence), so the two are compared in
this max-scaled form; the element-wise bounds against fp64 that our kernels are held to are in
test_gpu_parity.py and test_gpu_attention.py.
"""

import json
from pathlib import Path

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

GOLDEN = Path(__file__).resolve().parent / "golden"
ENTRIES = json.loads((GOLDEN / "ref_ptx" / "MANIFEST.json").read_text())["entries"]
FIXTURES = sorted(n for n, e in ENTRIES.items() if e["source"] == "fixture")
CONFIGS = sorted(n for n, e in ENTRIES.items() if e["source"] == "workload")


def _rel(name):
    return {"p": 0.0, "r": 1e-5, "f": 1e-5, "m": 1e-4, "a": 1e-4}[name[0]]


def _close(got, ref, rel):
    ref = np.asarray(ref, dtype=np.float64)
    got = np.asarray(got, dtype=np.float64).reshape(ref.shape)
    scale = float(np.max(np.abs(ref)))
    ok = np.abs(got - ref) <= rel * np.abs(ref) + rel * scale
    return bool(np.all(ok)), float(np.max(np.abs(got - ref)) / max(scale, 1e-30))


def _ref_ptx(name):
    return (GOLDEN / "ref_ptx" / f"{name}.ptx").read_text()


@pytest.mark.parametrize("pid", FIXTURES)
def test_fixture_ours_matches_reference_ptx(pid, gpu_runtime):
    from emmyptx.emit import compile_file
    from oracle.expressions import kernel_inputs, reference_outputs
    pdir = GOLDEN / "problems" / pid
    meta = json.loads((pdir / "meta.json").read_text())
    k = meta["kernels"][0]
    inputs = kernel_inputs(k)
    ours = gpu_runtime.run_kernel(compile_file(sorted(pdir.glob("*.ir.json"))[0]), k, inputs)[0]
    ref = gpu_runtime.run_kernel(_ref_ptx(pid), k, inputs)[0]
    exact = reference_outputs(meta)
    for out in meta["graph_outputs"]:
        if pid.startswith("p"):
            assert np.array_equal(ours[out], ref[out]), "pointwise must match bit for bit"
        else:
            ok, err = _close(ours[out], ref[out], _rel(pid))
            assert ok, f"ours vs reference PTX: {err:.3e}"
        ok, err = _close(ref[out], exact[out], max(_rel(pid), meta["rtol"]))
        assert ok, f"reference PTX vs fp64: {err:.3e}"


@pytest.mark.parametrize("name", [n for n in CONFIGS if not n.startswith("attention")])
def test_config_ours_matches_reference_ptx(name, gpu_runtime):
    """The benchmark workload (our IR and launch) against the reference compiler's PTX of the
    same computation in its accepted form, at the full configuration size."""
    from emmyptx import workloads
    from emmyptx.emit import compile_payload
    from oracle.expressions import kernel_inputs
    e = ENTRIES[name]
    fn, args, kwargs = e["call"]
    _, ref_meta = getattr(workloads, fn)(*args, **kwargs)
    payload, meta = workloads.WORKLOADS[e["mirrors"]]()
    k, kr = meta["kernels"][0], ref_meta["kernels"][0]
    inputs = kernel_inputs(k)
    ref_inputs = kernel_inputs(kr)
    for a in kr["args"]:
        if not a.get("output") and a["name"] in inputs:
            assert np.array_equal(ref_inputs[a["name"]], inputs[a["name"]])
    ptx, _, _ = compile_payload(payload, meta)
    ours = gpu_runtime.run_kernel(ptx, k, inputs)[0]
    ref = gpu_runtime.run_kernel(_ref_ptx(name), kr, ref_inputs)[0]
    (out,) = meta["graph_outputs"]
    (rout,) = ref_meta["graph_outputs"]
    rel = {"add": 0.0, "matmul_sq": 1e-4, "matmul_rect": 1e-4}.get(name, 1e-5)
    if rel == 0.0:
        assert np.array_equal(ours[out], ref[rout])
    else:
        ok, err = _close(ours[out], ref[rout], rel)
        assert ok, f"ours vs reference PTX: {err:.3e}"


@pytest.mark.parametrize("name", [n for n in CONFIGS if n.startswith("attention")])
def test_attention_ours_matches_reference_ptx_per_head(name, gpu_runtime):
    """[8,16,2048,D] on the tcgen05 template against the reference PTX run on single
    (batch, head) slices (its rank-2 form) for two heads."""
    from emmyptx import workloads
    from emmyptx.emit import compile_payload
    from oracle.expressions import kernel_inputs
    e = ENTRIES[name]
    fn, args, kwargs = e["call"]
    _, ref_meta = getattr(workloads, fn)(*args, **kwargs)
    payload, meta = workloads.WORKLOADS[e["mirrors"]]()
    k, kr = meta["kernels"][0], ref_meta["kernels"][0]
    inputs = kernel_inputs(k)
    ptx, used, _ = compile_payload(payload, meta)
    assert used == "attention"
    ours = gpu_runtime.run_kernel(ptx, k, inputs)[0]["matmul_1"]
    for b, h in ((0, 0), (7, 15)):
        head = {"div_c1": inputs["div_c1"], "q": inputs["q"][b, h].copy(),
                "kt": inputs["kt"][b, h].copy(), "v": inputs["v"][b, h].copy()}
        ref = gpu_runtime.run_kernel(_ref_ptx(name), kr, head)[0]["matmul_1"]
        ok, err = _close(ours[b, h], ref, 1e-4)
        assert ok, f"head ({b},{h}) ours vs reference PTX: {err:.3e}"
