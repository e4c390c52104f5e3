"""Parity of the emitted PTX on B200 against the oracle, through the C ABI (emmy_rt_run).

Tolerances (written here, per kernel family; the bounds themselves are in tolerance.py):
* pointwise: bit-exact (rtol = atol = 0) against numpy float32 and ``expected.npz``;
* row normalisations (RMSNorm, softmax, L2): every element within 1e-5 of the fp64 result,
  ``|got - ref| <= 1e-5 * |ref|`` (RMSNorm and L2 add an absolute floor of 1e-5 * 1e-6 *
  max|ref| only for elements below 1e-6 * max|ref|; softmax outputs are all positive and get
  none);
* sums (scalar sum and mean, row sums): every output within 1e-5 relative of fp64 as well,
  ``|got - ref| <= 1e-5 * |ref|``;
* matmul: ``|got - ref| <= 1e-4 * (|ref| + row max|ref|)``;
* every fixture also within its own meta.json rtol/atol against ``expected.npz``.
"""

import json

import numpy as np
import pytest

import tolerance as tol
from conftest import problem_dirs

pytestmark = pytest.mark.gpu

REL = 1e-5
FLOOR = 1e-6          # RMSNorm / L2: absolute floor only below this fraction of max|ref|
ROWS = ("rmsnorm", "softmax", "l2norm")


def _check(kind, got, exact, abs_sum=None, label=None):
    """The family's bound: every element within 1e-5 relative of fp64; RMSNorm and L2 have
    the small absolute floor. ``abs_sum`` (sum|x| per output of a sum) only feeds the error
    record, as the sum's condition: error / sum|x| is printed beside error / |ref|."""
    if kind in ROWS:
        return tol.elementwise(got, exact, REL, floor=None if kind == "softmax" else FLOOR,
                               label=label)
    ok, err = tol.elementwise(got, exact, REL, label=label)
    if abs_sum is not None and label is not None:
        tol.sums(got, exact, abs_sum, REL, label=label + " (error / sum|x|)")
    return ok, err


@pytest.mark.parametrize("pdir", problem_dirs(), ids=lambda p: p.name)
def test_fixture_on_gpu(pdir, gpu_runtime):
    from emmyptx.emit import compile_file
    from oracle.expressions import kernel_inputs
    meta = json.loads((pdir / "meta.json").read_text())
    expected = dict(np.load(pdir / "expected.npz"))
    fp64 = None
    for k in meta["kernels"]:
        ptx = compile_file(pdir / f"{k['entry']}.ir.json")
        outs, _ = gpu_runtime.run_kernel(ptx, k, kernel_inputs(k), iters=2)
        for name, got in outs.items():
            want = expected[name]
            got = got.reshape(want.shape)
            assert np.allclose(got, want, rtol=meta["rtol"], atol=meta["atol"]), name
            if meta["rtol"] == 0 and meta["atol"] == 0:
                assert np.array_equal(got, want)
    if meta["id"][0] in "rf":
        # stricter than the fixture tolerance: within 1e-5 of the exact result
        from oracle.expressions import problem_inputs
        args = [a.astype(np.float64) for a in problem_inputs(meta)]
        exact = _exact(meta["id"], args)
        kind = {"f01": "rmsnorm", "f02": "softmax", "f03": "l2norm"}.get(meta["id"][:3], "sum")
        abs_sum = _abs_sum(meta["id"], args)
        ok, err = _check(kind, got, exact, abs_sum, label=f"fixture {meta['id']}")
        assert ok, f"error {err:.3e} against the {kind} bound"


@pytest.mark.parametrize("pdir", problem_dirs(), ids=lambda p: p.name)
def test_fixture_through_general_walker(pdir, gpu_runtime):
    """The statement walker alone (no template) also meets every fixture's tolerance."""
    from emmyptx.emit import compile_file
    from oracle.expressions import kernel_inputs
    meta = json.loads((pdir / "meta.json").read_text())
    expected = dict(np.load(pdir / "expected.npz"))
    for k in meta["kernels"]:
        ptx = compile_file(pdir / f"{k['entry']}.ir.json", template="walker")
        outs, _ = gpu_runtime.run_kernel(ptx, k, kernel_inputs(k))
        for name, got in outs.items():
            want = expected[name]
            assert np.allclose(got.reshape(want.shape), want, rtol=meta["rtol"],
                               atol=meta["atol"]), name


def _exact(pid, args):
    x = args[0]
    if pid in ("r01_array_sum", "r02_big_sum"):
        return x.sum()
    if pid == "r03_mean":
        return x.mean()
    if pid == "r04_row_sum":
        return x.sum(-1)
    if pid == "f01_rmsnorm":
        return x / np.sqrt((x * x).mean(-1, keepdims=True) + 1e-5) * args[1]
    if pid == "f02_row_softmax":
        e = np.exp(x - x.max(-1, keepdims=True))
        return e / e.sum(-1, keepdims=True)
    if pid == "f03_l2norm":
        return x / np.sqrt((x * x).sum(-1, keepdims=True))
    raise KeyError(pid)


def _abs_sum(pid, args):
    """sum|x| behind each output of a sum fixture (None for the row normalisations)."""
    x = np.abs(args[0])
    if pid in ("r01_array_sum", "r02_big_sum"):
        return x.sum()
    if pid == "r03_mean":
        return x.mean()
    if pid == "r04_row_sum":
        return x.sum(-1)
    return None


def _workload_abs_sum(name, inputs):
    x = np.abs(inputs.get("x", inputs.get("x0")).astype(np.float64))
    return {"sum": lambda: x.sum(), "mean": lambda: x.mean(),
            "rowsum": lambda: x.sum(-1)}.get(name, lambda: None)()


def _workload_exact(name, inputs):
    x = inputs.get("x", inputs.get("x0")).astype(np.float64)
    if name == "add":
        return inputs["x0"] + inputs["x1"]           # float32, exact
    if name == "sum":
        return x.sum()
    if name == "mean":
        return x.mean()
    if name == "rmsnorm":
        return x / np.sqrt((x * x).mean(-1, keepdims=True) + 1e-6) * inputs["w"].astype(np.float64)
    if name == "softmax":
        e = np.exp(x - x.max(-1, keepdims=True))
        return e / e.sum(-1, keepdims=True)
    if name == "l2norm":
        return x / np.maximum(np.sqrt((x * x).sum(-1, keepdims=True)), 1e-12)
    if name == "rowsum":
        return x.sum(-1)
    raise KeyError(name)


@pytest.mark.parametrize("name", ["add", "sum", "mean", "rmsnorm", "softmax", "l2norm"])
def test_benchmark_workload_full_size(name, gpu_runtime):
    """Each benchmark-size workload (2^20 add, 2^26 sum/mean, 8192x4096 rows) against fp64."""
    from emmyptx import workloads
    from emmyptx.emit import compile_payload
    from oracle.expressions import kernel_inputs
    payload, meta = workloads.WORKLOADS[name]()
    ptx, template, _ = compile_payload(payload, meta)
    k = meta["kernels"][0]
    inputs = kernel_inputs(k)
    outs, _ = gpu_runtime.run_kernel(ptx, k, inputs, iters=2)
    got = list(outs.values())[0]
    exact = _workload_exact(name, inputs)
    if name == "add":
        assert template == "pointwise"
        assert np.array_equal(got, exact)
    else:
        ok, err = _check(name, got, exact, _workload_abs_sum(name, inputs),
                         label=f"config {name}")
        assert ok, f"{name}: error {err:.3e} against its bound"


@pytest.mark.parametrize("case", [
    ("sum", dict(n=1, grid=4)), ("sum", dict(n=3, grid=1)), ("sum", dict(n=1023, grid=7)),
    ("sum", dict(n=(1 << 20) + 5, grid=300)), ("mean", dict(n=777, grid=2)),
])
def test_full_reduce_ragged_and_tiny(case, gpu_runtime):
    """Ragged tails, more CTAs than elements, a single element: the cross-CTA finish stays exact."""
    from emmyptx import workloads
    from emmyptx.emit import compile_payload
    from oracle.expressions import kernel_inputs
    op, kw = case
    payload, meta = workloads.full_reduce(kw["n"], op, grid=kw["grid"])
    ptx, _, _ = compile_payload(payload, meta)
    k = meta["kernels"][0]
    inputs = kernel_inputs(k)
    for _ in range(2):                       # the ticket must reset itself between launches
        outs, _ = gpu_runtime.run_kernel(ptx, k, inputs, iters=3)
        exact = _workload_exact(op, inputs)
        ok, err = _check(op, list(outs.values())[0], exact, _workload_abs_sum(op, inputs),
                         label=f"{op} ragged/tiny")
        assert ok, err


@pytest.mark.parametrize("kind, rows, cols, block", [
    ("softmax", 3, 100, 128),      # ragged row, threads without elements (validity tracking)
    ("softmax", 5, 4096, 256), ("rmsnorm", 7, 1000, 64), ("l2norm", 2, 12, 32),
    ("rowsum", 9, 2048, 96), ("softmax", 4, 16384, 512),
])
def test_row_ops_shapes(kind, rows, cols, block, gpu_runtime):
    from emmyptx import workloads
    from emmyptx.emit import compile_payload
    from oracle.expressions import kernel_inputs
    from oracle.ir_eval import run_kernel as oracle_run
    payload, meta = workloads.row_op(kind, rows=rows, cols=cols, block=block)
    ptx, template, kernel = compile_payload(payload, meta)
    assert template == "rowreduce"
    k = meta["kernels"][0]
    inputs = kernel_inputs(k)
    outs, _ = gpu_runtime.run_kernel(ptx, k, inputs)
    got = list(outs.values())[0]
    ok, err = _check(kind, got, _workload_exact(kind, inputs), _workload_abs_sum(kind, inputs),
                     label=f"{kind} shapes")
    assert ok, f"error {err:.3e} against the {kind} bound"
    # The IR's literal schedule gives every one of its `block` threads a partial state; when
    # some own no element, folding two empty softmax states is -inf - -inf = NaN in the IR
    # itself. The interpreter reproduces that, so it is only a reference when cols >= block.
    if rows * cols <= 1 << 14 and cols >= block:
        want = list(oracle_run(kernel, k, inputs).values())[0]
        ok, err = _check(kind, got, want, _workload_abs_sum(kind, inputs))
        assert ok, f"vs interpreter {err:.3e}"


def test_misaligned_pointers_take_the_scalar_path(gpu_runtime):
    """Buffers offset by 4 bytes (not 16-byte aligned) still give exact pointwise results."""
    from emmyptx import workloads
    from emmyptx.emit import compile_payload
    payload, meta = workloads.pointwise_add(1000)
    ptx, _, _ = compile_payload(payload, meta)
    k = meta["kernels"][0]
    rt = gpu_runtime
    n = 1000
    rng = np.random.default_rng(3)
    a = rng.standard_normal(n).astype(np.float32)
    b = rng.standard_normal(n).astype(np.float32)
    bufs = [rt.DeviceBuffer(4 * (n + 4)) for _ in range(3)]
    for buf, arr in zip(bufs[:2], (a, b)):
        buf.upload(np.concatenate([np.zeros(1, np.float32), arr, np.zeros(3, np.float32)]))
    bufs[2].zero()
    mod = rt.Module(ptx, k["entry"])
    mod.launch(k["grid"], k["block"], 0, [bufs[0].ptr + 4, bufs[1].ptr + 4, bufs[2].ptr + 4])
    rt.sync()
    out = np.zeros(n + 4, np.float32)
    bufs[2].download(out)
    assert np.array_equal(out[1:n + 1], a + b)
    assert out[0] == 0 and np.all(out[n + 1:] == 0)


MATMUL_REL = 1e-4


@pytest.mark.parametrize("name", ["matmul_sq", "matmul_rect"])
def test_matmul_full_size_3xtf32(name, gpu_runtime):
    """4096^3 and 8192x2048x4096 on tcgen05 (3xTF32): within 1e-4 of the fp64 product."""
    from emmyptx import workloads
    from emmyptx.emit import compile_payload
    from oracle.expressions import kernel_inputs
    payload, meta = workloads.WORKLOADS[name]()
    ptx, template, _ = compile_payload(payload, meta)
    assert template == "contraction"
    k = meta["kernels"][0]
    inputs = kernel_inputs(k)
    outs, _ = gpu_runtime.run_kernel(ptx, k, inputs)
    got = outs["matmul"]
    exact = inputs["x0"].astype(np.float64) @ inputs["x1"].astype(np.float64)
    ok, err = tol.rowscaled(got, exact, MATMUL_REL, label=f"config {name}")
    assert ok, f"error {err:.3e} of the row maximum"      # plain TF32 would be ~1e-3 here


@pytest.mark.parametrize("shape", [(256, 256, 128, 2), (512, 512, 256, 2), (768, 512, 128, 3),
                                   (1024, 256, 64, 4), (4096, 4096, 64, 4),
                                   (512, 512, 128, 4, 128), (768, 768, 64, 4, 128)])
def test_matmul_cta_pairs(shape, gpu_runtime):
    """CTA-pair form (cta_group::2): one cluster walking two tiles, four clusters with two
    each, BN 256 with two and three stages; 4096 x 4096 x 64 with 74 working clusters (the
    rest leave at once) doing 222 whole tiles and 68 half-width units; 512^2 and 768^2 with
    128-wide IR tiles, made of half-width units only. Within 1e-4 of fp64, error word 0
    (run_kernel raises on a bounded wait that expired)."""
    from emmyptx import workloads
    from emmyptx.emit import compile_payload
    from oracle.expressions import kernel_inputs
    M, N, K, S = shape[:4]
    kw = {"TN": shape[4], "RN": 8} if len(shape) > 4 else {}
    payload, meta = workloads.matmul(M, N, K, S=S, **kw)
    ptx, template, _ = compile_payload(payload, meta)
    assert template == "contraction" and ".reqnctapercluster 2, 1, 1" in ptx
    k = meta["kernels"][0]
    inputs = kernel_inputs(k)
    got = gpu_runtime.run_kernel(ptx, k, inputs)[0]["matmul"]
    exact = inputs["x0"].astype(np.float64) @ inputs["x1"].astype(np.float64)
    ok, err = tol.rowscaled(got, exact, MATMUL_REL, label="matmul CTA pairs")
    assert ok, err


@pytest.mark.parametrize("shape", [(128, 256, 64, 3), (256, 512, 96, 2), (384, 256, 256, 4)])
def test_matmul_template_matches_walker_and_interpreter(shape, gpu_runtime):
    """Small matmuls: tcgen05 template vs the statement walker vs the interpreter."""
    from emmyptx import workloads
    from emmyptx.emit import compile_payload
    from oracle.expressions import kernel_inputs
    from oracle.ir_eval import run_kernel as oracle_run
    M, N, K, S = shape
    payload, meta = workloads.matmul(M, N, K, S=S)
    k = meta["kernels"][0]
    inputs = kernel_inputs(k)
    ptx_tc, t_tc, kernel = compile_payload(payload, meta, template="contraction")
    ptx_w, t_w, _ = compile_payload(payload, meta, template="walker")
    assert (t_tc, t_w) == ("contraction", "walker")
    got_tc = gpu_runtime.run_kernel(ptx_tc, k, inputs)[0]["matmul"]
    got_w = gpu_runtime.run_kernel(ptx_w, k, inputs)[0]["matmul"]
    exact = inputs["x0"].astype(np.float64) @ inputs["x1"].astype(np.float64)
    for got, tag in ((got_tc, "tcgen05"), (got_w, "walker")):
        ok, err = tol.rowscaled(got, exact, MATMUL_REL, label=f"matmul small {tag}")
        assert ok, err
    if M * N <= 128 * 256:
        want = oracle_run(kernel, k, inputs)["matmul"]
        ok, err = tol.rowscaled(got_tc, want, MATMUL_REL)
        assert ok, err


@pytest.mark.parametrize("shape", [(1024, 1024, 4096, 4), (384, 512, 3072, 3),
                                   (640, 256, 2048, 2)],
                         ids=["pairs-4way", "single-3way", "single-2way"])
def test_matmul_split_k_atomic_epilogue(shape, gpu_runtime):
    """Split-K IR in the m02 fixture's form (a K-split Tile axis, atomic writes, the output in
    ``zero_outputs``) above the tcgen05 threshold: the template computes each output tile
    over the whole K once and adds it with red.global.add.f32 into the zeroed output. Run
    through emmy_rt_run for three launches, so the runner's re-zeroing between launches is
    part of the check (a missing zero would double the result); within 1e-4 of fp64, for
    the CTA-pair and the single-CTA forms."""
    from emmyptx import workloads
    from emmyptx.emit import compile_payload
    from oracle.expressions import kernel_inputs
    M, N, K, splits = shape
    payload, meta = workloads.matmul(M, N, K, splits=splits)
    k = meta["kernels"][0]
    assert k["zero_outputs"] == ["matmul"] and k["grid"][0] == splits * (M // 128) * (N // 256)
    ptx, template, _ = compile_payload(payload, meta, template="contraction")
    assert template == "contraction" and "red.global.add.f32" in ptx
    assert (".reqnctapercluster 2, 1, 1" in ptx) == (M % 256 == 0)
    inputs = kernel_inputs(k)
    got = gpu_runtime.run_kernel(ptx, k, inputs, iters=3)[0]["matmul"]
    exact = inputs["x0"].astype(np.float64) @ inputs["x1"].astype(np.float64)
    ok, err = tol.rowscaled(got, exact, MATMUL_REL, label="matmul split-K atomic")
    assert ok, f"error {err:.3e} of the row maximum"
