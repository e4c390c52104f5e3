"""Attention on B200: the tcgen05 flash template against the fp64 oracle, through the C ABI.

Tolerance (written here): |got - ref| <= 1e-4 * |ref| + 1e-4 * max_row|ref| against
``softmax(q @ kt / c) @ v`` computed in float64 (3xTF32 products, f32 softmax), the maximum
taken over each query row's output vector (tests/tolerance.py:rowscaled).
"""

import numpy as np
import pytest

import tolerance as tol

pytestmark = pytest.mark.gpu

REL = 1e-4


def _close(got, ref, rel=REL, label=None):
    return tol.rowscaled(got, ref, rel, label=label)


def _ref_heads(inputs, heads):
    from oracle.expressions import _attention
    c = float(inputs["div_c1"][0])
    out = []
    for b, h in heads:
        out.append(_attention(inputs["q"][b, h], inputs["kt"][b, h], inputs["v"][b, h], c))
    return np.stack(out)


def _run(gpu_runtime, payload, meta, template=None, grid=None):
    from emmyptx.emit import compile_payload
    from oracle.expressions import kernel_inputs
    k = dict(meta["kernels"][0])
    if grid is not None:
        k["grid"] = [grid, 1, 1]
        meta = dict(meta, kernels=[k])
    ptx, used, _ = compile_payload(payload, meta, template=template)
    inputs = kernel_inputs(meta["kernels"][0])
    outs, _ = gpu_runtime.run_kernel(ptx, k, inputs)
    return used, inputs, outs["matmul_1"]


@pytest.mark.parametrize("name", ["attention_d128", "attention_d64"])
def test_attention_full_size(name, gpu_runtime):
    """[8,16,2048,D] on tcgen05: all 8 x 16 heads within 1e-4 of fp64 (the fp64 result is
    computed one batch entry, 16 heads, at a time)."""
    from emmyptx import workloads
    from oracle.expressions import _attention
    payload, meta = workloads.WORKLOADS[name]()
    used, inputs, got = _run(gpu_runtime, payload, meta)
    assert used == "attention"
    assert np.all(np.isfinite(got))
    c = float(inputs["div_c1"][0])
    for b in range(got.shape[0]):
        want = _attention(inputs["q"][b], inputs["kt"][b], inputs["v"][b], c)
        ok, err = _close(got[b], want, label=f"config {name}")
        assert ok, f"batch entry {b}: error {err:.3e} of the row maximum"


@pytest.mark.parametrize("shape", [(1, 2, 256, 128, None), (2, 1, 384, 64, None),
                                   (1, 1, 512, 128, 0.25), (1, 2, 256, 64, 0.125),
                                   (2, 4, 1024, 32, None), (1, 2, 256, 32, 0.125),
                                   (2, 2, 512, 96, None), (1, 1, 256, 96, 0.25)],
                         ids=["d128", "d64", "d128-peaked", "d64-peaked", "d32", "d32-peaked",
                              "d96", "d96-peaked"])
def test_attention_template_matches_fp64_and_walker(shape, gpu_runtime):
    """Small shapes: template and statement walker both within 1e-4 of fp64. A small divisor
    c makes the logits large, so the running maximum moves between key blocks and the
    rescaling of the row sum and the output accumulator is exercised. D = 96 takes an IR with
    two stages (three would ask for more than 227 KiB of shared memory)."""
    from emmyptx import workloads
    B, H, S, D, c = shape
    payload, meta = workloads.attention(B, H, S, D, scale=c, stages=2 if D == 96 else 3)
    used, inputs, got = _run(gpu_runtime, payload, meta)
    assert used == "attention"
    heads = [(b, h) for b in range(B) for h in range(H)]
    want = _ref_heads(inputs, heads).reshape(got.shape)
    ok, err = _close(got, want, label="attention small tcgen05")
    assert ok, f"template relative error {err:.3e}"
    used_w, _, got_w = _run(gpu_runtime, payload, meta, template="walker")
    assert used_w == "walker"
    ok, err = _close(got_w, want, label="attention small walker")
    assert ok, f"walker relative error {err:.3e}"


@pytest.mark.parametrize("grid", [1, 5])
def test_attention_grid_stride_over_work_items(grid, gpu_runtime):
    """Fewer CTAs than (head, query block) items: each CTA walks several items and the
    mbarrier phases carry across them."""
    from emmyptx import workloads
    payload, meta = workloads.attention(2, 2, 384, 128)
    used, inputs, got = _run(gpu_runtime, payload, meta, grid=grid)
    assert used == "attention"
    heads = [(b, h) for b in range(2) for h in range(2)]
    ok, err = _close(got, _ref_heads(inputs, heads).reshape(got.shape))
    assert ok, f"relative error {err:.3e}"


@pytest.mark.parametrize("form,args,grid", [
    ("rows", (300, 32), None),        # 2 full chunks of 128 keys + a 44-key tail
    ("rows", (33, 64), None),         # one 33-key chunk: second slot has a single key
    ("rows", (200, 96), None),        # three output columns per lane
    ("rows", (16, 160), None),        # 16 keys, five columns per lane
    ("rows", (128, 32), 7),           # 7 warps walk 128 rows
    ("tiled", (1, 2, 256, 48), None),  # D = 48: a partial group of output columns
    ("tiled", (2, 1, 128, 80), 3),
    ("tiled", (1, 1, 128, 160), 1000),  # more warps than rows
], ids=lambda v: str(v))
def test_attention_warp_template_matches_fp64(form, args, grid, gpu_runtime):
    """The CUDA-core attention (one warp per query row) for the shapes and launches the
    tcgen05 template declines, within 1e-4 of fp64, under the IR's own geometry and others."""
    from emmyptx import workloads
    from oracle.expressions import _attention
    if form == "rows":
        payload, meta = workloads.attention_rows(*args)
    else:       # two stages: the IR's shared-memory request stays within the 227 KiB limit
        payload, meta = workloads.attention(*args, stages=2)
    used, inputs, got = _run(gpu_runtime, payload, meta, grid=grid)
    assert used == "attention_warp"
    c = float(inputs["div_c1"][0])
    if form == "rows":
        want = _attention(inputs["q"], inputs["kt"], inputs["v"], c)
    else:
        B, H = args[0], args[1]
        want = _ref_heads(inputs, [(b, h) for b in range(B) for h in range(H)])
    ok, err = _close(got, np.asarray(want).reshape(got.shape), label="attention warp-per-row")
    assert ok, f"relative error {err:.3e}"
