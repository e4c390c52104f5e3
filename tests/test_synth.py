"""Synthesized IR beyond the fixtures (emmyptx/synth.py), on CPU: every case lowers and its
PTX assembles for sm_100a; the interpreter (the oracle the GPU tests compare against) agrees
with a direct numpy evaluation of the pointwise op DAGs and with fp64 on rows and reductions.
"""

import shutil
import subprocess

import numpy as np
import pytest

from emmyptx import synth
from emmyptx.emit import compile_payload

SEEDS = range(24)


def _ptxas(ptx, tmp_path):
    exe = shutil.which("ptxas") or "/usr/local/cuda/bin/ptxas"
    f = tmp_path / "k.ptx"
    f.write_text(ptx)
    r = subprocess.run([exe, "-arch=sm_100a", str(f), "-o", str(tmp_path / "k.cubin")],
                       capture_output=True, text=True)
    assert r.returncode == 0, r.stderr[-400:]


@pytest.mark.parametrize("family", ["pointwise", "rows", "reduction", "contraction",
                                    "contraction_tc", "contraction_ragged", "attention"])
def test_synthesized_kernels_lower_and_assemble(family, tmp_path):
    templates = set()
    # the forced-template families (pairs, half-width units, split-K, masked edges) are
    # compiled as their GPU tests compile them
    force = "contraction" if family in ("contraction_tc", "contraction_ragged") else None
    for seed in SEEDS:
        payload, meta, info = getattr(synth, family)(seed)
        ptx, template, _ = compile_payload(payload, meta, template=force)
        assert ".target sm_100a" in ptx
        _ptxas(ptx, tmp_path)
        templates.add(template)
    if family == "contraction":           # both the tcgen05 template and the walker occur
        assert templates == {"contraction", "walker"}
    if force:
        assert templates == {"contraction"}
    if family == "attention":             # tcgen05, the warp-per-row template and the walker
        assert templates == {"attention", "attention_warp", "walker"}


def _flat(a):
    return np.asarray(a, np.float32).reshape(-1)


@pytest.mark.parametrize("seed", SEEDS)
def test_pointwise_interpreter_matches_numpy_dag(seed):
    from oracle.expressions import kernel_inputs
    from oracle.ir_eval import elementwise, run_kernel
    payload, meta, info = synth.pointwise(seed, max_cells=400)
    k = meta["kernels"][0]
    _, _, kernel = compile_payload(payload, meta)
    inputs = kernel_inputs(k)
    got = run_kernel(kernel, k, inputs)["out"]
    env = {n: (_flat(v) if v.size > 1 else np.float32(v.reshape(-1)[0])) for n, v in inputs.items()}
    for name, op, args in info["ops"]:
        env[name] = elementwise(op, [env[a] for a in args])
    want = np.broadcast_to(np.asarray(env[info["ops"][-1][0]], np.float32), got.shape)
    assert np.array_equal(got, want, equal_nan=True)


@pytest.mark.parametrize("seed", range(12))
def test_rows_and_reductions_interpreter_match_fp64(seed):
    from oracle.expressions import kernel_inputs
    from oracle.ir_eval import run_kernel
    for payload, meta, info in (synth.rows(seed, max_rows=8, max_cols=700),
                                synth.reduction(seed, max_n=1 << 14)):
        if info.get("kind") == "softmax" and info["cols"] < info["block"]:
            continue    # threads with no column merge -inf states literally: NaN in the IR's
            #             own semantics; the template tracks validity (checked on the GPU)
        k = meta["kernels"][0]
        _, _, kernel = compile_payload(payload, meta)
        inputs = kernel_inputs(k)
        (out,) = meta["graph_outputs"]
        got = run_kernel(kernel, k, inputs)[out]
        want = _fp64(info, inputs)
        scale = max(float(np.max(np.abs(want))), 1e-30)
        assert np.max(np.abs(got.reshape(want.shape) - want)) <= 1e-5 * scale, info


def _fp64(info, inputs):
    if "op" in info:
        x = inputs[next(n for n in inputs if n not in ("mean_keepdim_count",))].astype(np.float64)
        return np.array([x.sum() if info["op"] == "sum" else x.mean()])
    x = inputs["x"].astype(np.float64)
    kind = info["kind"]
    if kind == "rowsum":
        return x.sum(-1)
    if kind == "softmax":
        e = np.exp(x - x.max(-1, keepdims=True))
        return e / e.sum(-1, keepdims=True)
    if kind == "l2norm":
        return x / np.maximum(np.sqrt((x * x).sum(-1, keepdims=True)), 1e-12)
    w = inputs["w"].astype(np.float64)
    return x / np.sqrt((x * x).mean(-1, keepdims=True) + 1e-6) * w


def test_contraction_tc_covers_every_template_form():
    """synth.contraction_tc's first 32 seeds include single-CTA kernels, CTA pairs, and pairs
    with half-width units, single and pair forms with the split-K atomic epilogue, and every
    one assembles for sm_100a."""
    import shutil
    import subprocess
    import tempfile
    from pathlib import Path

    from emmyptx import synth
    from emmyptx.emit import compile_payload
    forms = set()
    with tempfile.TemporaryDirectory() as tmp:
        for seed in range(32):
            payload, meta, _ = synth.contraction_tc(seed)
            ptx, template, _ = compile_payload(payload, meta, template="contraction")
            assert template == "contraction"
            form = "pair" if ".reqnctapercluster" in ptx else "single"
            if "$L_khalf" in ptx:
                form += "+half"
            forms.add(form)
            if "red.global.add.f32" in ptx:
                assert meta["kernels"][0]["zero_outputs"] == ["matmul"]
                forms.add(form.split("+")[0] + "+atomic")
            if shutil.which("ptxas") and seed < 4:
                f = Path(tmp) / "k.ptx"
                f.write_text(ptx)
                r = subprocess.run(["ptxas", "-arch=sm_100a", "-o", str(Path(tmp) / "k.cubin"),
                                    str(f)], capture_output=True, text=True)
                assert r.returncode == 0, r.stderr
    assert forms == {"single", "pair", "pair+half", "single+atomic", "pair+atomic"}
