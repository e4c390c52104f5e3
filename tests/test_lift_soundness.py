"""The pointwise lift is faithful to the IR it accepts: a plan evaluated in numpy gives the
oracle interpreter's result of the same IR, bit for bit, also on IR the fixtures and the
synthesizer never wrote.

Each case mutates one site of a pointwise body (an elementwise op replaced by another of the
same arity, the operands of a binary op swapped, a float literal scaled, an integer literal
in an index moved): whenever the lift still accepts the body, its element program, run on
the seeded inputs, must equal what the IR computes. The template emits that program op by
op (the GPU tests check the kernel against the interpreter on the unmutated forms), so a lift
that dropped or misread part of a body would show here as a mismatch.
"""

import json
import random
import re

import numpy as np
import pytest

from conftest import PROBLEMS

OPS2 = ["add", "subtract", "multiply", "maximum", "minimum", "divide"]
OPS1 = ["exp", "log", "sqrt", "reciprocal", "relu", "neg", "abs", "square", "copy"]


def _mutations(text, rng, n):
    sites = [("int", m) for m in re.finditer(r"Literal\(value=(-?\d+), dtype='int'\)", text)]
    sites += [("float", m) for m in re.finditer(r"Literal\(value=(-?[\d.]+), dtype='float'\)",
                                                 text)]
    sites += [("op", m) for m in re.finditer(r"ElementwiseImpl\('(\w+)'\)", text)]
    sites += [("swap", m) for m in re.finditer(r"args=\('(\w+)', '(\w+)'\)", text)]
    rng.shuffle(sites)
    for kind, m in sites[:n]:
        a, b = m.span(1)
        if kind == "int":
            new = str(int(m.group(1)) + rng.choice([-1, 1, 2]))
        elif kind == "float":
            new = repr(float(m.group(1)) * rng.choice([2.0, -1.0, 0.5]))
        elif kind == "op":
            pool = OPS2 if m.group(1) in OPS2 else OPS1 if m.group(1) in OPS1 else None
            if pool is None:
                continue
            new = rng.choice([o for o in pool if o != m.group(1)])
        else:
            a, b = m.span(1)[0], m.span(2)[1]
            new = f"{m.group(2)}', '{m.group(1)}"
        yield text[:a] + new + text[b:]


def _evaluate(plan, inputs, shapes):
    """The lifted element program over all plan.total elements at once (f32, the oracle's
    op semantics)."""
    from emmyptx.analysis import ElemLet, ElemLoad, ElemOp, ElemWrite
    from oracle.ir_eval import elementwise
    env, out = {}, {}
    n = plan.total
    for p in plan.program:
        if isinstance(p, ElemLoad):
            flat = np.asarray(inputs[p.buffer], np.float32).reshape(-1)
            env[p.name] = flat[:n] if p.kind == "elem" else np.full(n, flat[p.offset])
        elif isinstance(p, ElemLet):
            env[p.name] = np.full(n, np.float32(p.value))
        elif isinstance(p, ElemOp):
            env[p.name] = elementwise(p.op, [env[a] for a in p.args])
        elif isinstance(p, ElemWrite):
            buf = np.zeros(int(np.prod(shapes[p.buffer])), np.float32)
            buf[:n] = env[p.value]
            out[p.buffer] = buf
    return out


def _bodies():
    from emmyptx import synth
    for f in sorted(PROBLEMS.glob("p0*/*.ir.json")):
        meta = json.loads((f.parent / "meta.json").read_text())
        yield f.parent.name, json.loads(f.read_text()), meta
    for seed in range(12):
        payload, meta, _ = synth.pointwise(seed, max_cells=700)
        yield f"synth-{seed}", payload, meta


@pytest.mark.parametrize("tag,payload,meta", list(_bodies()), ids=lambda v: v if isinstance(v, str) else "")
def test_pointwise_lift_matches_the_interpreter_under_mutation(tag, payload, meta, tmp_path):
    from emmyptx.analysis import lift_pointwise
    from emmyptx.meta import EmmyIRParser
    from oracle.expressions import kernel_inputs
    from oracle.ir_eval import run_kernel
    k = meta["kernels"][0]
    node = next(n for n in payload["nodes"].values() if n["op"] == "KernelOp")
    text = node["op_fields"]["body"][0]
    inputs = kernel_inputs(k)
    rng = random.Random(tag)
    compared = 0
    for mutated in [text, *_mutations(text, rng, 16)]:
        node["op_fields"]["body"] = [mutated]
        (tmp_path / "k.ir.json").write_text(json.dumps(payload))
        (tmp_path / "meta.json").write_text(json.dumps(dict(meta, kernels=[dict(k, entry=node[
            "op_fields"]["name"])])))
        try:
            kernel = EmmyIRParser(tmp_path / "k.ir.json", require_meta=True).parse()
        except ValueError:
            continue
        plan = lift_pointwise(kernel)
        if plan is None:
            continue
        try:
            want = run_kernel(kernel, k, inputs)
        except (IndexError, ValueError, NotImplementedError):
            continue                    # the mutation made the IR itself invalid
        shapes = {a["name"]: tuple(a.get("shape") or (1,)) for a in k["args"]}
        got = _evaluate(plan, inputs, shapes)
        assert set(got) == set(want), tag
        for name, arr in want.items():
            assert np.array_equal(got[name], np.asarray(arr, np.float32).reshape(-1),
                                  equal_nan=True), (tag, name, mutated[:200])
        compared += 1
    assert compared >= 1, tag


@pytest.mark.parametrize("problem", ["r01_array_sum", "r02_big_sum", "r03_mean", "r04_row_sum",
                                     "f01_rmsnorm", "f02_row_softmax", "f03_l2norm"])
def test_row_lift_notices_every_change_of_result(problem, tmp_path):
    """Reductions and row normalisations: a mutation that changes what the IR computes (the
    oracle interpreter's output) must change the lifted plan or make the lift decline, so the
    row template never runs the unmutated program for a body that asks for another."""
    from emmyptx.analysis import lift_rowreduce
    from emmyptx.meta import EmmyIRParser
    from oracle.expressions import kernel_inputs
    from oracle.ir_eval import run_kernel
    pdir = PROBLEMS / problem
    meta = json.loads((pdir / "meta.json").read_text())
    k = meta["kernels"][0]
    payload = json.loads((pdir / f"{k['entry']}.ir.json").read_text())
    node = next(n for n in payload["nodes"].values() if n["op"] == "KernelOp")
    text = node["op_fields"]["body"][0]
    inputs = kernel_inputs(k)
    (tmp_path / "meta.json").write_text(json.dumps(meta))

    def parse(body):
        node["op_fields"]["body"] = [body]
        (tmp_path / f"{k['entry']}.ir.json").write_text(json.dumps(payload))
        return EmmyIRParser(tmp_path / f"{k['entry']}.ir.json", require_meta=True).parse()

    base = parse(text)
    base_plan = repr(lift_rowreduce(base))
    assert base_plan != "None"
    base_out = run_kernel(base, k, inputs)
    for mutated in _mutations(text, random.Random(problem), 24):
        try:
            kernel = parse(mutated)
        except ValueError:
            continue
        if repr(lift_rowreduce(kernel)) != base_plan:
            continue
        try:
            with np.errstate(all="ignore"):
                out = run_kernel(kernel, k, inputs)
        except (IndexError, ValueError, NotImplementedError):
            continue
        for name, arr in base_out.items():
            assert np.array_equal(np.asarray(out[name]), np.asarray(arr), equal_nan=True), \
                (problem, name, mutated[:200])
