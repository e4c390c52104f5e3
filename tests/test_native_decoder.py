"""The native IR decoder (emmy-ir-to-ptx_b200/csrc/emmy_irdecode.c) against the Python
decoders: the same node trees for every fixture, benchmark workload and synthesized body, and
the Python paths (with their error messages) for anything it does not take."""

import json

import pytest

from conftest import PROBLEMS


def _bodies():
    from emmyptx import synth, workloads
    for f in sorted(PROBLEMS.glob("*/*.ir.json")):
        yield f.parent.name, json.loads(f.read_text())
    for name, make in workloads.WORKLOADS.items():
        yield name, make()[0]
    for seed in range(6):
        for fn in (synth.pointwise, synth.rows, synth.reduction, synth.contraction,
                   synth.attention, synth.contraction_ragged):
            yield f"{fn.__name__}-{seed}", fn(seed)[0]


def _statements(payload):
    for node in payload["nodes"].values():
        if node["op"] == "KernelOp":
            yield from node["op_fields"]["body"]


def _python_decode(text):
    import ast

    from emmyptx import ir
    fast = ir._fast_json(text)
    if fast is not None:
        return ir._fast_build(json.loads(fast, strict=False))
    return ir._convert(ast.parse(text, mode="eval").body)


def test_native_decoder_is_built():
    from emmyptx import ir
    assert ir._native is not None, "build() compiles emmyptx/_irdecode"


@pytest.mark.parametrize("tag,payload", list(_bodies()), ids=lambda v: v if isinstance(v, str) else "")
def test_native_matches_python(tag, payload):
    from emmyptx import ir
    for text in _statements(payload):
        assert ir._native.decode(text) == _python_decode(text), tag


def test_shared_subtrees_are_one_object():
    from emmyptx import ir
    f32 = "DataType(name='f32', np=dtype('float32'), nbytes=4)"
    text = f"Let(name='a', value=Literal(value=1, dtype='int'), dtype={f32})"
    node = ir._native.decode(f"Cond(cond=Var(name='c'), body=({text}, {text}), else_body=())")
    assert node.body[0] is node.body[1]


@pytest.mark.parametrize("text,msg", [
    ("Frob(x=1)", "unknown IR constructor"),
    ("Var(name='a', bogus=1)", "no field"),
    ("Var()", "missing field"),
    ("Var('a', name='b')", "twice"),
])
def test_errors_keep_the_python_messages(text, msg):
    from emmyptx import ir
    with pytest.raises(ir.IRDecodeError, match=msg):
        ir.decode_statement(f"Sync(barrier_id={text}, count=None, warp=False)"
                            if text.startswith("Var") else text)


def test_outside_the_native_grammar_falls_back():
    from emmyptx import ir
    text = 'Var(name="quoted")'                       # double quotes: the ast path takes it
    with pytest.raises(ir._native.Fallback):
        ir._native.decode(text)
    assert ir.decode_body([f"Sync(barrier_id={text}, count=None, warp=False)"])


def test_decoding_without_the_native_module(monkeypatch):
    from emmyptx import ir, workloads
    payload, _ = workloads.WORKLOADS["rmsnorm"]()
    text = next(_statements(payload))
    with_native = ir.decode_statement(text)
    monkeypatch.setattr(ir, "_native", None)
    assert ir.decode_statement(text) == with_native
