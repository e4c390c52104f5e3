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


def _python_value(text):
    """The value the Python decoders give for any repr text (a statement or not): the JSON
    fast path, else the ast path when the JSON text does not load, as decode_statement does."""
    import ast

    from emmyptx import ir
    fast = ir._fast_json(text)
    if fast is not None:
        try:
            data = json.loads(fast, strict=False)
        except ValueError:
            data = None
        if type(data) is list:
            return ir._fast_build(data)
    return ir._convert(ast.parse(text, mode="eval").body)


def test_deep_nesting_fails_closed():
    """A body nested a million levels deep ends in a decode error: the native parser stops at
    its depth bound and the Python decoders' RecursionError becomes IRDecodeError. Run in a
    child process, so that a stack overflow would show as a failed test, not a lost run."""
    import subprocess
    import sys

    from conftest import PKG
    code = (
        "import sys; sys.path.insert(0, sys.argv[1])\n"
        "from emmyptx import ir\n"
        "d = 1_000_000\n"
        "t = 'Sync(barrier_id=' + '(' * d + '1' + ')' * d + ', count=None, warp=False)'\n"
        "try:\n"
        "    ir._native.decode(t)\n"
        "except ir._native.Fallback as e:\n"
        "    assert 'nesting' in str(e), e\n"
        "try:\n"
        "    ir.decode_statement(t)\n"
        "except ir.IRDecodeError as e:\n"
        "    print('refused:', e)\n")
    r = subprocess.run([sys.executable, "-c", code, str(PKG)], capture_output=True, text=True,
                       timeout=120)
    assert r.returncode == 0, r.stderr[-2000:]
    assert "refused: KernelOp body nests too deeply" in r.stdout


@pytest.mark.parametrize("value", ["+5", "007", "00", "007.5", "(5)", "('a')", "((5))", "- 5",
                                   "-(5)", "-", "+inf", "-True"])
def test_forms_python_reads_differently_fall_back(value):
    """Literal forms a repr never writes (a '+' sign, leading zeros, a parenthesized single
    value, a detached sign) are left to the Python decoders, whose result or error stands."""
    from emmyptx import ir
    text = f"Literal(value={value}, dtype='f32')"
    with pytest.raises(ir._native.Fallback):
        ir._native.decode(text)
    try:
        expected = _python_value(text).value
    except Exception as exc:            # noqa: BLE001 - the Python paths' own error
        expected = type(exc)
    try:
        got = ir.decode_statement(f"Sync(barrier_id={text}, count=None, warp=False)").barrier_id.value
    except Exception as exc:            # noqa: BLE001
        got = type(exc)
    if isinstance(expected, type):
        assert isinstance(got, type)
    else:
        assert got == expected


@pytest.mark.parametrize("value,expected", [("-inf", float("-inf")), ("inf", float("inf")),
                                            ("-5", -5), ("-0.25", -0.25), ("1e400", float("inf"))])
def test_signed_and_special_literals(value, expected):
    from emmyptx import ir
    text = f"Literal(value={value}, dtype='f32')"
    assert ir._native.decode(text).value == expected
    assert _python_value(text).value == expected


def test_mutated_bodies_decode_as_python_does():
    """Seeded mutations of the fixtures' statements (a character dropped, inserted or
    replaced, a cut, a repeated span): whenever the native decoder accepts a text, the Python
    decoders give the same tree."""
    import random

    from emmyptx import ir
    texts = [t for f in sorted(PROBLEMS.glob("*/*.ir.json"))
             for t in _statements(json.loads(f.read_text())) if len(t) < 20000]
    rng = random.Random(0)
    alphabet = "()[],='-.0123456789eE ainfNoeTruFls_xyz"
    accepted = 0
    for _ in range(3000):
        t = rng.choice(texts)
        k = rng.randrange(len(t) + 1)
        op = rng.randrange(5)
        if op == 0:
            t = t[:k] + t[k + 1:]
        elif op == 1:
            t = t[:k] + rng.choice(alphabet) + t[k:]
        elif op == 2:
            t = t[:k] + t[rng.randrange(len(t))] + t[k + 1:]
        elif op == 3:
            t = t[:k]
        else:
            j = rng.randrange(len(t) + 1)
            a, b = min(k, j), max(k, j)
            t = t[:a] + t[a:b] * 2 + t[b:]
        try:
            native = ir._native.decode(t)
        except Exception:               # noqa: BLE001 - a refusal is always allowed
            continue
        accepted += 1
        assert native == _python_value(t), t[:300]
    assert accepted > 100
