"""The reference compiler's stand-in IR reader (``tests/golden/emmy_stub``, used when the
reference-PTX goldens are generated) against this project's decoder: two independent readings
of every fixture and benchmark workload body give the same trees."""

import importlib.util
import json

import numpy as np
import pytest

from conftest import PROBLEMS, ROOT


def _stub():
    path = ROOT / "tests" / "golden" / "emmy_stub" / "emmy" / "compiler" / "graph.py"
    spec = importlib.util.spec_from_file_location("emmy_stub_graph", path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def _same(ours, theirs, where="body"):
    from emmyptx import ir
    if isinstance(ours, ir.Node):
        name = type(ours).__name__
        if name == "dtype":
            assert isinstance(theirs, np.dtype) and theirs.name == ours.name, where
            return
        assert type(theirs).__name__ == name, where
        for f in ours._fields:
            if f in theirs.__dict__:
                _same(getattr(ours, f), theirs.__dict__[f], f"{where}.{name}.{f}")
            else:   # a field the text leaves out: our decoder fills its default
                assert getattr(ours, f) == ir._DEFAULTS[name][f], f"{where}.{name}.{f}"
        assert set(theirs.__dict__) <= set(ours._fields), where
    elif isinstance(ours, (tuple, list)):
        assert isinstance(theirs, (tuple, list)) and len(ours) == len(theirs), where
        for i, (a, b) in enumerate(zip(ours, theirs)):
            _same(a, b, f"{where}[{i}]")
    elif isinstance(ours, float) and ours != ours:
        assert theirs != theirs, where
    else:
        assert ours == theirs and type(ours) is type(theirs), where


def _payloads():
    from emmyptx import workloads
    for f in sorted(PROBLEMS.glob("*/*.ir.json")):
        yield f.parent.name, json.loads(f.read_text())
    for name, make in workloads.WORKLOADS.items():
        yield name, make()[0]


@pytest.mark.parametrize("tag,payload", list(_payloads()), ids=lambda v: v if isinstance(v, str) else "")
def test_stub_and_decoder_agree(tag, payload):
    from emmyptx import ir
    stub = _stub()
    graph = stub.Graph.from_dict(payload)
    ours = ir.graph_from_dict(payload)
    assert set(graph.nodes) == set(ours.nodes)
    for key, node in ours.nodes.items():
        theirs = graph.nodes[key]
        assert type(theirs.op).__name__ == type(node.op).__name__
        assert tuple(theirs.inputs) == tuple(node.inputs)
        assert [t.name for t in theirs.outputs] == [t.name for t in node.outputs]
        if type(node.op).__name__ == "KernelOp":
            assert theirs.op.name == node.op.name
            _same(tuple(node.op.body), theirs.op.body)


def test_stub_needs_nothing_from_this_project():
    text = (ROOT / "tests" / "golden" / "emmy_stub" / "emmy" / "compiler" / "graph.py").read_text()
    assert "emmyptx" not in text.split('"""', 2)[2]
