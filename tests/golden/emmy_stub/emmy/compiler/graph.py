"""Stand-in for emmy-ml's ``emmy.compiler.graph`` (emmy-ml 0.3.11 is not installable offline),
used only to run the reference compiler when the reference-PTX goldens are generated.

``Graph.from_dict`` decodes each KernelOp body statement (the repr text Emmy serialises) with
Python's ``ast`` into plain objects named after their constructors, whose attributes are the
keyword fields of the text. It shares no code with this project's decoder, so the reference's
PTX cannot inherit a decoding mistake of ours. The reference reads the nodes through
``type(x).__name__`` and attribute access (reference ``compile.py:1831-1900`` and its
lowerers); the three positional forms Emmy writes are ``Dim(<value>)``,
``ElementwiseImpl('<name>')`` and numpy's ``dtype('<name>')`` (also read as
``dtype(name='<name>')``).
"""

from __future__ import annotations

import ast
import math

import numpy as np

_POSITIONAL = {"Dim": ("value",), "ElementwiseImpl": ("name",)}
_TYPES: dict = {}


class _Node:
    """A decoded IR constructor call: its keyword fields as attributes."""

    def __init__(self, **fields):
        self.__dict__.update(fields)

    def __repr__(self):
        inner = ", ".join(f"{k}={v!r}" for k, v in self.__dict__.items())
        return f"{type(self).__name__}({inner})"

    def __eq__(self, other):
        return type(self) is type(other) and self.__dict__ == other.__dict__

    def __hash__(self):
        return hash((type(self).__name__, repr(self)))


def _type(name):
    if name not in _TYPES:
        _TYPES[name] = type(name, (_Node,), {})
    return _TYPES[name]


def _value(node):
    if isinstance(node, ast.Constant):
        return node.value
    if isinstance(node, ast.Tuple):
        return tuple(_value(e) for e in node.elts)
    if isinstance(node, ast.List):
        return [_value(e) for e in node.elts]
    if isinstance(node, ast.UnaryOp) and isinstance(node.op, ast.USub):
        return -_value(node.operand)
    if isinstance(node, ast.Name) and node.id in ("inf", "nan"):
        return math.inf if node.id == "inf" else math.nan
    if isinstance(node, ast.Call) and isinstance(node.func, ast.Name):
        name = node.func.id
        args = [_value(a) for a in node.args]
        if name == "dtype":
            kw = {k.arg: _value(k.value) for k in node.keywords}
            return np.dtype(*(args or [kw["name"]]))
        fields = dict(zip(_POSITIONAL.get(name, ()), args))
        if len(args) > len(fields):
            raise ValueError(f"unexpected positional arguments to {name}")
        for kw in node.keywords:
            fields[kw.arg] = _value(kw.value)
        return _type(name)(**fields)
    raise ValueError(f"unsupported syntax in IR text: {ast.dump(node)[:80]}")


def decode_statement(text):
    return _value(ast.parse(text, mode="eval").body)


class Tensor(_Node):
    pass


class GraphNode(_Node):
    pass


class Graph:
    def __init__(self, inputs, outputs, nodes):
        self.inputs, self.outputs, self.nodes = tuple(inputs), tuple(outputs), nodes

    @classmethod
    def from_dict(cls, payload):
        nodes = {}
        for key, raw in payload["nodes"].items():
            fields = dict(raw.get("op_fields") or {})
            if raw["op"] == "KernelOp":
                fields["body"] = tuple(decode_statement(t) for t in fields.get("body", ()))
            op = _type(raw["op"])(**fields)
            outputs = tuple(Tensor(name=t["name"], shape=tuple(t.get("shape") or ()),
                                   dtype=t.get("dtype", "f32"))
                            for t in raw.get("outputs") or ())
            nodes[key] = GraphNode(op=op, inputs=tuple(raw.get("inputs") or ()), outputs=outputs)
        return cls(payload.get("inputs") or (), payload.get("outputs") or (), nodes)
