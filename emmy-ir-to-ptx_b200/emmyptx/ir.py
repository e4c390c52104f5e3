"""Emmy Kernel IR: node types and a whitelisted decoder for the KernelOp body.

The reference reads the IR through the third-party wheel ``emmy-ml==0.3.11``
(``Graph.from_dict``, reference ``compile.py:1838-1850``). That wheel is not
available, so this module decodes the graph JSON itself.

A ``KernelOp`` body is stored as one Python ``repr`` string per statement,
built from about 25 constructors (``Tile``, ``Load``, ``Assign`` ...; the
vocabulary is listed in the reference ``TASK.md:89-187``). Only calls to the
constructors named in :data:`NODE_FIELDS`, tuples, strings, numbers, ``None``
and booleans are accepted. Nothing is evaluated, so a malicious IR cannot run
code.

Two decoders read that grammar. The fast one rewrites the repr text into JSON
with two regular-expression passes (``Name(`` and ``field=`` become marked
JSON strings, parentheses become brackets), parses it with :func:`json.loads`
and builds the nodes, sharing identical subtrees; it takes about a quarter of
the time of :func:`ast.parse` on large bodies. It applies only when every
string literal is a plain token (no quotes, backslashes, parentheses, ``x=``
or the words ``None``/``True``/``False``); otherwise, or when the rewritten
text is not valid JSON, the body is parsed with :func:`ast.parse` and
converted node by node, which also produces the error for a malformed body.

Class names match Emmy's (``type(x).__name__``), ``Dim.value`` holds the
extent, ``ElementwiseImpl.name`` the operation and ``DataType.name`` the
scalar type name, so code written against Emmy objects reads the same.
"""

from __future__ import annotations

import ast
import json
import re

__all__ = [
    "Node", "NODE_FIELDS", "IRDecodeError", "decode_statement", "decode_body",
    "Graph", "GraphNode", "Tensor", "graph_from_dict", "load_graph", "walk",
]


class IRDecodeError(ValueError):
    """Raised when a KernelOp body or graph does not follow the IR grammar."""


class Node:
    """Base of every IR node: immutable, keyword-constructed, structural equality."""

    __slots__ = ()
    _fields: tuple = ()

    def __init__(self, *args, **kwargs):
        fields = self._fields
        if len(args) > len(fields):
            raise TypeError(f"{type(self).__name__} takes at most {len(fields)} positional arguments")
        values = dict(zip(fields, args))
        for key, value in kwargs.items():
            if key not in fields:
                raise TypeError(f"{type(self).__name__} has no field {key!r}")
            if key in values:
                raise TypeError(f"{type(self).__name__} got {key!r} twice")
            values[key] = value
        defaults = _DEFAULTS.get(type(self).__name__, {})
        for f in fields:
            if f in values:
                v = values[f]
            elif f in defaults:
                v = defaults[f]
            else:
                raise TypeError(f"{type(self).__name__} is missing field {f!r}")
            object.__setattr__(self, f, v)

    def __setattr__(self, key, value):
        raise AttributeError(f"{type(self).__name__} is immutable")

    def __iter__(self):
        return iter(getattr(self, f) for f in self._fields)

    def __eq__(self, other):
        return type(self) is type(other) and all(
            getattr(self, f) == getattr(other, f) for f in self._fields)

    def __hash__(self):
        return hash((type(self).__name__,) + tuple(_hashable(getattr(self, f)) for f in self._fields))

    def __repr__(self):
        inner = ", ".join(f"{f}={getattr(self, f)!r}" for f in self._fields)
        return f"{type(self).__name__}({inner})"

    def replace(self, **changes):
        values = {f: getattr(self, f) for f in self._fields}
        values.update(changes)
        return type(self)(**values)


def _hashable(v):
    if isinstance(v, list):
        return tuple(_hashable(x) for x in v)
    if isinstance(v, dict):
        return tuple(sorted((k, _hashable(x)) for k, x in v.items()))
    return v


# Field lists per constructor. Statements and expressions follow the IR
# reference table (reference TASK.md:89-187); the extra value types
# (Axis, Dim, Window, DataType, ElementwiseImpl, dtype) are the ones that
# appear inside them in the shipped fixtures.
NODE_FIELDS: dict[str, tuple[str, ...]] = {
    # launch / structure
    "Tile": ("axes", "body", "block_threads", "aux_threads", "raster_axes", "raster_group",
             "raster_orient"),
    "Axis": ("name", "extent", "window"),
    "Dim": ("value",),
    "Window": ("parent", "base", "bound", "partition"),
    # scalar compute
    "Load": ("names", "input", "index", "dtype"),
    "Assign": ("name", "op", "args", "dtype"),
    "Let": ("name", "value", "dtype"),
    "Accum": ("name", "value", "op", "dtype", "axes", "base"),
    "Init": ("name", "identity", "dtype"),
    "Write": ("output", "index", "values", "value_dtype", "atomic", "swizzle"),
    "Loop": ("axis", "body", "unroll", "seed"),
    "StridedLoop": ("axis", "start", "step", "body", "unroll", "end", "seed"),
    "Cond": ("cond", "body", "else_body"),
    # shared memory and barriers
    "Smem": ("name", "extents", "dtype", "align"),
    "Sync": ("barrier_id", "count", "warp"),
    "CpAsyncCopy": ("smem", "smem_index", "src", "src_index", "nbytes", "swizzle", "lane_index",
                    "lane_rows"),
    "CpAsyncCommit": (),
    "CpAsyncWait": ("group",),
    # cross-thread combine
    "WarpShuffle": ("state", "state_b", "combine_states", "length", "dtype"),
    "TreeHalve": ("bufs", "state", "state_b", "combine_states", "length", "tid_var", "dtype",
                  "barrier_id", "barrier_count", "inner"),
    # expressions
    "Var": ("name",),
    "Literal": ("value", "dtype"),
    "BinaryExpr": ("op", "left", "right"),
    "TernaryExpr": ("cond", "if_true", "if_false"),
    # value types
    "DataType": ("name", "np", "nbytes"),
    "ElementwiseImpl": ("name",),
    "dtype": ("name",),
}

_DEFAULTS: dict[str, dict] = {
    "Tile": {"block_threads": None, "aux_threads": 0, "raster_axes": None, "raster_group": None,
             "raster_orient": "m"},
    "Axis": {"window": None},
    "Window": {"base": None, "bound": None, "partition": False},
    "Load": {"dtype": None},
    "Assign": {"dtype": None},
    "Let": {"dtype": None},
    "Accum": {"dtype": None, "axes": (), "base": None},
    "Init": {"dtype": None},
    "Write": {"value_dtype": None, "atomic": False, "swizzle": "NONE"},
    "Loop": {"unroll": False, "seed": True},
    "StridedLoop": {"unroll": False, "end": None, "seed": True},
    "Cond": {"else_body": ()},
    "Smem": {"align": 0},
    "Sync": {"barrier_id": 0, "count": None, "warp": False},
    "CpAsyncCopy": {"swizzle": "NONE", "lane_index": None, "lane_rows": 0},
    "CpAsyncWait": {"group": 0},
    "WarpShuffle": {"state_b": (), "combine_states": (), "dtype": None},
    "TreeHalve": {"state_b": (), "combine_states": (), "tid_var": "warp", "dtype": None,
                  "barrier_id": 0, "barrier_count": None, "inner": None},
    "DataType": {"np": None, "nbytes": 4},
}

_CLASSES: dict[str, type] = {}
for _name, _fields in NODE_FIELDS.items():
    _CLASSES[_name] = type(_name, (Node,), {"__slots__": _fields, "_fields": _fields})
globals().update(_CLASSES)
__all__ += list(_CLASSES)

STATEMENT_KINDS = frozenset({
    "Tile", "Load", "Assign", "Let", "Accum", "Init", "Write", "Loop", "StridedLoop", "Cond",
    "Smem", "Sync", "CpAsyncCopy", "CpAsyncCommit", "CpAsyncWait", "WarpShuffle", "TreeHalve",
})
def _convert(node):
    """Turn one ``ast`` node of a KernelOp repr into IR values (no evaluation)."""
    if isinstance(node, ast.Call):
        if not isinstance(node.func, ast.Name) or node.func.id not in _CLASSES:
            raise IRDecodeError(f"unknown IR constructor: {ast.unparse(node.func)}")
        cls = _CLASSES[node.func.id]
        if any(k.arg is None for k in node.keywords):
            raise IRDecodeError("**kwargs are not part of the IR grammar")
        args = [_convert(a) for a in node.args]
        kwargs = {k.arg: _convert(k.value) for k in node.keywords}
        try:
            return cls(*args, **kwargs)
        except TypeError as exc:
            raise IRDecodeError(str(exc)) from exc
    if isinstance(node, ast.Constant):
        if node.value is None or isinstance(node.value, (bool, int, float, str)):
            return node.value
        raise IRDecodeError(f"unsupported constant {node.value!r}")
    if isinstance(node, ast.Tuple):
        return tuple(_convert(e) for e in node.elts)
    if isinstance(node, ast.List):
        return tuple(_convert(e) for e in node.elts)
    if isinstance(node, ast.UnaryOp) and isinstance(node.op, ast.USub) \
            and isinstance(node.operand, ast.Constant) \
            and isinstance(node.operand.value, (int, float)) \
            and not isinstance(node.operand.value, bool):
        return -node.operand.value
    if isinstance(node, ast.UnaryOp) and isinstance(node.op, ast.USub) \
            and isinstance(node.operand, ast.Name) and node.operand.id in ("inf", "nan"):
        return -float(node.operand.id)        # repr(float("-inf")) is "-inf"
    if isinstance(node, ast.Name) and node.id in ("inf", "nan"):
        return float(node.id)
    raise IRDecodeError(f"unsupported syntax in IR body: {ast.dump(node)[:80]}")


_FAST_CALL = re.compile(r"\b(\w++)\(")
_FAST_KW = re.compile(r"\b(\w++)=")
_FAST_STR = re.compile(r"'([^']*)'")
_FAST_BAD_STR = re.compile(r"[()\\\"]|\w=|\b(?:None|True|False)\b")
_FAST_BRACKETS = str.maketrans({"(": "[", ")": "]", "'": '"'})
_CALL_MARK, _KW_MARK = "\x02", "\x01"
_MISSING = object()
assert not any(w in n for n in list(NODE_FIELDS) + [f for fs in NODE_FIELDS.values() for f in fs]
               for w in ("None", "True", "False"))


def _fast_json(text: str):
    """The repr text rewritten as JSON, or None when the fast path does not apply."""
    if '"' in text or "\\" in text or _CALL_MARK in text or _KW_MARK in text:
        return None
    if _FAST_BAD_STR.search("\x00".join(_FAST_STR.findall(text))):
        return None
    t = _FAST_CALL.sub('["\x02\\1",', text)
    t = _FAST_KW.sub('"\x01\\1",', t)
    t = t.translate(_FAST_BRACKETS).replace(",]", "]")
    if "None" in t:
        t = t.replace("None", "null")
    if "True" in t:
        t = t.replace("True", "true")
    if "False" in t:
        t = t.replace("False", "false")
    return t


def _make_node(name, pos, kw):
    """Construct ``name(*pos, **kw)`` with the same checks as :meth:`Node.__init__`."""
    cls = _CLASSES.get(name)
    if cls is None:
        raise IRDecodeError(f"unknown IR constructor: {name}")
    fields = cls._fields
    if pos:
        if len(pos) > len(fields):
            raise IRDecodeError(f"{name} takes at most {len(fields)} positional arguments")
        for f, v in zip(fields, pos):
            if f in kw:
                raise IRDecodeError(f"{name} got {f!r} twice")
            kw[f] = v
    obj = object.__new__(cls)
    defaults = _DEFAULTS.get(name)
    used = 0
    for f in fields:
        v = kw.get(f, _MISSING)
        if v is _MISSING:
            if defaults is None or f not in defaults:
                raise IRDecodeError(f"{name} is missing field {f!r}")
            v = defaults[f]
        else:
            used += 1
        object.__setattr__(obj, f, v)
    if used != len(kw):
        bad = next(k for k in kw if k not in fields)
        raise IRDecodeError(f"{name} has no field {bad!r}")
    return obj


def _fast_build(data):
    """Nodes from the JSON form; identical subtrees are built once and shared (nodes are
    immutable)."""
    memo = {}

    def build(x):
        head = x[0] if x else None
        if type(head) is not str or head[:1] != _CALL_MARK:
            return tuple([build(e) if type(e) is list else e for e in x])
        pos, kw, key = [], {}, [head]
        i, n = 1, len(x)
        while i < n:
            e = x[i]
            if type(e) is str and e[:1] == _KW_MARK:
                if i + 1 >= n:
                    raise IRDecodeError("keyword without a value in IR body")
                v = x[i + 1]
                if type(v) is list:
                    v = build(v)
                kw[e[1:]] = v
                key.append(e)
                i += 2
            else:
                v = build(e) if type(e) is list else e
                pos.append(v)
                i += 1
            key.append(id(v) if isinstance(v, (Node, tuple)) else (type(v), v))
        key = tuple(key)
        hit = memo.get(key)
        if hit is None:
            hit = _make_node(head[1:], pos, kw)
            memo[key] = (hit, pos, kw)     # keep children alive so their ids stay unique
            return hit
        return hit[0]

    return build(data)


try:  # the native decoder (csrc/emmy_irdecode.c), built in-tree by __graft_entry__.build()
    from . import _irdecode as _native
    _native.setup(_CLASSES, NODE_FIELDS, _DEFAULTS, IRDecodeError)
except ImportError:
    _native = None


def decode_statement(text: str):
    """Decode one statement repr string into IR nodes.

    The native decoder reads the grammar in one pass when it is built; on anything it does
    not cover, and on any error, the statement is decoded again here (the JSON fast path,
    else :func:`ast.parse`), so results and error messages are the Python decoders'."""
    if not isinstance(text, str):
        raise IRDecodeError("KernelOp body entries must be strings")
    if _native is not None:
        try:
            value = _native.decode(text)
        except Exception:           # noqa: BLE001 - Fallback, or an error the paths below name
            value = None
        if isinstance(value, Node) and type(value).__name__ in STATEMENT_KINDS:
            return value
    try:
        return _decode_python(text)
    except RecursionError:
        raise IRDecodeError("KernelOp body nests too deeply") from None


def _decode_python(text: str):
    fast = _fast_json(text)
    if fast is not None:
        try:
            data = json.loads(fast, strict=False)
        except ValueError:
            data = None
        if type(data) is list:
            value = _fast_build(data)
            if not isinstance(value, Node) or type(value).__name__ not in STATEMENT_KINDS:
                raise IRDecodeError("KernelOp body entry is not an IR statement")
            return value
    try:
        tree = ast.parse(text, mode="eval")
    except SyntaxError as exc:
        raise IRDecodeError(f"KernelOp body is not a valid repr: {exc.msg}") from exc
    value = _convert(tree.body)
    if not isinstance(value, Node) or type(value).__name__ not in STATEMENT_KINDS:
        raise IRDecodeError("KernelOp body entry is not an IR statement")
    return value


def decode_body(body) -> tuple:
    if isinstance(body, str):
        body = [body]
    if not isinstance(body, (list, tuple)):
        raise IRDecodeError("KernelOp body must be a list of statement strings")
    return tuple(decode_statement(s) for s in body)


# ---------------------------------------------------------------------------
# Graph level (plain JSON: inputs, outputs, nodes{op, op_fields, inputs, outputs})
# ---------------------------------------------------------------------------

class Tensor:
    __slots__ = ("name", "shape", "dtype")

    def __init__(self, name, shape, dtype):
        self.name, self.shape, self.dtype = name, tuple(shape or ()), dtype

    def __repr__(self):
        return f"Tensor({self.name!r}, {self.shape}, {self.dtype!r})"


class _Op:
    """Graph operator: ``InputOp``, ``ConstantOp`` or ``KernelOp`` (class name = op name)."""

    def __init__(self, **fields):
        self.__dict__.update(fields)

    def __repr__(self):
        return f"{type(self).__name__}({', '.join(sorted(self.__dict__))})"


class InputOp(_Op):
    pass


class ConstantOp(_Op):
    pass


class KernelOp(_Op):
    pass


_OPS = {"InputOp": InputOp, "ConstantOp": ConstantOp, "KernelOp": KernelOp}


class GraphNode:
    __slots__ = ("op", "inputs", "outputs")

    def __init__(self, op, inputs, outputs):
        self.op, self.inputs, self.outputs = op, inputs, outputs


class Graph:
    __slots__ = ("inputs", "outputs", "nodes")

    def __init__(self, inputs, outputs, nodes):
        self.inputs, self.outputs, self.nodes = tuple(inputs), tuple(outputs), nodes

    @classmethod
    def from_dict(cls, payload):
        return graph_from_dict(payload)


def graph_from_dict(payload) -> Graph:
    """Build a :class:`Graph` from the IR JSON object (replaces emmy's ``Graph.from_dict``)."""
    if not isinstance(payload, dict):
        raise IRDecodeError("IR JSON must be an object")
    nodes_in = payload.get("nodes")
    if not isinstance(nodes_in, dict):
        raise IRDecodeError("IR JSON has no 'nodes' mapping")
    nodes = {}
    for key, raw in nodes_in.items():
        if not isinstance(raw, dict):
            raise IRDecodeError(f"node {key!r} is not an object")
        op_name = raw.get("op")
        if op_name not in _OPS:
            raise IRDecodeError(f"node {key!r}: unknown op {op_name!r}")
        fields = dict(raw.get("op_fields") or {})
        if op_name == "KernelOp":
            fields["body"] = decode_body(fields.get("body", ()))
            fields.setdefault("zero_delegated", ())
            fields.setdefault("serial", ())
        outputs = []
        for t in raw.get("outputs") or ():
            if not isinstance(t, dict) or "name" not in t:
                raise IRDecodeError(f"node {key!r}: malformed output tensor")
            outputs.append(Tensor(t["name"], t.get("shape") or (), t.get("dtype", "f32")))
        nodes[key] = GraphNode(_OPS[op_name](**fields), tuple(raw.get("inputs") or ()),
                               tuple(outputs))
    return Graph(payload.get("inputs") or (), payload.get("outputs") or (), nodes)


def load_graph(path) -> Graph:
    with open(path, "r", encoding="utf-8") as fh:
        return graph_from_dict(json.load(fh))


def walk(statements):
    """Yield every statement in ``statements``, depth first, including nested bodies."""
    for stmt in statements:
        yield stmt
        kind = type(stmt).__name__
        if kind in ("Tile", "Loop", "StridedLoop"):
            yield from walk(stmt.body)
        elif kind == "Cond":
            yield from walk(stmt.body)
            yield from walk(stmt.else_body)


def dim_value(extent) -> int:
    """Integer value of an ``Axis.extent`` (a ``Dim`` or a bare int)."""
    v = extent.value if isinstance(extent, _CLASSES["Dim"]) else extent
    if type(v) is not int:
        raise IRDecodeError(f"symbolic extent {v!r} (dynamic shapes are not supported)")
    return v


def op_name(op) -> str:
    """Name of an elementwise op (``ElementwiseImpl('add')`` -> ``'add'``)."""
    if isinstance(op, _CLASSES["ElementwiseImpl"]):
        return op.name
    if isinstance(op, str):
        return op
    raise IRDecodeError(f"unsupported elementwise descriptor {op!r}")


def dtype_name(dt) -> str | None:
    """Scalar type name of a ``DataType`` (``'f32'``), or None when untyped."""
    if dt is None:
        return None
    if isinstance(dt, _CLASSES["DataType"]):
        return dt.name
    if isinstance(dt, str):
        return dt
    raise IRDecodeError(f"unsupported dtype {dt!r}")
