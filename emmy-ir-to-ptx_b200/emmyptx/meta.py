"""Kernel view and parser: IR JSON + sibling ``meta.json`` -> :class:`EmmyKernelIR`.

Mirrors the reference's public API (``EmmyKernelIR`` and
``EmmyIRParser(path, *, meta_path=None, require_meta=False).parse()``,
reference ``compile.py:1769-1994``) with the same error behaviour: exactly one
``KernelOp``; the meta record is selected by graph node *and* entry name;
``arg_order`` from ``meta.json`` is the ABI, not the node's inputs
(reference ``TASK.md:23-27``).
"""

from __future__ import annotations

import json
from dataclasses import dataclass
from pathlib import Path
from typing import Mapping

from .ir import IRDecodeError, graph_from_dict


@dataclass(frozen=True)
class EmmyKernelIR:
    """Validated kernel view: a frozen dataclass with the fields of reference
    ``compile.py:1769-1780``, so ``dataclasses.replace`` derives a variant as it does there."""

    name: str
    body: tuple
    graph: object
    node_key: str
    inputs: tuple
    outputs: tuple
    arg_order: tuple | None
    launch: dict
    metadata: dict

    @property
    def selected(self) -> dict:
        return self.metadata.get("selected_kernel", {})

    def arg(self, name: str) -> dict:
        for a in self.selected.get("args", ()):
            if a.get("name") == name:
                return a
        raise KeyError(name)

    def shape(self, name: str) -> tuple:
        return tuple(self.arg(name).get("shape") or (1,))


def _read_json(path):
    try:
        with Path(path).open("r", encoding="utf-8") as stream:
            result = json.load(stream)
    except OSError as exc:
        raise ValueError(f"Cannot read {path}: {exc}") from exc
    except json.JSONDecodeError as exc:
        raise ValueError(f"Invalid JSON in {path}: {exc}") from exc
    except RecursionError:
        raise ValueError(f"Invalid JSON in {path}: nested too deeply") from None
    if not isinstance(result, dict):
        raise ValueError(f"Expected a JSON object in {path}")
    return result


def _string_names(value, field):
    if value is None:
        return ()
    if not isinstance(value, (tuple, list)):
        raise ValueError(f"{field} must be a list/tuple of names")
    result = tuple(value)
    if any(not isinstance(n, str) or not n for n in result):
        raise ValueError(f"{field} contains an invalid name")
    if len(result) != len(set(result)):
        raise ValueError(f"{field} contains duplicate names")
    return result


class EmmyIRParser:
    """Read one Kernel IR file and its launch record.

    ``meta.json`` (the sibling of the IR file unless ``meta_path`` is given) is
    optional for exploration and required for a submission-grade signature
    (``require_meta=True``), as in the reference.
    """

    def __init__(self, input_path, *, meta_path=None, require_meta=False, payload=None,
                 meta=None):
        self.input_path = Path(input_path)
        self.meta_path = Path(meta_path) if meta_path is not None else None
        self.require_meta = require_meta
        self._payload = payload
        self._meta = meta

    def _metadata_path(self):
        if self.meta_path is not None:
            return self.meta_path
        return self.input_path.parent / "meta.json"

    def parse(self) -> EmmyKernelIR:
        payload = self._payload if self._payload is not None else _read_json(self.input_path)
        try:
            graph = graph_from_dict(payload)
        except IRDecodeError as exc:
            raise ValueError(f"Emmy could not deserialize {self.input_path}: {exc}") from exc

        nodes = graph.nodes
        if not isinstance(nodes, Mapping):
            raise ValueError("Deserialized Emmy Graph has no nodes mapping")
        kernels = [(k, n.op) for k, n in nodes.items() if type(n.op).__name__ == "KernelOp"]
        if len(kernels) != 1:
            raise ValueError(f"Expected exactly one KernelOp, found {len(kernels)}")
        key, op = kernels[0]
        name = getattr(op, "name", None)
        body = getattr(op, "body", None)
        if not isinstance(name, str) or not name:
            raise ValueError("KernelOp.name is missing or invalid")
        if body is None:
            raise ValueError("KernelOp.body is missing")

        node = nodes[key]
        inputs = _string_names(node.inputs, "node.inputs")
        outputs = _string_names([t.name for t in node.outputs], "node.outputs")

        if self._meta is not None:
            metadata = self._meta
        else:
            mpath = self._metadata_path()
            if mpath.is_file():
                metadata = _read_json(mpath)
            elif self.require_meta:
                raise ValueError(f"Missing required metadata file: {mpath}")
            else:
                metadata = {}

        records = metadata.get("kernels")
        if records is None:
            if self.require_meta:
                raise ValueError("meta.json is missing the 'kernels' array")
            kmeta = {}
        else:
            if not isinstance(records, list):
                raise ValueError("meta.kernels must be a list")
            matches = [r for r in records if isinstance(r, dict)
                       and r.get("node") == str(key) and r.get("entry") == name]
            if len(matches) != 1:
                raise ValueError(f"Expected exactly one metadata record for node={key!r}, "
                                 f"entry={name!r}; found {len(matches)}")
            kmeta = matches[0]

        order = kmeta.get("arg_order")
        if order is not None:
            order = _string_names(order, "meta.kernels[].arg_order")
            if not order:
                raise ValueError("Kernel arg_order cannot be empty")
        elif self.require_meta:
            raise ValueError(f"Missing arg_order for kernel {name!r}")

        launch = {f: kmeta[f] for f in ("grid", "block", "smem_bytes") if f in kmeta}
        metadata = {**metadata, "selected_kernel": kmeta}
        return EmmyKernelIR(name=name, body=body, graph=graph, node_key=str(key),
                            inputs=inputs, outputs=outputs, arg_order=order, launch=launch,
                            metadata=metadata)
