"""PTX module and kernel builder for sm_100a.

:class:`PTXKernelGenerator` keeps the reference's allocation API
(``register``, ``shared``, ``emit``, ``label``, ``parameter``,
``thread_index_1d``, ``render_entry``; reference ``compile.py:1997-2268``)
and adds what the Blackwell templates need: module-scope declarations
(``.global`` scratch words for cross-CTA finishes and bounded-wait error
flags), register vectors, unique labels and raw template blocks.

Registers are virtual (``%r``, ``%rd``, ``%f``, ``%p`` ...) and declared in
ranges (``.reg .f32 %f<12>;``); ptxas performs the real allocation.
"""

from __future__ import annotations

import re

PTX_VERSION = "8.8"
TARGET_ARCH = "sm_100a"
ADDRESS_SIZE = 64

_IDENT = re.compile(r"(?:[A-Za-z][A-Za-z0-9_$]*|[_$%][A-Za-z0-9_$]+)\Z", re.ASCII)

# register class -> (PTX declaration type, name prefix)
_REG_CLASSES = {
    ".pred": (".pred", "%p"),
    ".f32": (".f32", "%f"),
    ".f64": (".f64", "%fd"),
    ".b16": (".b16", "%h"),
    ".u16": (".b16", "%h"),
    ".u32": (".b32", "%r"),
    ".s32": (".b32", "%r"),
    ".b32": (".b32", "%r"),
    ".u64": (".b64", "%rd"),
    ".s64": (".b64", "%rd"),
    ".b64": (".b64", "%rd"),
}


def module_header() -> str:
    return f".version {PTX_VERSION}\n.target {TARGET_ARCH}\n.address_size {ADDRESS_SIZE}\n"


def identifier(name: str) -> str:
    if not isinstance(name, str) or not _IDENT.match(name):
        raise ValueError(f"Invalid PTX identifier: {name!r}")
    return name


def f32_literal(value: float) -> str:
    """Exact PTX hex literal of an f32 value (``0f3F800000`` for 1.0)."""
    import struct
    return "0f%08X" % struct.unpack("<I", struct.pack("<f", float(value)))[0]


class PTXKernelGenerator:
    """Build one ``.visible .entry`` whose parameters follow ``arg_order``.

    Every argument is a ``.u64`` device pointer named ``param_<arg>``
    (reference ``compile.py:2090-2093``, ``2237-2246``).
    """

    def __init__(self, kernel, *, extra_params=()):
        from .meta import EmmyKernelIR
        if not isinstance(kernel, EmmyKernelIR):
            raise TypeError("Expected an EmmyKernelIR instance")
        self.kernel = kernel
        self.name = identifier(kernel.name)
        if not kernel.arg_order:
            raise ValueError("Kernel requires metadata arg_order")
        selected = kernel.metadata.get("selected_kernel")
        if not isinstance(selected, dict):
            raise ValueError("Missing selected_kernel metadata")
        if selected.get("entry") != kernel.name:
            raise ValueError("Kernel entry does not match metadata")
        if selected.get("node") != kernel.node_key:
            raise ValueError("Kernel node does not match metadata")
        args = selected.get("args")
        if not isinstance(args, list):
            raise ValueError("Kernel metadata requires an args list")
        self.arg_order = tuple(kernel.arg_order)
        if len(set(self.arg_order)) != len(self.arg_order):
            raise ValueError("Duplicate kernel arguments")
        self.arguments = {}
        for arg in args:
            if not isinstance(arg, dict):
                raise ValueError("Invalid argument metadata")
            name = arg.get("name")
            identifier(name)
            if name in self.arguments:
                raise ValueError(f"Duplicate argument metadata: {name}")
            if arg.get("scalar"):
                raise NotImplementedError(f"scalar (by-value) argument {name!r} is not supported")
            if arg.get("dtype", "f32") != "f32":     # every buffer is f32 (reference :2297-2306)
                raise NotImplementedError(f"Unsupported tensor dtype or rank: {name}, "
                                          f"dtype={arg.get('dtype')}, shape={arg.get('shape')}")
            self.arguments[name] = arg
        if set(self.arguments) != set(self.arg_order):
            raise ValueError("arg_order and args metadata do not match")
        self._params = {a: "param_" + a for a in self.arg_order}
        for extra in extra_params:
            self._params[extra] = "param_" + identifier(extra)
        self._param_list = list(self.arg_order) + list(extra_params)
        self._shared = []
        self._module = []
        self._lines = []
        self._labels = set()
        self._counts = {}
        self._label_seq = 0
        self.maxntid = None
        self.minnctapersm = None
        self.cluster = None              # CTAs per cluster along x (compile-time cluster)

    # -- naming ---------------------------------------------------------
    def parameter(self, name: str) -> str:
        if name not in self._params:
            raise KeyError(f"Unknown kernel argument: {name}")
        return self._params[name]

    def register(self, dtype: str = ".u32") -> str:
        cls = _REG_CLASSES.get(dtype)
        if cls is None:
            raise ValueError(f"unsupported register type {dtype!r}")
        prefix = cls[1]
        index = self._counts.get(prefix, 0)
        self._counts[prefix] = index + 1
        return f"{prefix}{index}"

    def registers(self, dtype: str, count: int) -> list:
        return [self.register(dtype) for _ in range(count)]

    def new_label(self, hint: str = "L") -> str:
        self._label_seq += 1
        return f"$L_{hint}_{self._label_seq}"

    # -- declarations ---------------------------------------------------
    def shared(self, name: str, dtype: str, *, length: int, align: int | None = None) -> str:
        identifier(name)
        if type(length) is not int or length <= 0:
            raise ValueError("Shared-memory length must be positive")
        al = f" .align {int(align)}" if align else ""
        decl = f".shared{al} {dtype} {name}[{length}];"
        if any(d.split()[-1].split("[")[0] == name for d in self._shared):
            raise ValueError(f"Duplicate shared declaration: {name}")
        self._shared.append(decl)
        return name

    def module_decl(self, text: str) -> None:
        text.encode("ascii")
        if text not in self._module:
            self._module.append(text)

    # -- body -----------------------------------------------------------
    @staticmethod
    def _validate_line(line: str) -> str:
        """One instruction per call: a line break anywhere (a trailing one included) is
        refused before the surrounding blanks are stripped (reference ``compile.py:2096-2119``)."""
        if type(line) is not str:
            raise TypeError("PTX instruction must be text")
        if "\n" in line or "\r" in line:
            raise ValueError("Expected exactly one ASCII PTX instruction")
        text = line.strip()
        if text.count(";") != 1 or text[-1:] != ";" or not text.isascii():
            raise ValueError("Expected exactly one ASCII PTX instruction")
        return text

    def emit(self, instruction: str) -> None:
        self._lines.append(self._validate_line(instruction))

    def raw(self, text: str) -> None:
        """Append a block of template lines (instructions, labels, braces)."""
        text.encode("ascii")
        for line in text.splitlines():
            line = line.strip()
            if line:
                self._lines.append(line)

    def label(self, name: str) -> None:
        identifier(name.lstrip("$") if name.startswith("$") else name)
        if name in self._labels:
            raise ValueError(f"Duplicate PTX label: {name}")
        self._labels.add(name)
        self._lines.append(f"{name}:")

    def thread_index_1d(self) -> str:
        """``%ctaid.x * %ntid.x + %tid.x`` in a fresh ``.u32`` register: the reference's
        instruction sequence and register numbering (``compile.py:2201-2228``); ptxas fuses
        the multiply and add."""
        tid, bid, ntid, prod, index = (self.register(".u32") for _ in range(5))
        self.emit(f"mov.u32 {tid}, %tid.x;")
        self.emit(f"mov.u32 {bid}, %ctaid.x;")
        self.emit(f"mov.u32 {ntid}, %ntid.x;")
        self.emit(f"mul.lo.u32 {prod}, {bid}, {ntid};")
        self.emit(f"add.u32 {index}, {prod}, {tid};")
        return index

    # -- rendering ------------------------------------------------------
    def _reg_decls(self) -> list:
        out = []
        order = ["%p", "%h", "%r", "%rd", "%f", "%fd"]
        types = {"%p": ".pred", "%h": ".b16", "%r": ".b32", "%rd": ".b64", "%f": ".f32",
                 "%fd": ".f64"}
        for prefix in order:
            n = self._counts.get(prefix, 0)
            if n:
                out.append(f".reg {types[prefix]} {prefix}<{n}>;")
        return out

    def render_module_decls(self) -> str:
        return "".join(d + "\n" for d in self._module)

    def render_entry(self) -> str:
        params = ",\n".join(f"    .param .u64 {self._params[n]}" for n in self._param_list)
        perf = ""
        if self.maxntid:
            perf += f".maxntid {self.maxntid}, 1, 1\n"
        if self.minnctapersm:
            perf += f".minnctapersm {self.minnctapersm}\n"
        if self.cluster:
            perf += f".reqnctapercluster {self.cluster}, 1, 1\n"
        parts = [f".visible .entry {self.name}(\n{params}\n)\n{perf}{{\n"]
        for d in self._reg_decls():
            parts.append(f"    {d}\n")
        for d in self._shared:
            parts.append(f"    {d}\n")
        if self._lines:
            parts.append("\n")
        for line in self._lines:
            if line.endswith(":"):
                parts.append(f"{line}\n")
            else:
                parts.append(f"    {line}\n")
        if not self._lines or self._lines[-1] != "ret;":
            parts.append("    ret;\n")
        parts.append("}\n")
        return "".join(parts)
