"""Elementwise f32 code generation shared by every template.

The op table follows the reference's operation names (reference
``compile.py:2462-2594``) with one deliberate difference: every add, subtract
and multiply carries an explicit ``.rn`` rounding modifier, so ptxas cannot
contract a multiply and an add into an FMA. Pointwise kernels are therefore
bit-identical to PyTorch-CPU / numpy float32 results.

Transcendentals use PTX's approximate unit instructions on a range reduction
written out here: ``exp(x) = ex2.approx(x * log2(e))`` and
``log(x) = lg2.approx(x) * ln(2)`` (the textbook base change), ``rsqrt`` is
``rsqrt.approx``; ``sqrt``, ``div`` and ``reciprocal`` use the IEEE
round-to-nearest instructions ``sqrt.rn``, ``div.rn``, ``rcp.rn``.
"""

from __future__ import annotations

from .analysis import ElemAccum, ElemLet, ElemLoad, ElemOp, ElemWrite, IDENTITY
from .ptx import f32_literal

LOG2E = "0f3FB8AA3B"     # log2(e) rounded to f32
LN2 = "0f3F317218"       # ln(2) rounded to f32

def emit_op(gen, op: str, args: list, dst: str | None = None) -> str:
    """Emit one f32 elementwise op; returns the destination register."""
    op = op.lower()
    d = dst or gen.register(".f32")
    e = gen.emit
    if len(args) == 1:
        a = args[0]
        if op in ("exp", "exponential"):
            t = gen.register(".f32")
            e(f"mul.rn.f32 {t}, {a}, {LOG2E};")
            e(f"ex2.approx.f32 {d}, {t};")
        elif op == "exp2":
            e(f"ex2.approx.f32 {d}, {a};")
        elif op in ("reciprocal", "recip"):
            e(f"rcp.rn.f32 {d}, {a};")
        elif op in ("log", "ln"):
            t = gen.register(".f32")
            e(f"lg2.approx.f32 {t}, {a};")
            e(f"mul.rn.f32 {d}, {t}, {LN2};")
        elif op == "log2":
            e(f"lg2.approx.f32 {d}, {a};")
        elif op in ("square", "sqr"):
            e(f"mul.rn.f32 {d}, {a}, {a};")
        elif op in ("relu", "relu_", "positive"):
            e(f"max.NaN.f32 {d}, {a}, 0f00000000;")
        elif op in ("neg", "negative"):
            e(f"neg.f32 {d}, {a};")
        elif op in ("identity", "clone", "copy"):
            e(f"mov.f32 {d}, {a};")
        elif op in ("abs", "absolute"):
            e(f"abs.f32 {d}, {a};")
        elif op in ("sqrt", "square_root"):
            e(f"sqrt.rn.f32 {d}, {a};")
        elif op in ("rsqrt", "reciprocal_sqrt"):
            e(f"rsqrt.approx.f32 {d}, {a};")
        elif op == "tanh":
            e(f"tanh.approx.f32 {d}, {a};")
        elif op in ("sigmoid", "silu"):
            # sigmoid(x) = 1 / (1 + 2^(-x*log2 e))
            t = gen.register(".f32")
            e(f"mul.rn.f32 {t}, {a}, 0fBFB8AA3B;")
            e(f"ex2.approx.f32 {t}, {t};")
            e(f"add.rn.f32 {t}, {t}, 0f3F800000;")
            if op == "sigmoid":
                e(f"rcp.rn.f32 {d}, {t};")
            else:
                e(f"div.rn.f32 {d}, {a}, {t};")
        else:
            raise NotImplementedError(f"Unsupported unary elementwise operation: {op}")
        return d
    if len(args) == 2:
        a, b = args
        if op in ("add", "sum"):
            e(f"add.rn.f32 {d}, {a}, {b};")
        elif op in ("subtract", "sub"):
            e(f"sub.rn.f32 {d}, {a}, {b};")
        elif op in ("multiply", "mul"):
            e(f"mul.rn.f32 {d}, {a}, {b};")
        elif op in ("maximum", "max"):
            e(f"max.NaN.f32 {d}, {a}, {b};")
        elif op in ("minimum", "min"):
            e(f"min.NaN.f32 {d}, {a}, {b};")
        elif op in ("divide", "div", "true_divide"):
            e(f"div.rn.f32 {d}, {a}, {b};")
        else:
            raise NotImplementedError(f"Unsupported binary elementwise operation: {op}")
        return d
    raise NotImplementedError(f"Unsupported arity {len(args)} for elementwise operation {op}")


def identity_literal(op: str) -> str:
    if op not in IDENTITY:
        raise NotImplementedError(f"no identity for accumulate op {op!r}")
    v = IDENTITY[op]
    if v == float("inf"):
        return "0f7F800000"
    if v == float("-inf"):
        return "0fFF800000"
    return f32_literal(v)


def run_program(gen, program, env: dict, *, load=None, write=None, accum_regs=None,
                lets=None, accum=None):
    """Emit an element program.

    ``env`` maps SSA names to registers and is updated in place. ``load(p)``
    returns the register for an :class:`ElemLoad`; ``write(p, reg)`` stores an
    :class:`ElemWrite`. ``accum_regs`` maps accumulator names to their
    carried registers, updated by :class:`ElemAccum` entries; a program may read
    an accumulator before its ``Accum`` statement (the online-softmax update).
    ``accum(p, base, value, acc)``, when given, emits the update of accumulator
    ``acc`` instead of the plain accumulate op (a compensated sum).
    """
    if accum_regs:
        for name, reg in accum_regs.items():
            env.setdefault(name, reg)
    for p in program:
        if isinstance(p, ElemLoad):
            env[p.name] = load(p)
        elif isinstance(p, ElemLet):
            if lets is not None and p.name in lets:
                env[p.name] = lets[p.name]
            else:
                r = gen.register(".f32")
                gen.emit(f"mov.f32 {r}, {f32_literal(p.value)};")
                env[p.name] = r
        elif isinstance(p, ElemOp):
            try:
                args = [env[a] for a in p.args]
            except KeyError as exc:
                raise ValueError(f"undefined elementwise input {exc.args[0]!r}") from None
            env[p.name] = emit_op(gen, p.op, args)
        elif isinstance(p, ElemAccum):
            acc = accum_regs[p.name]
            base = env[p.base] if p.base is not None else acc
            if accum is not None:
                accum(p, base, env[p.value], acc)
            else:
                emit_op(gen, p.op, [base, env[p.value]], dst=acc)
            env[p.name] = acc
        elif isinstance(p, ElemWrite):
            write(p, env[p.value])
        else:
            raise TypeError(p)
    return env
