"""Helpers shared by the sm_100a lowering templates."""

from __future__ import annotations

WAIT_LIMIT = 1 << 24          # try_wait iterations before a bounded wait gives up


def load_pointers(gen, names) -> dict:
    """``ld.param`` each buffer pointer and convert it to a global address."""
    ptrs = {}
    for name in names:
        raw = gen.register(".u64")
        g = gen.register(".u64")
        gen.emit(f"ld.param.u64 {raw}, [{gen.parameter(name)}];")
        gen.emit(f"cvta.to.global.u64 {g}, {raw};")
        ptrs[name] = g
    return ptrs


def aligned_predicate(gen, ptrs, names, align=16) -> str:
    """A predicate that is true when every pointer in ``names`` is ``align``-byte aligned."""
    acc = gen.register(".u64")
    gen.emit(f"mov.u64 {acc}, 0;")
    for n in names:
        gen.emit(f"or.b64 {acc}, {acc}, {ptrs[n]};")
    low = gen.register(".u64")
    gen.emit(f"and.b64 {low}, {acc}, {align - 1};")
    p = gen.register(".pred")
    gen.emit(f"setp.eq.u64 {p}, {low}, 0;")
    return p


def addr(gen, base, index_u32, scale=4) -> str:
    """``base + index * scale`` as a 64-bit address (index is an unsigned 32-bit register)."""
    off = gen.register(".u64")
    gen.emit(f"mul.wide.u32 {off}, {index_u32}, {scale};")
    a = gen.register(".u64")
    gen.emit(f"add.s64 {a}, {base}, {off};")
    return a


def tf32_split(gen, x) -> tuple:
    """3xTF32 operand split of the f32 register ``x`` on the integer and FMA pipes.

    ``hi`` is ``x`` with its 13 low mantissa bits cleared (a TF32 value, one ``and``), and
    ``lo = x - hi`` is exact in f32 with at most 13 significant bits; the tensor core reads
    lo's top 10 mantissa bits. The products hi*hi + hi*lo + lo*hi then carry an error of
    about 2^-19 relative each (the dropped lo*lo and lo's own truncation), against 2^-21 when
    hi is rounded first, for two instructions per element instead of three.
    """
    h = gen.register(".b32")
    gen.emit(f"and.b32 {h}, {x}, -8192;")
    lo = gen.register(".f32")
    gen.emit(f"sub.rn.f32 {lo}, {x}, {h};")
    return h, lo


def pack2(gen, a, b) -> str:
    """The f32 pair (a, b) as one .b64 register (operand of the packed .f32x2 instructions)."""
    d = gen.register(".b64")
    gen.emit(f"mov.b64 {d}, {{{a}, {b}}};")
    return d


def unpack2(gen, d) -> tuple:
    a, b = gen.register(".f32"), gen.register(".f32")
    gen.emit(f"mov.b64 {{{a}, {b}}}, {d};")
    return a, b


def tf32_split_pairs(gen, xs) -> tuple:
    """:func:`tf32_split` of an even number of registers, the subtraction done two elements
    per instruction (``sub.rn.f32x2``, rounded per element exactly as ``sub.rn.f32``)."""
    his, los = [], []
    for x, y in zip(xs[0::2], xs[1::2]):
        hx, hy = gen.register(".b32"), gen.register(".b32")
        gen.emit(f"and.b32 {hx}, {x}, -8192;")
        gen.emit(f"and.b32 {hy}, {y}, -8192;")
        d = gen.register(".b64")
        gen.emit(f"sub.rn.f32x2 {d}, {pack2(gen, x, y)}, {pack2(gen, hx, hy)};")
        lx, ly = unpack2(gen, d)
        his += [hx, hy]
        los += [lx, ly]
    return his, los
