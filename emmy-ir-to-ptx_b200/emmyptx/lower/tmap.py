"""Tensor maps for TMA loads, written by the runtime at launch time.

The reference's PTX ABI passes only pointers (reference ``compile.py:5860-5879``: one
``.param .u64`` per ``arg_order`` entry), so a kernel cannot receive a ``CUtensorMap``
argument. A template that wants TMA declares three module globals instead:

* ``emmy_tmap_desc`` (``.u32``, initialised): what to encode, one record per map;
* ``emmy_tmap`` (128 bytes per map, 128-aligned): the encoded maps;
* ``emmy_tmap_key`` (``.u64`` per map, zero at load): the pointer each map was encoded for.

``libemmyrt`` reads the table when it loads the module and, before each launch whose
pointers differ from the keys, encodes the maps with ``cuTensorMapEncodeTiled`` and copies
maps and keys in front of the kernel on the launch stream. The kernel compares every key with
its own parameter and takes the TMA path only when all of them match; with any other runner
the keys stay zero and the kernel keeps its register-staged loads, so the PTX stays a drop-in.

Record layout (``TMAP_WORDS`` words per map, after the two header words
``TMAP_MAGIC, count``): parameter index, rank, five dims, four 64-bit byte strides as
(lo, hi) pairs, five box dims, swizzle (``CUtensorMapSwizzle``), data type
(``CUtensorMapDataType``), L2 promotion (``CUtensorMapL2promotion``), and a reserved word.
"""

from __future__ import annotations

TMAP_MAGIC = 0x454D5401
TMAP_WORDS = 24
MAX_MAPS = 4
SWIZZLE_128B_ATOM_32B = 4       # CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B
DTYPE_FLOAT32 = 7               # CU_TENSOR_MAP_DATA_TYPE_FLOAT32
L2_PROMOTION_256B = 3           # CU_TENSOR_MAP_L2_PROMOTION_L2_256B


def record(param, dims, strides, box, swizzle=SWIZZLE_128B_ATOM_32B, dtype=DTYPE_FLOAT32,
           l2=L2_PROMOTION_256B):
    """One map's record. ``dims`` and ``box`` run innermost first; ``strides`` are the byte
    strides of dims 1.. (the innermost is contiguous)."""
    rank = len(dims)
    if not 1 <= rank <= 5 or len(box) != rank or len(strides) != rank - 1:
        raise ValueError("tensor map rank, box and strides disagree")
    if any(s % 16 for s in strides):
        raise ValueError("tensor map strides must be multiples of 16 bytes")
    if any(not 1 <= b <= 256 for b in box):
        raise ValueError("tensor map box dims must be within 1..256")
    words = [int(param), rank]
    words += [int(d) for d in dims] + [1] * (5 - rank)
    for s in list(strides) + [0] * (4 - len(strides)):
        words += [s & 0xFFFFFFFF, s >> 32]
    words += [int(b) for b in box] + [1] * (5 - rank)
    words += [swizzle, dtype, l2, 0]
    assert len(words) == TMAP_WORDS
    return words


def declare(gen, records):
    """Declare the descriptor table, the maps and their keys; returns nothing (the kernel
    addresses them by name)."""
    if not 1 <= len(records) <= MAX_MAPS:
        raise ValueError("between 1 and 4 tensor maps per module")
    words = [TMAP_MAGIC, len(records)] + [w for r in records for w in r]
    init = ", ".join(str(w) for w in words)
    gen.module_decl(f".global .align 128 .b8 emmy_tmap[{128 * len(records)}];")
    gen.module_decl(f".global .align 8 .u64 emmy_tmap_key[{len(records)}];")
    gen.module_decl(f".global .align 4 .u32 emmy_tmap_desc[{len(words)}] = {{{init}}};")
    gen.module_decl(".global .align 4 .u32 emmy_path;")


def keys_match(gen, raws):
    """A predicate true when ``emmy_tmap_key[i]`` equals the raw parameter ``raws[i]`` for
    every map (L2-coherent loads: the keys are written between launches)."""
    p = None
    for i, raw in enumerate(raws):
        k = gen.register(".u64")
        gen.emit(f"ld.global.cg.u64 {k}, [emmy_tmap_key+{8 * i}];")
        q = gen.register(".pred")
        if p is None:
            gen.emit(f"setp.eq.u64 {q}, {k}, {raw};")
        else:
            gen.emit(f"setp.eq.and.u64 {q}, {k}, {raw}, {p};")
        p = q
    nz = gen.register(".pred")
    gen.emit(f"setp.ne.and.u64 {nz}, {raws[0]}, 0, {p};")
    return nz


def map_address(gen, index):
    """Generic address of map ``index`` in a fresh ``.u64`` register."""
    a, g = gen.register(".u64"), gen.register(".u64")
    gen.emit(f"mov.u64 {a}, emmy_tmap;")
    gen.emit(f"cvta.global.u64 {g}, {a};")
    if index:
        gen.emit(f"add.s64 {g}, {g}, {128 * index};")
    return g
