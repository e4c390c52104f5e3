"""Pointwise template: 128-bit vector loads/stores over a grid-stride loop.

The IR assigns ``U`` consecutive elements to each Tile cell and one cell to
each thread (reference ``problems/p00_scalar_add``..``p03_relu_mul``). On
B200 the template instead gives every thread whole 16-byte chunks: four
consecutive elements per ``ld.global.v4.f32`` / ``st.global.v4.f32``, so a
warp moves 512 contiguous bytes per instruction. Chunks are distributed over
*all* threads of the launch (``%nctaid.x * %ntid.x``) in a grid-stride loop,
which keeps the kernel correct for any grid/block in ``meta.json``, including
launches with more threads than cells (the Tile-extent guard of reference
``compile.py:2642-2669`` becomes the loop bound).

The leftover ``E mod 4`` elements, and any call whose buffers are not 16-byte
aligned, take a scalar path with the same arithmetic.

Overlapped launches: the kernel executes ``griddepcontrol.launch_dependents``
at entry, so a kernel launched after it with programmatic stream
serialization (``emmy_rt_launch_ex``, ``EMMY_RT_LAUNCH_OVERLAP``) can be
scheduled while this one runs, and ``griddepcontrol.wait`` before its first
global access, so it reads nothing before the previous kernel on the stream
has completed (a chain of pointwise kernels stays ordered). A small launch is
dominated by its fixed launch cost; overlapping consecutive launches hides it.
Under a plain launch both instructions do nothing.
"""

from __future__ import annotations

from ..analysis import ElemLoad
from ..codegen import run_program
from .common import addr, aligned_predicate, load_pointers


def lower_pointwise(gen, kernel, plan) -> None:
    E = plan.total
    V = E // 4
    buffers = list(dict.fromkeys(plan.inputs + plan.outputs + [b for b, _ in plan.uniforms]))
    ptrs = load_pointers(gen, [a for a in kernel.arg_order if a in buffers])
    written = set(plan.outputs)
    gen.emit("griddepcontrol.launch_dependents;")
    gen.emit("griddepcontrol.wait;")
    ld_elem = "ld.global.v4.f32" if written & set(plan.inputs) else \
        "ld.global.nc.L1::no_allocate.v4.f32"
    ld_scalar = "ld.global.f32" if written & set(plan.inputs) else "ld.global.nc.f32"

    # uniform (1-element constant) operands, loaded once per thread
    uniforms = {}
    for p in plan.program:
        if isinstance(p, ElemLoad) and p.kind == "uniform" and p.name not in uniforms:
            r = gen.register(".f32")
            off = p.offset * 4
            gen.emit(f"ld.global.nc.f32 {r}, [{ptrs[p.buffer]}+{off}];")
            uniforms[p.name] = r

    gtid = gen.thread_index_1d()
    nthr = gen.register(".u32")
    ncta = gen.register(".u32")
    ntid = gen.register(".u32")
    gen.emit(f"mov.u32 {ncta}, %nctaid.x;")
    gen.emit(f"mov.u32 {ntid}, %ntid.x;")
    gen.emit(f"mul.lo.u32 {nthr}, {ncta}, {ntid};")

    scalar_start = gen.register(".u32")
    L_scalar = gen.new_label("scalar")
    L_end = gen.new_label("end")
    if V > 0:
        ok = aligned_predicate(gen, ptrs, [b for b in buffers if b in ptrs])
        gen.emit(f"mov.u32 {scalar_start}, {gtid};")
        gen.emit(f"@!{ok} bra {L_scalar};")
        v = gen.register(".u32")
        gen.emit(f"mov.u32 {v}, {gtid};")
        L_loop = gen.new_label("vec")
        L_vdone = gen.new_label("vecdone")
        pv = gen.register(".pred")
        gen.label(L_loop)
        gen.emit(f"setp.ge.u32 {pv}, {v}, {V};")
        gen.emit(f"@{pv} bra {L_vdone};")
        off = gen.register(".u64")
        gen.emit(f"mul.wide.u32 {off}, {v}, 16;")
        lanes = {}
        for b in plan.inputs:
            a = gen.register(".u64")
            gen.emit(f"add.s64 {a}, {ptrs[b]}, {off};")
            regs = gen.registers(".f32", 4)
            gen.emit(f"{ld_elem} {{{', '.join(regs)}}}, [{a}];")
            lanes[b] = regs
        results = {b: [None] * 4 for b in plan.outputs}
        for lane in range(4):
            def load(p, lane=lane):
                return uniforms[p.name] if p.kind == "uniform" else lanes[p.buffer][lane]

            def write(p, reg, lane=lane):
                results[p.buffer][lane] = reg
            run_program(gen, plan.program, {}, load=load, write=write)
        for b in plan.outputs:
            a = gen.register(".u64")
            gen.emit(f"add.s64 {a}, {ptrs[b]}, {off};")
            gen.emit(f"st.global.v4.f32 [{a}], {{{', '.join(results[b])}}};")
        gen.emit(f"add.u32 {v}, {v}, {nthr};")
        gen.emit(f"bra.uni {L_loop};")
        gen.label(L_vdone)
        gen.emit(f"add.u32 {scalar_start}, {gtid}, {V * 4};")
    else:
        gen.emit(f"mov.u32 {scalar_start}, {gtid};")

    # scalar path: the E mod 4 tail after the vector loop, or everything if misaligned
    gen.label(L_scalar)
    e = gen.register(".u32")
    gen.emit(f"mov.u32 {e}, {scalar_start};")
    L_sloop = gen.new_label("sloop")
    ps = gen.register(".pred")
    gen.label(L_sloop)
    gen.emit(f"setp.ge.u32 {ps}, {e}, {E};")
    gen.emit(f"@{ps} bra {L_end};")
    scal = {}
    for b in plan.inputs:
        a = addr(gen, ptrs[b], e)
        r = gen.register(".f32")
        gen.emit(f"{ld_scalar} {r}, [{a}];")
        scal[b] = r

    def sload(p):
        return uniforms[p.name] if p.kind == "uniform" else scal[p.buffer]

    def swrite(p, reg):
        a = addr(gen, ptrs[p.buffer], e)
        gen.emit(f"st.global.f32 [{a}], {reg};")
    run_program(gen, plan.program, {}, load=sload, write=swrite)
    gen.emit(f"add.u32 {e}, {e}, {nthr};")
    gen.emit(f"bra.uni {L_sloop};")
    gen.label(L_end)
    gen.emit("ret;")
