"""General statement walker: lowers any Tile body statement by statement.

This is the fallback for bodies no sm_100a template lifts. It keeps the IR's
own schedule (one cell per thread, the IR's loops, shared arrays, cp.async
copies and barriers) and translates each statement kind directly, covering
the whole working vocabulary of the IR reference (reference
``TASK.md:89-187``): ``Tile, Load, Assign, Let, Init, Accum, Loop,
StridedLoop, Cond, Smem, Sync, CpAsyncCopy, CpAsyncCommit, CpAsyncWait,
Write (scalar, grouped, atomic), WarpShuffle, TreeHalve`` and the
expressions ``Var, Literal, BinaryExpr, TernaryExpr``.

Semantics follow the reference lowerer where the IR reference is silent
(reference ``compile.py:4858-5579``): the thread -> cell decode is row-major
over the Tile axes from ``%ctaid.x * %ntid.x + %tid.x``; an ``Accum`` starts
at its op's identity when a loop over one of its ``axes`` starts (unless the
name was declared by ``Init``); ``base`` replaces the previous value (the
online-softmax rescale). Differences by design: every f32 add/sub/mul is
``.rn`` (no FMA contraction), except that a product accumulated straight into an
add-``Accum`` (a dot-product step) becomes one ``fma.rn``; integer division is C-style ``div.s32``;
``TreeHalve`` folds the shared partials in each thread (a broadcast with no
extra barrier); leaf loops are unrolled whenever they are short, whatever
their ``unroll`` flag says.
"""

from __future__ import annotations

import math

from ..codegen import emit_op, identity_literal
from ..ir import dim_value, dtype_name, op_name, walk
from ..ptx import f32_literal
from .common import load_pointers

MAX_UNROLL = 64
MAX_UNROLL_STATEMENTS = 2048
SMEM_STATIC_LIMIT = 48 * 1024


def _value_uses(stmts) -> dict:
    """How many times each f32 value name is read anywhere in the kernel body."""
    uses = {}

    def use(name):
        if isinstance(name, str):
            uses[name] = uses.get(name, 0) + 1

    for s in walk(stmts):
        kind = type(s).__name__
        if kind == "Assign":
            for a in s.args:
                use(a)
        elif kind == "Accum":
            use(s.value)
            use(s.base)
        elif kind == "Write":
            for v in s.values:
                use(v)
        elif kind in ("WarpShuffle", "TreeHalve"):
            for v in tuple(s.state) + tuple(s.state_b):
                use(v)
            for c in s.combine_states:
                for a in getattr(c, "args", ()):
                    use(a)
    return uses


class _Walker:
    def __init__(self, gen, kernel):
        self.gen = gen
        self.kernel = kernel
        self.values = {}      # SSA name -> f32 register
        self.ints = {}        # integer names (axes, loop vars, Let ints) -> int | register
        self.carried = set()
        self.live_seeded = set()
        self.smem = {}        # name -> (base register or symbol, dims)
        self.shapes = {a: kernel.shape(a) for a in kernel.arg_order}
        self.ptrs = {}
        self.pool_used = 0
        self.pool = False
        self.uses = _value_uses(kernel.body)

    # -- integer expressions ------------------------------------------------
    def _reg_of(self, v):
        if isinstance(v, int):
            r = self.gen.register(".s32")
            self.gen.emit(f"mov.s32 {r}, {v};")
            return r
        return v

    def iexpr(self, e):
        """Lower an integer/boolean expression: a Python int, a ``%r`` or a ``%p`` register."""
        k = type(e).__name__
        if k == "Literal":
            v = e.value
            if isinstance(v, bool):
                return int(v)
            if isinstance(v, int):
                return v
            raise NotImplementedError(f"non-integer literal {v!r} in an index expression")
        if k == "Var":
            if e.name in self.ints:
                return self.ints[e.name]
            raise NotImplementedError(f"Unknown index variable: {e.name}")
        if k == "BinaryExpr":
            return self._binary(e.op, self.iexpr(e.left), self.iexpr(e.right))
        if k == "TernaryExpr":
            c = self.iexpr(e.cond)
            a, b = self.iexpr(e.if_true), self.iexpr(e.if_false)
            if isinstance(c, int):
                return a if c else b
            if isinstance(a, int) and isinstance(b, int) and a == b:
                return a
            d = self.gen.register(".s32")
            self.gen.emit(f"selp.b32 {d}, {self._reg_of(a) if not isinstance(a, int) else a}, "
                          f"{self._reg_of(b) if not isinstance(b, int) else b}, {c};")
            return d
        raise NotImplementedError(f"Index expression: {k}")

    def _binary(self, op, a, b):
        gen = self.gen
        if isinstance(a, int) and isinstance(b, int):
            return _fold(op, a, b)
        if op in ("&&", "and", "||", "or"):
            pa = self._pred(a)
            pb = self._pred(b)
            d = gen.register(".pred")
            gen.emit(f"{'and' if op in ('&&', 'and') else 'or'}.pred {d}, {pa}, {pb};")
            return d
        cmp = {"<": "lt", "<=": "le", ">": "gt", ">=": "ge", "==": "eq", "!=": "ne"}
        if op in cmp:
            d = gen.register(".pred")
            ra = self._reg_of(a)
            gen.emit(f"setp.{cmp[op]}.s32 {d}, {ra}, {b};")
            return d
        # algebraic shortcuts keep unrolled index math small
        if op == "+" and b == 0:
            return a
        if op == "+" and a == 0:
            return b
        if op == "-" and b == 0:
            return a
        if op == "*" and (a == 0 or b == 0):
            return 0
        if op == "*" and b == 1:
            return a
        if op == "*" and a == 1:
            return b
        if op in ("/", "//") and b == 1:
            return a
        if op == "%" and b == 1:
            return 0
        inst = {"+": "add.s32", "-": "sub.s32", "*": "mul.lo.s32", "/": "div.s32",
                "//": "div.s32", "%": "rem.s32"}.get(op)
        if inst is None:
            raise NotImplementedError(f"Index operator: {op}")
        d = gen.register(".s32")
        if isinstance(a, int):
            if op in ("+", "*"):
                a, b = b, a
            else:
                a = self._reg_of(a)
        gen.emit(f"{inst} {d}, {a}, {b};")
        return d

    def _pred(self, v):
        if isinstance(v, int):
            p = self.gen.register(".pred")
            self.gen.emit(f"setp.ne.s32 {p}, {self._reg_of(v)}, 0;")
            return p
        if v.startswith("%p"):
            return v
        p = self.gen.register(".pred")
        self.gen.emit(f"setp.ne.s32 {p}, {v}, 0;")
        return p

    def flat(self, index, dims):
        idx = list(index)
        dims = tuple(dims)
        if not idx:
            return 0
        if len(idx) != len(dims):
            if len(idx) == 1:
                dims = (math.prod(dims),)
            else:
                raise NotImplementedError("index rank does not match the buffer")
        out = 0
        for e, d in zip(idx, dims):
            out = self._binary("+", self._binary("*", out, d), self.iexpr(e))
        return out

    def address(self, base, flat, offset=0, shared=False):
        """``base + 4*flat``; returns an operand string ``[reg+imm]``."""
        gen = self.gen
        if isinstance(flat, int):
            return f"[{base}+{4 * (flat + offset)}]"
        if shared:
            o = gen.register(".u32")
            gen.emit(f"shl.b32 {o}, {flat}, 2;")
            a = gen.register(".u32")
            gen.emit(f"add.u32 {a}, {base}, {o};")
        else:
            o = gen.register(".s64")
            gen.emit(f"mul.wide.s32 {o}, {flat}, 4;")
            a = gen.register(".u64")
            gen.emit(f"add.s64 {a}, {base}, {o};")
        return f"[{a}+{4 * offset}]"

    # -- statements ---------------------------------------------------------
    def body(self, stmts):
        stmts = list(stmts)
        i = 0
        while i < len(stmts):
            s = stmts[i]
            if i + 1 < len(stmts) and self._fusable(s, stmts[i + 1]):
                self._accum_fma(stmts[i + 1], s)
                i += 2
                continue
            getattr(self, "s_" + type(s).__name__, self._unsupported)(s)
            i += 1

    def _fusable(self, s, nxt):
        """``v = multiply(a, b)`` immediately accumulated by an add-``Accum`` that is v's only
        reader: a dot-product step, lowered as one ``fma.rn`` (one rounding instead of two;
        f32 accumulations are checked against tolerances, and pointwise bodies, which must
        round every op, contain no ``Accum``)."""
        return (type(s).__name__ == "Assign" and type(nxt).__name__ == "Accum"
                and op_name(s.op) in ("multiply", "mul") and len(s.args) == 2
                and dtype_name(s.dtype) in (None, "f32")
                and op_name(nxt.op) in ("add", "sum") and nxt.value == s.name
                and self.uses.get(s.name, 0) == 1 and s.name not in self.carried
                and s.name != nxt.name and nxt.base != s.name)

    def _accum_fma(self, acc, mul):
        a, b = (self._f32(x) for x in mul.args)
        r = self.values.get(acc.name)
        if r is None:
            r = self.gen.register(".f32")
            self.gen.emit(f"mov.f32 {r}, {identity_literal('add')};")
            self.values[acc.name] = r
        prev = self._f32(acc.base) if acc.base is not None else r
        self.gen.emit(f"fma.rn.f32 {r}, {a}, {b}, {prev};")

    def _unsupported(self, s):
        raise NotImplementedError(f"General lowering does not support {type(s).__name__}")

    def s_Tile(self, t):
        raise NotImplementedError("nested Tile")

    def _f32(self, name):
        if name not in self.values:
            raise ValueError(f"undefined value {name!r}")
        return self.values[name]

    def s_Load(self, s):
        if dtype_name(s.dtype) not in (None, "f32"):
            raise NotImplementedError(f"Load of {dtype_name(s.dtype)}")
        gen = self.gen
        if s.input in self.smem:
            base, dims = self.smem[s.input]
            flat = self.flat(s.index, dims)
            for j, nm in enumerate(s.names):
                r = gen.register(".f32")
                gen.emit(f"ld.shared.f32 {r}, {self.address(base, flat, j, shared=True)};")
                self.values[nm] = r
            return
        if s.input not in self.ptrs:
            raise ValueError(f"Unknown buffer: {s.input}")
        flat = self.flat(s.index, self.shapes[s.input])
        for j, nm in enumerate(s.names):
            r = gen.register(".f32")
            gen.emit(f"ld.global.f32 {r}, {self.address(self.ptrs[s.input], flat, j)};")
            self.values[nm] = r

    def s_Assign(self, s):
        if dtype_name(s.dtype) not in (None, "f32"):
            raise NotImplementedError(f"Assign of {dtype_name(s.dtype)} (only f32 assignments)")
        args = [self._f32(a) for a in s.args]
        if s.name in self.carried and s.name in self.values:
            emit_op(self.gen, op_name(s.op), args, dst=self.values[s.name])
        else:
            self.values[s.name] = emit_op(self.gen, op_name(s.op), args)

    def s_Let(self, s):
        v = s.value
        if type(v).__name__ == "Literal" and isinstance(v.value, float):
            r = self.gen.register(".f32")
            self.gen.emit(f"mov.f32 {r}, {f32_literal(v.value)};")
            self.values[s.name] = r
            return
        if dtype_name(s.dtype) == "f32" and type(v).__name__ == "Literal":
            r = self.gen.register(".f32")
            self.gen.emit(f"mov.f32 {r}, {f32_literal(float(v.value))};")
            self.values[s.name] = r
            return
        self.ints[s.name] = self.iexpr(v)

    def s_Init(self, s):
        r = self.gen.register(".f32")
        self.gen.emit(f"mov.f32 {r}, {f32_literal(float(s.identity))};")
        self.values[s.name] = r
        self.carried.add(s.name)

    def _seed(self, axis, stmts):
        started = []
        for st in walk(stmts):
            if type(st).__name__ == "Accum" and axis in tuple(st.axes) \
                    and st.name not in self.carried and st.name not in self.live_seeded:
                r = self.values.get(st.name)
                if r is None:
                    r = self.gen.register(".f32")
                    self.values[st.name] = r
                self.gen.emit(f"mov.f32 {r}, {identity_literal(op_name(st.op))};")
                self.live_seeded.add(st.name)
                started.append(st.name)
        return started

    def s_Accum(self, s):
        op = op_name(s.op)
        r = self.values.get(s.name)
        if r is None:
            r = self.gen.register(".f32")
            self.gen.emit(f"mov.f32 {r}, {identity_literal(op)};")
            self.values[s.name] = r
        prev = self._f32(s.base) if s.base is not None else r
        emit_op(self.gen, op, [prev, self._f32(s.value)], dst=r)

    def _loop(self, axis, start, step, end, body, unroll, seed):
        gen = self.gen
        started = self._seed(axis, body) if seed else []
        stmts = list(walk(body))
        inner = any(type(x).__name__ in ("Loop", "StridedLoop") for x in stmts)
        if isinstance(start, int) and isinstance(end, int):
            trips = len(range(start, end, step))
            if not inner and trips <= MAX_UNROLL and trips * len(stmts) <= MAX_UNROLL_STATEMENTS:
                for v in range(start, end, step):
                    self.ints[axis] = v
                    self.body(body)
                self.ints.pop(axis, None)
                for n in started:
                    self.live_seeded.discard(n)
                return
        ctr = gen.register(".s32")
        gen.emit(f"mov.s32 {ctr}, {start};")
        top, done = gen.new_label("loop"), gen.new_label("loopend")
        p = gen.register(".pred")
        gen.label(top)
        gen.emit(f"setp.ge.s32 {p}, {ctr}, {end};")
        gen.emit(f"@{p} bra {done};")
        self.ints[axis] = ctr
        self.body(body)
        gen.emit(f"add.s32 {ctr}, {ctr}, {step};")
        gen.emit(f"bra {top};")
        gen.label(done)
        self.ints.pop(axis, None)
        for n in started:
            self.live_seeded.discard(n)

    def s_Loop(self, s):
        self._loop(s.axis.name, 0, 1, dim_value(s.axis.extent), s.body, s.unroll, s.seed)

    def s_StridedLoop(self, s):
        start = self.iexpr(s.start)
        step = self.iexpr(s.step)
        if not isinstance(step, int) or step <= 0:
            raise NotImplementedError("Loop step must be a positive constant")
        end = dim_value(s.axis.extent) if s.end is None else self.iexpr(s.end)
        self._loop(s.axis.name, start, step, end, s.body, s.unroll, s.seed)

    def s_Cond(self, s):
        c = self.iexpr(s.cond)
        if isinstance(c, int):
            self.body(s.body if c else s.else_body)
            return
        p = self._pred(c)
        gen = self.gen
        l_else, l_end = gen.new_label("else"), gen.new_label("endif")
        gen.emit(f"@!{p} bra {l_else};")
        self.body(s.body)
        if s.else_body:
            gen.emit(f"bra {l_end};")
            gen.label(l_else)
            self.body(s.else_body)
            gen.label(l_end)
        else:
            gen.label(l_else)

    def s_Sync(self, s):
        if s.warp:
            self.gen.emit("bar.warp.sync -1;")
        elif s.count:
            self.gen.emit(f"bar.sync {int(s.barrier_id)}, {int(s.count)};")
        else:
            self.gen.emit(f"bar.sync {int(s.barrier_id or 0)};")

    def s_Smem(self, s):
        if s.name in self.smem:
            return
        if s.dtype not in ("float", "f32"):
            raise NotImplementedError("Only f32 shared arrays supported")
        dims = tuple(dim_value(e) for e in s.extents)
        count = math.prod(dims)
        align = max(int(s.align or 0), 4)
        base = self.gen.register(".u32")
        if self.pool:
            off = -(-self.pool_used // align) * align
            self.pool_used = off + 4 * count
            self.gen.emit(f"mov.u32 {base}, emmy_smem_pool;")
            if off:
                self.gen.emit(f"add.u32 {base}, {base}, {off};")
        else:
            self.gen.shared(s.name, ".f32", length=count, align=align)
            self.gen.emit(f"mov.u32 {base}, {s.name};")
        self.smem[s.name] = (base, dims)

    def s_CpAsyncCopy(self, s):
        if str(s.swizzle).upper() != "NONE":
            raise NotImplementedError("Swizzled cp.async is not supported")
        if s.nbytes not in (4, 8, 16):
            raise NotImplementedError("cp.async copies 4, 8 or 16 bytes")
        base, dims = self.smem[s.smem]
        coords = list(s.smem_index)
        if s.lane_index is not None:
            from ..ir import BinaryExpr
            coords = [BinaryExpr(op="+", left=c, right=l) for c, l in zip(coords, s.lane_index)]
        dflat = self.flat(coords, dims)
        sflat = self.flat(s.src_index, self.shapes[s.src])
        dst = self.address(base, dflat, 0, shared=True)
        src = self.address(self.ptrs[s.src], sflat, 0)
        cache = "cg" if s.nbytes == 16 else "ca"
        self.gen.emit(f"cp.async.{cache}.shared.global {dst}, {src}, {s.nbytes};")

    def s_CpAsyncCommit(self, s):
        self.gen.emit("cp.async.commit_group;")

    def s_CpAsyncWait(self, s):
        self.gen.emit(f"cp.async.wait_group {int(s.group)};")

    def s_Write(self, s):
        gen = self.gen
        if s.output in self.smem:
            base, dims = self.smem[s.output]
            flat = self.flat(s.index, dims)
            for j, v in enumerate(s.values):
                gen.emit(f"st.shared.f32 {self.address(base, flat, j, shared=True)}, "
                         f"{self._f32(v)};")
            return
        if s.output not in self.ptrs:
            raise ValueError(f"Unknown buffer: {s.output}")
        flat = self.flat(s.index, self.shapes[s.output])
        for j, v in enumerate(s.values):
            a = self.address(self.ptrs[s.output], flat, j)
            if s.atomic:
                gen.emit(f"red.global.add.f32 {a}, {self._f32(v)};")
            else:
                gen.emit(f"st.global.f32 {a}, {self._f32(v)};")

    def _combine(self, states, partners, program, other):
        env = {x: self._f32(x) for x in states}
        env.update(zip(partners, other))
        for a in program:
            env[a.name] = emit_op(self.gen, op_name(a.op), [env[x] for x in a.args])
        return [env[x] for x in states]

    def s_WarpShuffle(self, s):
        states, partners = list(s.state), list(s.state_b)
        off = int(s.length) // 2
        while off >= 1:
            other = []
            for x in states:
                o = self.gen.register(".f32")
                self.gen.emit(f"shfl.sync.bfly.b32 {o}, {self._f32(x)}, {off}, 31, -1;")
                other.append(o)
            new = self._combine(states, partners, s.combine_states, other)
            for x, r in zip(states, new):
                self.gen.emit(f"mov.f32 {self.values[x]}, {r};")
            off //= 2

    def s_TreeHalve(self, s):
        states, partners = list(s.state), list(s.state_b)
        bases = [self.smem[b][0] for b in s.bufs]
        for x, b in zip(states, bases):
            self.gen.emit(f"ld.shared.f32 {self.values[x]}, [{b}];")
        for i in range(1, int(s.length)):
            other = []
            for b in bases:
                o = self.gen.register(".f32")
                self.gen.emit(f"ld.shared.f32 {o}, [{b}+{4 * i}];")
                other.append(o)
            new = self._combine(states, partners, s.combine_states, other)
            for x, r in zip(states, new):
                self.gen.emit(f"mov.f32 {self.values[x]}, {r};")


def _fold(op, a, b):
    if op == "+":
        return a + b
    if op == "-":
        return a - b
    if op == "*":
        return a * b
    if op in ("/", "//"):
        q = abs(a) // abs(b)
        return q if (a >= 0) == (b > 0) else -q
    if op == "%":
        q = abs(a) // abs(b)
        q = q if (a >= 0) == (b > 0) else -q
        return a - b * q
    if op == "<":
        return int(a < b)
    if op == "<=":
        return int(a <= b)
    if op == ">":
        return int(a > b)
    if op == ">=":
        return int(a >= b)
    if op == "==":
        return int(a == b)
    if op == "!=":
        return int(a != b)
    if op in ("&&", "and"):
        return int(bool(a) and bool(b))
    if op in ("||", "or"):
        return int(bool(a) or bool(b))
    raise NotImplementedError(f"Index operator: {op}")


def _check_convergence(stmts, under=None):
    """Every thread of a CTA must reach each ``Sync`` (a CTA barrier) and every lane of a warp
    each ``WarpShuffle`` (its mask names all 32 lanes). A barrier or shuffle inside a ``Cond``,
    or inside a ``StridedLoop`` whose start, step or end names a variable (a trip count that
    can differ between threads), could leave the threads that skip it waiting forever, so such
    a body is refused rather than lowered. The IR forms seen so far keep them at the Tile's
    top level or in loops with constant bounds."""
    from ..analysis import _vars_in
    for s in stmts:
        kind = type(s).__name__
        if kind in ("Sync", "WarpShuffle") and under:
            raise NotImplementedError(f"{kind} inside {under}: not every thread is sure to "
                                      "reach it")
        if kind == "Cond":
            _check_convergence(s.body, "a Cond")
            _check_convergence(s.else_body, "a Cond")
        elif kind == "StridedLoop":
            varying = any(_vars_in(e) for e in (s.start, s.step, s.end) if e is not None)
            _check_convergence(s.body, under or ("a StridedLoop with variable bounds"
                                                 if varying else None))
        elif kind in ("Loop", "Tile"):
            _check_convergence(s.body, under)


def lower_general(gen, kernel):
    body = kernel.body
    if len(body) != 1 or type(body[0]).__name__ != "Tile":
        kinds = ", ".join(type(s).__name__ for s in body) or "nothing"
        raise NotImplementedError(f"kernel body must be a single Tile, got {kinds}")
    tile = body[0]
    if getattr(tile, "aux_threads", 0):
        raise NotImplementedError("Auxiliary threads are not supported")
    launch = kernel.launch
    block = list(launch.get("block", [1, 1, 1]))
    grid = list(launch.get("grid", [1, 1, 1]))
    if block[1:] != [1, 1] or grid[1:] != [1, 1]:
        raise NotImplementedError("general lowering needs a 1-D launch")
    B = block[0]
    axes = [(a.name, dim_value(a.extent)) for a in tile.axes]
    cells = math.prod(e for _, e in axes)
    cooperative = any(type(x).__name__ in ("Sync", "WarpShuffle", "TreeHalve", "Smem",
                                            "CpAsyncCopy") for x in walk(tile.body))
    if cooperative and cells % B:
        raise NotImplementedError("cooperative Tile whose cells do not fill whole CTAs")
    # the shuffles name all 32 lanes: a CTA that ends in a partial warp would have them wait
    # on lanes that do not exist
    if B % 32 and any(type(x).__name__ == "WarpShuffle" or (type(x).__name__ == "Sync"
                                                          and x.warp)
                      for x in walk(tile.body)):
        raise NotImplementedError(f"WarpShuffle needs whole warps; the launch has {B} threads "
                                  "per CTA")
    for x in walk(tile.body):           # a barrier waits for its count of threads
        if type(x).__name__ == "Sync" and not x.warp:
            bid, count = int(x.barrier_id or 0), x.count
            if not 0 <= bid <= 15:
                raise NotImplementedError(f"barrier id {bid} outside the 16 CTA barriers")
            if count and (int(count) % 32 or not 0 < int(count) <= B):
                raise NotImplementedError(f"barrier count {count} is not a whole number of "
                                          f"warps within the {B}-thread CTA")
    _check_convergence(tile.body)

    w = _Walker(gen, kernel)
    w.ptrs = load_pointers(gen, list(kernel.arg_order))
    # shared memory: static declarations, or the dynamic pool when meta provides it
    total = 0
    for st in walk(tile.body):
        if type(st).__name__ == "Smem":
            al = max(int(st.align or 0), 4)
            total = -(-total // al) * al + 4 * math.prod(dim_value(e) for e in st.extents)
    provided = int(launch.get("smem_bytes", 0) or 0)
    if total > SMEM_STATIC_LIMIT or (total and provided >= total):
        if provided < total:
            raise NotImplementedError("shared arrays exceed 48 KiB without dynamic smem")
        gen.module_decl(".extern .shared .align 16 .b8 emmy_smem_pool[];")
        w.pool = True

    tid, cta, flat = (gen.register(".s32") for _ in range(3))
    gen.emit(f"mov.u32 {tid}, %tid.x;")
    gen.emit(f"mov.u32 {cta}, %ctaid.x;")
    gen.emit(f"mad.lo.s32 {flat}, {cta}, {B}, {tid};")
    lane, warp = gen.register(".s32"), gen.register(".s32")
    gen.emit(f"and.b32 {lane}, {tid}, 31;")
    gen.emit(f"shr.u32 {warp}, {tid}, 5;")
    w.ints.update({"lane": lane, "warp": warp})
    end = gen.new_label("tile_end")
    p = gen.register(".pred")
    gen.emit(f"setp.ge.s32 {p}, {flat}, {cells};")
    gen.emit(f"@{p} bra {end};")
    rem = flat
    for i, (name, extent) in enumerate(reversed(axes)):
        if extent == 1:
            w.ints[name] = 0
        elif i == len(axes) - 1:
            w.ints[name] = rem
        else:
            r = gen.register(".s32")
            gen.emit(f"rem.s32 {r}, {rem}, {extent};")
            q = gen.register(".s32")
            gen.emit(f"div.s32 {q}, {rem}, {extent};")
            w.ints[name] = r
            rem = q
    w.body(tile.body)
    gen.label(end)
    gen.emit("ret;")
