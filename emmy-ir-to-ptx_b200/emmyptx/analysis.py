"""Lift a scheduled Tile body into the kernel class it computes.

Emmy's Kernel IR is a thread-level schedule written for sm_89 (per-thread
unrolled cells, 128-thread cooperative rows, scalar FMA tiles). The B200
templates do not replay that schedule: they recover *what* the body computes
and lay the work out for sm_100a. This module does the recovery.

* :func:`affine` turns an index expression into ``{var: coeff, 1: const}``.
* :func:`lift_pointwise` recognises a one-cell-per-thread elementwise body
  whose loads and writes touch elements ``U*cell + k`` (reference
  ``compile.py:2642-2669`` walks the same bodies statement by statement).
* :func:`lift_rowreduce` recognises the cooperative reduction skeleton
  ``StridedLoop(Accum) -> WarpShuffle -> Smem -> Cond(lane==0) -> Sync ->
  TreeHalve -> scalars -> (Cond(co==0) Write | StridedLoop(Write))`` used for
  sum/mean, row sums, RMSNorm, softmax and L2-norm (reference
  ``compile.py:2703-4856``), with any elementwise program inside.

Both return ``None`` when the body is outside the recognised form; the
lowering then uses the general statement walker, which handles every
statement kind directly.
"""

from __future__ import annotations

from ._record import factory, record

from .ir import dim_value, dtype_name, op_name

ONE = 1  # key of the constant term in an affine map


# ---------------------------------------------------------------------------
# index expressions
# ---------------------------------------------------------------------------

def affine(expr, env=None):
    """``{var: coeff, ONE: const}`` for an integer index expression, or None.

    ``env`` maps names bound by ``Let`` to their own affine maps.
    """
    kind = type(expr).__name__
    if kind == "Literal":
        v = expr.value
        if type(v) is not int:
            return None
        return {ONE: v}
    if kind == "Var":
        if env and expr.name in env:
            return dict(env[expr.name])
        return {expr.name: 1}
    if kind == "BinaryExpr":
        left = affine(expr.left, env)
        right = affine(expr.right, env)
        if left is None or right is None:
            return None
        op = expr.op
        if op == "+":
            return _add(left, right, 1)
        if op == "-":
            return _add(left, right, -1)
        if op == "*":
            if set(left) == {ONE}:
                return _scale(right, left[ONE])
            if set(right) == {ONE}:
                return _scale(left, right[ONE])
            return None
        if op in ("/", "//", "%") and set(left) == {ONE} and set(right) == {ONE} and right[ONE]:
            a, b = left[ONE], right[ONE]
            if op == "%":
                return {ONE: _c_rem(a, b)}
            return {ONE: _c_div(a, b)}
        return None
    return None


def _c_div(a, b):
    q = abs(a) // abs(b)
    return q if (a >= 0) == (b > 0) else -q


def _c_rem(a, b):
    return a - b * _c_div(a, b)


def _add(a, b, sign):
    out = dict(a)
    for k, v in b.items():
        out[k] = out.get(k, 0) + sign * v
    return {k: v for k, v in out.items() if v or k == ONE}


def _scale(a, s):
    return {k: v * s for k, v in a.items() if v * s or k == ONE}


def flat_affine(index, shape, env=None):
    """Row-major flat element offset of a multi-dimensional index, as an affine map."""
    index = tuple(index)
    shape = tuple(shape)
    if not index:
        return {ONE: 0}
    if len(index) != len(shape):
        if len(index) == 1 and len(shape) > 1:
            shape = (1,) * 0 + (int(_prod(shape)),)
        else:
            return None
    out = {ONE: 0}
    stride = 1
    for expr, extent in reversed(list(zip(index, shape))):
        a = affine(expr, env)
        if a is None:
            return None
        out = _add(out, _scale(a, stride), 1)
        stride *= extent
    return out


def _prod(xs):
    p = 1
    for x in xs:
        p *= int(x)
    return p


def const_of(aff):
    """The value of a constant affine map, or None if it depends on a variable."""
    if aff is not None and set(aff) <= {ONE}:
        return aff.get(ONE, 0)
    return None


# ---------------------------------------------------------------------------
# element programs (SSA lists over one element / one row)
# ---------------------------------------------------------------------------

@record
class ElemLoad:
    name: str
    buffer: str
    kind: str          # 'elem' (element index), 'col' (column of a row), 'uniform' (fixed offset)
    offset: int = 0    # fixed offset for 'uniform'


@record
class ElemLet:
    name: str
    value: float


@record
class ElemOp:
    name: str
    op: str
    args: tuple


@record
class ElemAccum:
    name: str
    op: str
    value: str
    base: str | None


@record
class ElemWrite:
    buffer: str
    value: str
    kind: str          # 'elem' | 'row' (one value per row) | 'scalar'
    atomic: bool = False


IDENTITY = {"add": 0.0, "sum": 0.0, "maximum": float("-inf"), "max": float("-inf"),
            "minimum": float("inf"), "min": float("inf"), "multiply": 1.0, "mul": 1.0}


# ---------------------------------------------------------------------------
# pointwise
# ---------------------------------------------------------------------------

@record
class PointwisePlan:
    total: int                        # elements per buffer touched (E = cells * U)
    cells: int
    per_cell: int                     # U
    program: list                     # ElemLoad/ElemLet/ElemOp/ElemWrite over one element
    inputs: list                      # buffers loaded per element
    uniforms: list                    # (buffer, offset) loaded once
    outputs: list


def _tile_axes(tile):
    return [(a.name, dim_value(a.extent)) for a in tile.axes]


def _all_f32(stmts):
    """Every typed statement works on f32 (``Smem`` arrays are typed ``'float'``): the
    templates load, compute and store f32 only, so any other type is left to a lowering that
    refuses it by name."""
    for s in stmts:
        for attr in ("dtype", "value_dtype"):
            dt = getattr(s, attr, None)
            if dt is not None and (dt if isinstance(dt, str) else dtype_name(dt)) \
                    not in ("f32", "float"):
                return False
    return True


def lift_pointwise(kernel):
    body = kernel.body
    if len(body) != 1 or type(body[0]).__name__ != "Tile":
        return None
    tile = body[0]
    if getattr(tile, "aux_threads", 0):
        return None
    axes = _tile_axes(tile)
    if not axes:
        return None
    allowed = {"Load", "Assign", "Let", "Write"}
    if any(type(s).__name__ not in allowed for s in tile.body):
        return None
    cells = _prod(e for _, e in axes)
    # row-major flat cell index coefficients of each axis
    coeff = {}
    stride = 1
    for name, extent in reversed(axes):
        coeff[name] = stride
        stride *= extent

    shapes = {a: kernel.shape(a) for a in kernel.arg_order}

    def cell_form(aff):
        """(U, k) when aff == U*cell + k, ('uniform', c) when constant, else None."""
        c = const_of(aff)
        if c is not None:
            return ("uniform", c)
        vars_ = [k for k in aff if k != ONE]
        if set(vars_) - set(coeff):
            return None
        # every tile axis must appear with coefficient U * coeff[axis]
        u = None
        for name, _ in axes:
            got = aff.get(name, 0)
            if coeff[name] == 0:
                continue
            if got % coeff[name]:
                return None
            this = got // coeff[name]
            if u is None:
                u = this
            elif u != this:
                return None
        if not u or u <= 0:
            return None
        return (u, aff.get(ONE, 0))

    defs = {}          # name -> ('load', buf, k) | ('uload', buf, off) | ('let', v) | ('op', op, args)
    writes = []        # (buf, k, name)
    per_cell = None
    for stmt in tile.body:
        kind = type(stmt).__name__
        if kind == "Load":
            if dtype_name(stmt.dtype) not in (None, "f32") or stmt.input not in shapes:
                return None
            aff = flat_affine(stmt.index, shapes[stmt.input])
            form = cell_form(aff) if aff is not None else None
            if form is None:
                return None
            for j, nm in enumerate(stmt.names):
                if form[0] == "uniform":
                    defs[nm] = ("uload", stmt.input, form[1] + j)
                else:
                    if per_cell is None:
                        per_cell = form[0]
                    elif per_cell != form[0]:
                        return None
                    defs[nm] = ("load", stmt.input, form[1] + j)
        elif kind == "Let":
            v = stmt.value
            if type(v).__name__ != "Literal" or not isinstance(v.value, (int, float)):
                return None
            defs[stmt.name] = ("let", float(v.value))
        elif kind == "Assign":
            if dtype_name(stmt.dtype) not in (None, "f32"):
                return None
            defs[stmt.name] = ("op", op_name(stmt.op), tuple(stmt.args))
        elif kind == "Write":
            if stmt.atomic or dtype_name(stmt.value_dtype) not in (None, "f32") \
                    or stmt.output not in shapes:
                return None
            aff = flat_affine(stmt.index, shapes[stmt.output])
            form = cell_form(aff) if aff is not None else None
            if form is None or form[0] == "uniform":
                return None
            if per_cell is None:
                per_cell = form[0]
            elif per_cell != form[0]:
                return None
            for j, nm in enumerate(stmt.values):
                writes.append((stmt.output, form[1] + j, nm))
    if per_cell is None or not writes:
        return None
    U = per_cell
    total = cells * U

    # element tree of each written value, relative to its own element offset
    def tree(name, k, depth=0):
        if depth > 256 or name not in defs:
            raise KeyError(name)
        d = defs[name]
        if d[0] == "load":
            if d[2] != k:
                raise KeyError(name)      # reads a different element: not elementwise
            return ("load", d[1])
        if d[0] == "uload":
            return ("uload", d[1], d[2])
        if d[0] == "let":
            return ("let", d[1])
        return ("op", d[1]) + tuple(tree(a, k, depth + 1) for a in d[2])

    out_trees = {}
    seen = {}
    try:
        for buf, k, nm in writes:
            if not (0 <= k < U):
                return None
            t = tree(nm, k)
            seen.setdefault(buf, set())
            if k in seen[buf]:
                return None
            seen[buf].add(k)
            if buf in out_trees and out_trees[buf] != t:
                return None
            out_trees[buf] = t
    except KeyError:
        return None
    for buf, ks in seen.items():
        if ks != set(range(U)):
            return None

    # flatten the trees into one SSA program with common subexpressions shared
    program, inputs, uniforms = [], [], []
    memo = {}

    def emit(t):
        if t in memo:
            return memo[t]
        if t[0] == "load":
            nm = f"e_{t[1]}"
            program.append(ElemLoad(nm, t[1], "elem"))
            if t[1] not in inputs:
                inputs.append(t[1])
        elif t[0] == "uload":
            nm = f"u_{t[1]}_{t[2]}"
            program.append(ElemLoad(nm, t[1], "uniform", t[2]))
            uniforms.append((t[1], t[2]))
        elif t[0] == "let":
            nm = f"c{len(memo)}"
            program.append(ElemLet(nm, t[1]))
        else:
            args = tuple(emit(a) for a in t[2:])
            nm = f"t{len(memo)}"
            program.append(ElemOp(nm, t[1], args))
        memo[t] = nm
        return nm

    outputs = []
    for buf, t in out_trees.items():
        program.append(ElemWrite(buf, emit(t), "elem"))
        outputs.append(buf)
    for buf in inputs + outputs:
        if _prod(shapes[buf]) < total:
            return None
    return PointwisePlan(total=total, cells=cells, per_cell=U, program=program, inputs=inputs,
                         uniforms=uniforms, outputs=outputs)


# ---------------------------------------------------------------------------
# cooperative reductions (full, per-row, fused row ops)
# ---------------------------------------------------------------------------

@record
class RowReducePlan:
    rows: int                  # 1 for a full reduction
    length: int                # elements reduced per row
    threads: int               # cooperating threads per row in the IR schedule
    full: bool                 # single global result (rows == 1, one co axis)
    states: list               # accumulator names in WarpShuffle order
    state_ops: dict            # state -> accumulate op (identity source)
    pass1: list                # element program with ElemAccum entries
    combine: list              # ElemOp program over (state, state_b) -> state
    partner: dict              # state -> its partner name in the combine program
    post: list                 # scalar program after the block combine
    pass2: list | None         # element program writing a row (fused ops)
    final: list                # scalar program + ElemWrite of the reduced value(s)
    row_buffers: list = factory(list)   # buffers read as x[row, j]
    col_buffers: list = factory(list)   # buffers read as w[j]
    out_buffers: list = factory(list)


def _is_var(expr, name):
    return type(expr).__name__ == "Var" and expr.name == name


def _cond_eq(cond, var, value):
    return (type(cond).__name__ == "BinaryExpr" and cond.op == "=="
            and _is_var(cond.left, var) and type(cond.right).__name__ == "Literal"
            and cond.right.value == value)


def lift_rowreduce(kernel):
    body = kernel.body
    if len(body) != 1 or type(body[0]).__name__ != "Tile":
        return None
    tile = body[0]
    if getattr(tile, "aux_threads", 0):
        return None
    axes = _tile_axes(tile)
    stmts = list(tile.body)
    kinds = [type(s).__name__ for s in stmts]
    if "StridedLoop" not in kinds or "WarpShuffle" not in kinds or "TreeHalve" not in kinds:
        return None
    if len(axes) == 1:
        co, threads = axes[0]
        row_var, rows = None, 1
    elif len(axes) == 2:
        (row_var, rows), (co, threads) = axes
    else:
        return None
    if tile.block_threads not in (None, threads):
        return None
    shapes = {a: kernel.shape(a) for a in kernel.arg_order}

    i = 0
    # optional uniform prologue is not part of the fixture grammar; require the loop first
    if kinds[i] != "StridedLoop":
        return None
    loop = stmts[i]
    i += 1
    length = dim_value(loop.axis.extent)
    if not _is_var(loop.start, co) or const_of(affine(loop.step)) != threads:
        return None
    if loop.end is not None:
        return None
    jvar = loop.axis.name

    def load_kind(stmt, jname):
        shp = shapes.get(stmt.input)
        if shp is None:
            return None
        aff = flat_affine(stmt.index, shp)
        if aff is None:
            return None
        c = const_of(aff)
        if c is not None:
            return ("uniform", c)
        keys = set(aff) - {ONE}
        if aff.get(ONE, 0) != 0:
            return None
        if row_var is not None and keys == {row_var, jname} and aff[jname] == 1 \
                and aff[row_var] == length:
            return ("elem",)
        if keys == {jname} and aff[jname] == 1:
            if row_var is None:
                return ("elem",)
            if _prod(shp) == length:
                return ("col",)
        return None

    def element_program(stmts_, jname, allow_accum, allow_write):
        prog = []
        for s in stmts_:
            k = type(s).__name__
            if k == "Load":
                if dtype_name(s.dtype) not in (None, "f32") or len(s.names) != 1:
                    return None
                lk = load_kind(s, jname)
                if lk is None:
                    return None
                if lk[0] == "uniform":
                    prog.append(ElemLoad(s.names[0], s.input, "uniform", lk[1]))
                else:
                    prog.append(ElemLoad(s.names[0], s.input, lk[0]))
            elif k == "Let":
                v = s.value
                if type(v).__name__ != "Literal" or not isinstance(v.value, (int, float)):
                    return None
                prog.append(ElemLet(s.name, float(v.value)))
            elif k == "Assign":
                if dtype_name(s.dtype) not in (None, "f32"):
                    return None
                prog.append(ElemOp(s.name, op_name(s.op), tuple(s.args)))
            elif k == "Accum" and allow_accum:
                if dtype_name(s.dtype) not in (None, "f32"):
                    return None
                prog.append(ElemAccum(s.name, op_name(s.op), s.value, s.base))
            elif k == "Write" and allow_write:
                if s.atomic or len(s.values) != 1 or s.output not in shapes:
                    return None
                aff = flat_affine(s.index, shapes[s.output])
                if aff is None or aff.get(ONE, 0) != 0:
                    return None
                keys = set(aff) - {ONE}
                ok = (row_var is not None and keys == {row_var, jname} and aff[jname] == 1
                      and aff[row_var] == length) or \
                     (row_var is None and keys == {jname} and aff[jname] == 1)
                if not ok:
                    return None
                prog.append(ElemWrite(s.output, s.values[0], "elem"))
            else:
                return None
        return prog

    pass1 = element_program(loop.body, jvar, True, False)
    if pass1 is None:
        return None
    accums = [p for p in pass1 if isinstance(p, ElemAccum)]
    if not accums:
        return None

    if i >= len(stmts) or kinds[i] != "WarpShuffle":
        return None
    ws = stmts[i]
    i += 1
    states = list(ws.state)
    partners = list(ws.state_b)
    if ws.length != 32 or len(states) != len(partners) or not states:
        return None
    state_ops = {}
    for s in states:
        ops = {a.op for a in accums if a.name == s}
        if len(ops) != 1:
            return None
        state_ops[s] = ops.pop()
        if state_ops[s] not in IDENTITY:
            return None
    combine = []
    for a in ws.combine_states:
        if type(a).__name__ != "Assign":
            return None
        combine.append(ElemOp(a.name, op_name(a.op), tuple(a.args)))

    # Smem declarations, the lane-0 partial store, the barrier, the tree
    while i < len(stmts) and kinds[i] == "Smem":
        i += 1
    if i >= len(stmts) or kinds[i] != "Cond" or not _cond_eq(stmts[i].cond, "lane", 0):
        return None
    i += 1
    if i >= len(stmts) or kinds[i] != "Sync":
        return None
    i += 1
    if i >= len(stmts) or kinds[i] != "TreeHalve":
        return None
    th = stmts[i]
    i += 1
    if list(th.state) != states:
        return None
    th_combine = [ElemOp(a.name, op_name(a.op), tuple(a.args)) for a in th.combine_states]
    if th_combine != combine:
        return None

    post, pass2, final = [], None, []
    rest = stmts[i:]
    j = 0
    while j < len(rest) and type(rest[j]).__name__ in ("Load", "Let", "Assign"):
        j += 1
    post = element_program(rest[:j], None, False, False)
    if post is None or any(isinstance(p, ElemLoad) and p.kind != "uniform" for p in post):
        return None
    tail = rest[j:]
    if len(tail) != 1:
        return None
    last = tail[0]
    lk = type(last).__name__
    if lk == "StridedLoop":
        if not _is_var(last.start, co) or const_of(affine(last.step)) != threads \
                or dim_value(last.axis.extent) != length or last.end is not None:
            return None
        pass2 = element_program(last.body, last.axis.name, False, True)
        if pass2 is None or not any(isinstance(p, ElemWrite) for p in pass2):
            return None
    elif lk == "Cond":
        if not _cond_eq(last.cond, co, 0) or last.else_body:
            return None
        for s in last.body:
            k = type(s).__name__
            if k in ("Load", "Let", "Assign"):
                prog = element_program([s], None, False, False)
                if prog is None or any(isinstance(p, ElemLoad) and p.kind != "uniform"
                                       for p in prog):
                    return None
                final.extend(prog)
            elif k == "Write":
                if len(s.values) != 1 or s.output not in shapes or s.atomic:
                    return None
                aff = flat_affine(s.index, shapes[s.output])
                if aff is None:
                    return None
                if row_var is None:
                    if const_of(aff) != 0:
                        return None
                    final.append(ElemWrite(s.output, s.values[0], "scalar"))
                else:
                    if set(aff) - {ONE} != {row_var} or aff[row_var] != 1 or aff.get(ONE, 0):
                        return None
                    final.append(ElemWrite(s.output, s.values[0], "row"))
            else:
                return None
        if not any(isinstance(p, ElemWrite) for p in final):
            return None
    else:
        return None

    row_bufs, col_bufs = [], []
    for p in pass1 + (pass2 or []):
        if isinstance(p, ElemLoad):
            if p.kind == "elem" and p.buffer not in row_bufs:
                row_bufs.append(p.buffer)
            if p.kind == "col" and p.buffer not in col_bufs:
                col_bufs.append(p.buffer)
    outs = []
    for p in (pass2 or []) + final:
        if isinstance(p, ElemWrite) and p.buffer not in outs:
            outs.append(p.buffer)
    for b in row_bufs:
        if _prod(shapes[b]) < rows * length:
            return None
    return RowReducePlan(rows=rows, length=length, threads=threads, full=row_var is None,
                         states=states, state_ops=state_ops, pass1=pass1, combine=combine,
                         partner=dict(zip(states, partners)), post=post, pass2=pass2,
                         final=final, row_buffers=row_bufs, col_buffers=col_bufs,
                         out_buffers=outs)


# ---------------------------------------------------------------------------
# contractions (matmul)
# ---------------------------------------------------------------------------

@record
class ContractionPlan:
    a: str            # [M, K]
    b: str            # [K, N]
    c: str            # [M, N]
    M: int
    N: int
    K: int
    atomic: bool


def _vars_in(expr):
    k = type(expr).__name__
    if k == "Var":
        return {expr.name}
    if k == "BinaryExpr":
        return _vars_in(expr.left) | _vars_in(expr.right)
    if k == "TernaryExpr":
        return _vars_in(expr.cond) | _vars_in(expr.if_true) | _vars_in(expr.if_false)
    return set()


def lift_contraction(kernel):
    """Recognise ``C (+)= A @ B`` written as an accumulate-of-products schedule.

    Accepted bodies contain only ``Init`` (identity 0), shared arrays, ``cp.async``
    copies from global memory, loops, barriers, loads, ``multiply`` assignments,
    ``add`` accumulators and writes of accumulators to one 2-D output. Every product
    must multiply one value that came from the A operand by one from B.
    """
    from .ir import walk
    body = kernel.body
    if len(body) != 1 or type(body[0]).__name__ != "Tile":
        return None
    tile = body[0]
    allowed = {"Init", "Smem", "CpAsyncCopy", "CpAsyncCommit", "CpAsyncWait", "Loop",
               "StridedLoop", "Sync", "Load", "Assign", "Accum", "Write"}
    stmts = list(walk(tile.body))
    if any(type(s).__name__ not in allowed for s in stmts) or not _all_f32(stmts):
        return None
    if not any(type(s).__name__ == "Accum" for s in stmts):
        return None
    shapes = {a: kernel.shape(a) for a in kernel.arg_order}
    outs = [a["name"] for a in kernel.selected.get("args", ()) if a.get("output")]
    if len(outs) != 1 or len(shapes[outs[0]]) != 2:
        return None
    c = outs[0]
    M, N = shapes[c]
    smem = {s.name for s in stmts if type(s).__name__ == "Smem"}
    smem_src = {}                               # shared array -> global buffer it copies
    for s in stmts:
        if type(s).__name__ == "CpAsyncCopy":
            if s.src not in shapes or s.smem not in smem:
                return None
            if smem_src.setdefault(s.smem, s.src) != s.src:
                return None
    origin = {}                                 # SSA value -> global buffer it was read from
    sources = {}                                # global buffer -> index tuples that read it
    for s in stmts:
        if type(s).__name__ == "CpAsyncCopy":
            sources.setdefault(s.src, []).append(tuple(s.src_index))
    inits = set()
    products = {}
    writes = []
    for s in stmts:
        k = type(s).__name__
        if k == "Init":
            if float(s.identity) != 0.0:
                return None
            inits.add(s.name)
        elif k == "Load":
            if len(s.names) != 1:
                return None
            if s.input in smem:
                if s.input not in smem_src:
                    return None
                origin[s.names[0]] = smem_src[s.input]
            elif s.input in shapes and s.input != c:
                origin[s.names[0]] = s.input
                sources.setdefault(s.input, []).append(tuple(s.index))
            else:
                return None
        elif k == "Assign":
            if op_name(s.op) != "multiply" or len(s.args) != 2:
                return None
            if any(a not in origin for a in s.args):
                return None
            products[s.name] = tuple(origin[a] for a in s.args)
        elif k == "Accum":
            if op_name(s.op) != "add" or s.base is not None or s.value not in products:
                return None
            inits.add(s.name)
        elif k == "Write":
            if s.output != c or any(v not in inits for v in s.values):
                return None
            writes.append(s)
    if not writes or len(sources) != 2:
        return None
    atomic = {bool(w.atomic) for w in writes}
    if len(atomic) != 1:
        return None
    x, y = sorted(sources)
    if len(shapes[x]) != 2 or len(shapes[y]) != 2:
        return None
    row_vars = _vars_in(writes[0].index[0])
    col_vars = _vars_in(writes[0].index[1]) if len(writes[0].index) > 1 else set()

    def dim_vars(buf, d):
        out = set()
        for idx in sources[buf]:
            if len(idx) == 2:
                out |= _vars_in(idx[d])
        return out

    cands = []
    for a, b in ((x, y), (y, x)):
        (am, ak), (bk, bn) = shapes[a], shapes[b]
        if am == M and bn == N and ak == bk:
            score = len(dim_vars(a, 0) & row_vars) + len(dim_vars(b, 1) & col_vars)
            cands.append((score, a, b, ak))
    if not cands:
        return None
    cands.sort(reverse=True)
    if len(cands) == 2 and cands[0][0] == cands[1][0]:
        return None                              # cannot tell A from B
    _, a, b, K = cands[0]
    for pa, pb in products.values():
        if {pa, pb} != {a, b}:
            return None
    return ContractionPlan(a=a, b=b, c=c, M=M, N=N, K=K, atomic=atomic.pop())


# ---------------------------------------------------------------------------
# attention: softmax(scale * q @ kt) @ v with an online-softmax key loop
# ---------------------------------------------------------------------------

@record
class AttentionPlan:
    q: str            # [..., Sq, D]
    kt: str           # [..., D, Skv]  (keys pre-transposed, reference tools/expressions_open.py:92)
    v: str            # [..., Skv, Dv]
    out: str          # [..., Sq, Dv]
    scale_buf: str    # 1-element buffer c; the scores are scaled by 1 / c
    G: int            # product of the leading (batch, head) dimensions
    Sq: int
    Skv: int
    D: int
    Dv: int


_COMMUTATIVE = frozenset({"add", "multiply", "maximum", "minimum"})


def _online_softmax_dataflow(body, q, kt, v, scale_buf, smem_src, out) -> bool:
    """True when the statements compute exactly ``softmax(q @ kt * (1/c)) @ v`` with the online
    softmax the attention templates implement; the checks above only look at which ops and
    buffers occur, and a body that arranges the same ops differently (the scale applied
    after the softmax, another normalisation) must go to a lowering that follows it
    statement by statement.

    Every value is evaluated symbolically: a load is its global buffer (through the shared
    array a ``cp.async`` fills), an accumulator read is that accumulator's running value, and
    add / multiply / maximum arguments are put in a canonical order. Then:

    * each dot accumulator ``D`` adds ``q * kt`` in a seeded loop of its own;
    * each max accumulator ``M`` takes ``s = D * reciprocal(c)``; with ``g = max(M, s)``,
      ``alpha = exp(M - g)`` and ``beta = exp(s - g)``, the sum accumulator ``L`` adds ``beta``
      to ``L * alpha`` and each output accumulator ``O`` adds ``v * beta`` to ``O * alpha``,
      all in the key loop that encloses ``D``'s loop;
    * every write, after the key loop, stores ``O * reciprocal(L)`` into the output, and every
      accumulator is one of these.

    The shapes of the reference's attention IR (``problems/a01_attention``,
    ``problems/a02_attention_128``) and of the tiled form all have this dataflow."""
    env, updates, writes = {}, {}, []
    table = {}                              # expression -> id (equal expressions, equal ids)

    def node(*key):
        return table.setdefault(key, len(table))

    one = node("lit", 1.0)

    def canon(op, *args):
        if op == "multiply" and len(args) == 2 and one in args:
            return args[0] if args[1] == one else args[1]
        if op in _COMMUTATIVE:
            args = sorted(args)
        return node(op, *args)

    def ev(name):
        return env[name] if name in env else node("acc", name)

    def visit(stmts, path):
        for st in stmts:
            kind = type(st).__name__
            if kind in ("Loop", "StridedLoop"):
                visit(st.body, path + ((id(st), bool(st.seed)),))
            elif kind == "Load":
                src = smem_src.get(st.input, st.input)
                for nm in st.names:
                    env[nm] = node("ld", src)
            elif kind == "Let":
                val = st.value.value if type(st.value).__name__ == "Literal" else st.value
                if not isinstance(val, (int, float)):
                    return False
                env[st.name] = node("lit", float(val))
            elif kind == "Assign":
                env[st.name] = canon(op_name(st.op), *(ev(a) for a in st.args))
            elif kind == "Accum":
                if st.name in updates:
                    return False
                base = ev(st.base) if st.base is not None else node("acc", st.name)
                updates[st.name] = (op_name(st.op), base, ev(st.value), path)
                env[st.name] = node("acc", st.name)
            elif kind == "Write":
                if st.output != out:
                    return False
                writes.extend((ev(x), path) for x in st.values)
            elif kind == "Init":
                return False            # the fixture forms seed their loops instead
        return True

    if not visit(body, ()):
        return False
    dot = canon("multiply", node("ld", q), node("ld", kt))
    recip = canon("reciprocal", node("ld", scale_buf))
    D = {n for n, (op, base, val, _) in updates.items()
         if op == "add" and base == node("acc", n) and val == dot}
    seen, key_loop, outs = set(D), None, {}
    for m, (op, base, val, path) in updates.items():
        if op != "maximum":
            continue
        d = next((d for d in D if val == canon("multiply", node("acc", d), recip)), None)
        if d is None or base != node("acc", m):
            return False
        dpath = updates[d][3]
        if not dpath or not dpath[-1][1] or dpath[:-1] != path:
            return False                # D's own seeded loop, directly inside the key loop
        if key_loop not in (None, path):
            return False
        key_loop = path
        s_ = val
        g = canon("maximum", node("acc", m), s_)
        alpha = canon("exp", canon("subtract", node("acc", m), g))
        beta = canon("exp", canon("subtract", s_, g))
        sums = [n for n, (op2, b2, v2, p2) in updates.items()
                if op2 == "add" and p2 == path and v2 == beta
                and b2 == canon("multiply", node("acc", n), alpha)]
        if len(sums) != 1:
            return False
        acc_o = [n for n, (op2, b2, v2, p2) in updates.items()
                 if op2 == "add" and p2 == path and v2 == canon("multiply", node("ld", v), beta)
                 and b2 == canon("multiply", node("acc", n), alpha)]
        for o in acc_o:
            outs[canon("multiply", node("acc", o), canon("reciprocal", node("acc", sums[0])))] = o
        seen |= {m, sums[0], *acc_o}
    if key_loop is None or seen != set(updates) or not outs:
        return False
    written = set()
    for val, path in writes:
        if val not in outs or len(path) >= len(key_loop) or key_loop[:len(path)] != path:
            return False
        written.add(outs[val])
    return written == set(outs.values())


def lift_attention(kernel):
    """Recognise the attention family (reference ``problems/a01_attention``): the body scales
    q.kt dot products by ``reciprocal(c)``, keeps an online (max, sum) softmax with ``exp`` and
    ``maximum``, accumulates v rows weighted by it and writes the normalised rows."""
    from .ir import walk
    body = kernel.body
    if len(body) != 1 or type(body[0]).__name__ != "Tile":
        return None
    stmts = list(walk(body[0].body))
    allowed = {"Load", "Assign", "Let", "Init", "Accum", "Loop", "StridedLoop", "Smem",
               "CpAsyncCopy", "CpAsyncCommit", "CpAsyncWait", "Sync", "Write"}
    if any(type(s).__name__ not in allowed for s in stmts) or not _all_f32(stmts):
        return None
    shapes = {a: kernel.shape(a) for a in kernel.arg_order}
    outs = [a["name"] for a in kernel.selected.get("args", ()) if a.get("output")]
    if len(outs) != 1 or len(shapes[outs[0]]) < 2:
        return None
    out = outs[0]
    ops = {op_name(s.op) for s in stmts if type(s).__name__ == "Assign"}
    acc_ops = {op_name(s.op) for s in stmts if type(s).__name__ == "Accum"}
    if not ops <= {"multiply", "reciprocal", "maximum", "subtract", "exp", "add"} \
            or not {"exp", "maximum", "reciprocal"} <= ops or not acc_ops <= {"add", "maximum"} \
            or "maximum" not in acc_ops:
        return None
    smem = {s.name for s in stmts if type(s).__name__ == "Smem"}
    smem_src = {}
    for s in stmts:
        if type(s).__name__ == "CpAsyncCopy":
            if smem_src.setdefault(s.smem, s.src) != s.src:
                return None
    origin = {}
    scalar_loads = {}
    for s in stmts:
        if type(s).__name__ != "Load":
            continue
        src = smem_src.get(s.input) if s.input in smem else s.input
        if src is None or src not in shapes:
            return None
        for nm in s.names:
            origin[nm] = src
            if len(shapes[src]) == 1 and shapes[src][0] == 1:
                scalar_loads[nm] = src
    scale_buf = None
    for s in stmts:
        if type(s).__name__ == "Assign" and op_name(s.op) == "reciprocal" \
                and len(s.args) == 1 and s.args[0] in scalar_loads:
            scale_buf = scalar_loads[s.args[0]]
    if scale_buf is None:
        return None
    # the dot product: products of two loaded values from two different buffers
    pairs = set()
    for s in stmts:
        if type(s).__name__ == "Assign" and op_name(s.op) == "multiply" and len(s.args) == 2 \
                and all(a in origin and a not in scalar_loads for a in s.args):
            pairs.add(frozenset(origin[a] for a in s.args))
    tensors = [b for b in set(origin.values()) if b != scale_buf]
    if len(tensors) != 3 or len(pairs) != 1:
        return None
    qk = next(iter(pairs))
    if len(qk) != 2:
        return None
    (vbuf,) = [b for b in tensors if b not in qk]
    so, sv = shapes[out], shapes[vbuf]
    lead = so[:-2]
    cands = []
    for q, kt in (tuple(qk), tuple(qk)[::-1]):
        sq, sk = shapes[q], shapes[kt]
        if len(sq) == len(sk) == len(sv) == len(so) and sq[:-2] == sk[:-2] == sv[:-2] == lead \
                and sq[-2] == so[-2] and sq[-1] == sk[-2] and sk[-1] == sv[-2] \
                and sv[-1] == so[-1]:
            cands.append((q, kt))
    if len(cands) != 1:
        # square shapes: q is the buffer whose rows follow the output rows
        rows = set()
        for s in stmts:
            if type(s).__name__ == "Write" and s.output == out and len(s.index) >= 2:
                rows |= _vars_in(s.index[-2])
        picks = []
        for q, kt in cands:
            qrow = set()
            for s in stmts:
                if type(s).__name__ == "Load" and s.input == q and len(s.index) >= 2:
                    qrow |= _vars_in(s.index[-2])
            if qrow and qrow <= rows:
                picks.append((q, kt))
        if len(picks) != 1:
            return None
        cands = picks
    q, kt = cands[0]
    if not _online_softmax_dataflow(body[0].body, q, kt, vbuf, scale_buf, smem_src, out):
        return None
    G = 1
    for d in lead:
        G *= d
    return AttentionPlan(q=q, kt=kt, v=vbuf, out=out, scale_buf=scale_buf, G=G,
                         Sq=shapes[q][-2], Skv=shapes[kt][-1], D=shapes[q][-1], Dv=sv[-1])
