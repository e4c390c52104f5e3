"""Seeded synthesis of Kernel IR beyond the benchmark configurations.

The reference's evaluation set holds more shapes and op mixes per category than its fifteen
fixtures (reference ``TASK.md:45-46``; its generator is ``tools/generate.py:74-206``, driven by
Emmy, which is absent here). These generators write the same statement forms as the fixtures
at random sizes and with random op mixes, deterministically from a seed, so the lowerers can
be checked far outside the shapes they were developed on:

* :func:`pointwise` -- a random op DAG over 1-3 inputs and 0-2 scalar constants, 1, 2 or 4
  elements per cell, any cell count (ragged against the 16-byte vectors and the grid);
* :func:`rows` -- RMSNorm, row softmax, L2-norm or row sum at random rows x cols and block;
* :func:`reduction` -- full sum or mean at a random length, grid and block;
* :func:`contraction` -- matmul at random sizes and schedules, inside and outside the tcgen05
  template's conditions (the walker takes the rest); :func:`contraction_tc` -- matmul shapes
  inside them (CTA pairs, single CTAs, half-width units);
* :func:`attention` -- attention in the rank-2 fixture form or the tiled form (head widths
  32, 64, 96 and 128) at random sizes and score divisors.

Each returns ``(payload, meta, info)``; ``info`` says whether every op rounds exactly
(``exact``: the result must match numpy float32 bit for bit) and describes the case.
"""

from __future__ import annotations

import random

from . import workloads
from .ir import Assign, Axis, BinaryExpr, Dim, ElementwiseImpl, Literal, Load, Tile, Var, Write
from .workloads import F32T, _package

# ops whose f32 result is correctly rounded in both PTX (.rn) and numpy float32
EXACT_UNARY = ["relu", "neg", "abs", "square", "copy", "sqrt", "reciprocal"]
EXACT_BINARY = ["add", "subtract", "multiply", "divide", "maximum", "minimum"]
# ops lowered to the approximate special-function unit (ex2 / lg2 / rsqrt / tanh)
APPROX_UNARY = ["exp", "log", "rsqrt", "sigmoid", "tanh", "silu"]


def _lit(v):
    return Literal(value=v, dtype="int" if isinstance(v, int) else "float")


def _bin(op, a, b):
    return BinaryExpr(op=op, left=a, right=b)


def pointwise(seed: int, *, exact_only: bool = False, max_cells: int = 6000):
    """A random elementwise kernel: ``out[i] = f(x0[i], .., c0, ..)``."""
    rng = random.Random(seed)
    n_in = rng.randint(1, 3)
    n_c = rng.randint(0, 2)
    U = rng.choice([1, 2, 4])
    cells = rng.randint(1, max_cells)
    block = rng.choice([32, 64, 128, 256, 512])
    n_ops = rng.randint(1, 6)
    inputs = [f"x{i}" for i in range(n_in)]
    consts = [(f"c{i}", round(rng.uniform(-2.0, 2.0), 3)) for i in range(n_c)]
    unary = EXACT_UNARY + ([] if exact_only else APPROX_UNARY)
    ops = []                       # (name, op, args) over symbolic names per element
    avail = list(inputs) + [c for c, _ in consts]
    for j in range(n_ops):
        if rng.random() < 0.45:
            op = rng.choice(unary)
            args = (rng.choice(avail),)
        else:
            op = rng.choice(EXACT_BINARY)
            args = (rng.choice(avail), rng.choice(avail))
        ops.append((f"v{j}", op, args))
        avail.append(f"v{j}")
    # the output is the last op; make sure it depends on an input
    if not any(a in inputs for _, _, args in ops for a in args):
        ops.append((f"v{n_ops}", "add", (ops[-1][0], inputs[0])))
    a0 = Var(name="a0")
    stmts, names = [], []
    for u in range(U):
        idx = (_bin("+", _bin("*", a0, _lit(U)), _lit(u)),)
        sfx = f"__u{u}"
        for x in inputs:
            stmts.append(Load(names=(x + sfx,), input=x, index=idx, dtype=F32T))
        for c, _ in consts:
            stmts.append(Load(names=(c + sfx,), input=c, index=(_lit(0),), dtype=F32T))
        for name, op, args in ops:
            stmts.append(Assign(name=name + sfx, op=ElementwiseImpl(op),
                                args=tuple(a + sfx for a in args), dtype=F32T))
        names.append(ops[-1][0] + sfx)
    stmts.append(Write(output="out", index=(_bin("+", _bin("*", a0, _lit(U)), _lit(0)),),
                       values=tuple(names), value_dtype=F32T, atomic=False, swizzle="NONE"))
    tile = Tile(axes=(Axis(name="a0", extent=Dim(cells), window=None),), body=tuple(stmts),
                block_threads=None, aux_threads=0, raster_axes=None, raster_group=None,
                raster_orient="m")
    n = cells * U
    args = [{"name": c, "dtype": "f32", "shape": [1], "data": [v]} for c, v in consts]
    args += [{"name": x, "dtype": "f32", "shape": [n], "seed": i} for i, x in enumerate(inputs)]
    args.append({"name": "out", "dtype": "f32", "shape": [n], "output": True})
    expr = "; ".join(f"{nm} = {op}({', '.join(a)})" for nm, op, a in ops)
    payload, meta = _package(f"k_synth_pw_{seed}", "out", tile, [(x, (n,)) for x in inputs],
                             consts, "out", (n,), args, [-(-cells // block), 1, 1],
                             [block, 1, 1], expr, 0, 0)
    exact = all(op in EXACT_UNARY + EXACT_BINARY for _, op, _ in ops)
    return payload, meta, {"exact": exact, "n": n, "U": U, "block": block, "ops": ops}


def rows(seed: int, *, max_rows: int = 96, max_cols: int = 3000):
    """A random row operation (RMSNorm, softmax, L2-norm or row sum)."""
    rng = random.Random(seed)
    kind = rng.choice(["rmsnorm", "softmax", "l2norm", "rowsum"])
    r = rng.randint(1, max_rows)
    c = rng.randint(1, max_cols)
    block = rng.choice([32, 64, 128, 256, 512, 1024])
    payload, meta = workloads.row_op(kind, rows=r, cols=c, block=block)
    return payload, meta, {"kind": kind, "rows": r, "cols": c, "block": block}


def reduction(seed: int, *, max_n: int = 1 << 22):
    """A random full sum or mean."""
    rng = random.Random(seed)
    op = rng.choice(["sum", "mean"])
    n = rng.choice([rng.randint(1, 4096), rng.randint(1, max_n)])
    grid = rng.choice([1, 7, 64, 148, 592, 1184])
    block = rng.choice([32, 64, 128, 256, 512, 1024])
    payload, meta = workloads.full_reduce(n, op, block=block, grid=grid)
    return payload, meta, {"op": op, "n": n, "grid": grid, "block": block}


def contraction(seed: int):
    """A random matmul: sizes and schedule drawn so that some cases meet the tcgen05
    template's conditions (M % 128, K % 32, enough dynamic shared memory) and some do not."""
    rng = random.Random(seed)
    TM, TN, RM, RN = rng.choice([(128, 256, 8, 16), (128, 128, 8, 16), (64, 64, 4, 4),
                                 (32, 64, 4, 8)])
    M = TM * rng.randint(1, 3)
    N = TN * rng.randint(1, 2)
    K = rng.choice([32, 64, 96, 128, 256])
    S = rng.choice([1, 2, 3, 4])
    payload, meta = workloads.matmul(M, N, K, TM=TM, TN=TN, RM=RM, RN=RN, S=S)
    return payload, meta, {"M": M, "N": N, "K": K, "tile": (TM, TN, RM, RN), "S": S}


def contraction_tc(seed: int):
    """A random matmul inside the tcgen05 template's conditions (M % 128, K % 32, 256
    threads, dynamic shared memory), small enough for a quick fp64 check: grids come out even
    and odd, so both the CTA-pair and the single-CTA forms occur, with several tiles per CTA
    or cluster and, for some, half-width units; some in the split-K form with atomic writes
    (compile with ``template="contraction"``: shapes this small would otherwise go to the
    walker)."""
    rng = random.Random(seed)
    TN, RN = rng.choice([(256, 16), (128, 8)])
    M = 128 * rng.randint(1, 8)
    N = 256 * rng.randint(1, 4)
    K = 32 * rng.randint(1, 8)
    S = rng.choice([2, 3, 4])
    if rng.random() < 1 / 3:
        # 128-wide IR tiles with four stages offer the shared memory of 256-wide pair tiles:
        # then the template's tiles are half as many as the clusters, all run as half units
        TN, RN, S, M = 128, 8, 4, 256 * rng.randint(1, 4)
    # some in the split-K form (atomic writes into a zeroed output, as the m02 fixture)
    splits = rng.choice([1, 1, 2, 3, 4])
    if (K // 32) % splits:
        splits = 1
    payload, meta = workloads.matmul(M, N, K, TM=128, TN=TN, RM=8, RN=RN, S=S, splits=splits)
    return payload, meta, {"M": M, "N": N, "K": K, "TN": TN, "S": S, "splits": splits}


def contraction_ragged(seed: int):
    """A random matmul whose shape is not a multiple of the tcgen05 template's tile: M not a
    multiple of 128, N or K not of the template's tile width or K step (N and K multiples of
    4), from IR schedules whose own tiles do divide the shape (64 x 64, 64 x 16 and
    128 x 256 tiles with K steps of 32, 64 and 16). Compile with ``template="contraction"``."""
    rng = random.Random(1000 + seed)
    TM, TN, RM, RN, BKs = rng.choice([(64, 64, 4, 4, 32), (64, 16, 4, 1, 64),
                                      (128, 256, 8, 16, 16)])
    M = TM * rng.randint(1, 6)
    N = TN * rng.randint(1, 6)
    K = BKs * rng.randint(1, 6)
    S = rng.choice([2, 3, 4])
    payload, meta = workloads.matmul(M, N, K, TM=TM, TN=TN, RM=RM, RN=RN, BKs=BKs, S=S)
    return payload, meta, {"M": M, "N": N, "K": K, "tile": (TM, TN, RM, RN, BKs), "S": S}


def attention(seed: int):
    """A random attention problem, in the a02 fixture's rank-2 form (one query row per CTA,
    walker) or in the tiled form (query blocks of 128 rows; the tcgen05 template when the
    shapes and shared memory allow, the walker otherwise), with a random score divisor."""
    rng = random.Random(seed)
    scale = rng.choice([None, 0.5, 2.0, 11.3])
    if rng.random() < 0.5:
        S = rng.choice([16, 48, 64, 100, 128, 256])
        D = rng.choice([16, 32, 64])
        payload, meta = workloads.attention_rows(S, D, scale=scale)
        return payload, meta, {"form": "rows", "S": S, "D": D, "scale": scale}
    D = rng.choice([32, 64, 96, 128])
    B, H = rng.randint(1, 2), rng.randint(1, 3)
    S = 128 * rng.randint(1, 3)
    stages = rng.choice([2, 3])
    if D == 96:        # three stages of the IR's tiles would ask for more than 227 KiB
        stages = 2
    payload, meta = workloads.attention(B, H, S, D, stages=stages, scale=scale)
    return payload, meta, {"form": "tiled", "B": B, "H": H, "S": S, "D": D, "stages": stages,
                           "scale": scale}
