"""``EmmyIRLowering``: pick the sm_100a template for a kernel and emit its entry.

Dispatch order (the reference matches fixed statement-kind tuples, reference
``compile.py:5581-5654``; here each template *lifts* the body and declines
when it does not fit):

1. contraction (matmul) and attention templates on tcgen05 + TMEM,
2. attention on the CUDA cores, one warp per query row, for the attention bodies the tcgen05
   template declines (short sequences, other head widths, the fixtures' launch geometry),
3. cooperative reductions and fused row operations,
4. vectorised pointwise,
5. the general statement walker, which lowers every statement kind one by
   one and is the fallback for any body the templates decline.

Unsupported IR raises ``NotImplementedError`` (fail closed, as the
reference does): no PTX is ever emitted for a body that was not understood.
"""

from __future__ import annotations

import importlib

from ..analysis import lift_attention, lift_contraction, lift_pointwise, lift_rowreduce
from ..ptx import PTXKernelGenerator


# below this many multiply-adds the tcgen05 template's fixed costs (tensor-memory
# allocation, barrier set-up, one CTA per output tile) exceed the work: small split-K IRs
# such as m02 (128 x 64 x 256, 512 CTAs adding into one tile) run faster as scheduled
MIN_CONTRACTION_MACS = 1 << 22


def _fits_contraction(kernel, forced=False):
    plan = lift_contraction(kernel)
    if plan is None or (not forced and plan.M * plan.N * plan.K < MIN_CONTRACTION_MACS):
        return None
    from .matmul import plan_tiles      # the template module only once the body lifted
    block = list(kernel.launch.get("block", [1, 1, 1]))
    if block[1:] != [1, 1] or list(kernel.launch.get("grid", [1, 1, 1]))[1:] != [1, 1]:
        return None
    if plan_tiles(plan.M, plan.N, plan.K, int(kernel.launch.get("smem_bytes", 0) or 0),
                  block[0]) is None:
        return None
    return plan


def _fits_attention(kernel):
    plan = lift_attention(kernel)
    if plan is None:
        return None
    from .attention import fits
    return plan if fits(plan, kernel.launch) else None


def _fits_attention_warp(kernel):
    plan = lift_attention(kernel)
    if plan is None:
        return None
    from .attention_warp import fits
    return plan if fits(plan, kernel.launch) else None


_EMITTERS = {"matmul": "lower_contraction", "attention": "lower_attention",
             "attention_warp": "lower_attention_warp",
             "reduce": "lower_rowreduce", "pointwise": "lower_pointwise"}


def _check_launch(launch) -> None:
    """The meta.json launch record must describe a launch CUDA can make: grid and block of
    three positive integers, at most 1024 threads per CTA (z at most 64), grid y and z at most
    65535, and a non-negative integer ``smem_bytes``. The templates size their work from these
    numbers, so a record outside them is refused instead of compiled into a kernel that could
    not be launched as described."""
    def count(x):                       # an integer of any integral type, not a bool
        return hasattr(x, "__index__") and not isinstance(x, bool)

    for field in ("grid", "block"):
        v = launch.get(field, [1, 1, 1])
        if not (isinstance(v, (list, tuple)) and len(v) == 3
                and all(count(x) and x >= 1 for x in v)):
            raise ValueError(f"launch {field} must be three positive integers, got {v!r}")
    block, grid = launch.get("block", [1, 1, 1]), launch.get("grid", [1, 1, 1])
    if block[0] * block[1] * block[2] > 1024 or block[2] > 64:
        raise ValueError(f"launch block {list(block)} exceeds 1024 threads per CTA")
    if grid[0] > 2**31 - 1 or grid[1] > 65535 or grid[2] > 65535:
        raise ValueError(f"launch grid {list(grid)} exceeds the grid limits")
    smem = launch.get("smem_bytes", 0) or 0
    if not count(smem) or smem < 0:
        raise ValueError(f"launch smem_bytes must be a non-negative integer, got {smem!r}")


class EmmyIRLowering:
    """Lower one parsed kernel to the text of its ``.entry`` (module declarations first)."""

    def __init__(self, kernel, *, template: str | None = None):
        self.kernel = kernel
        self.gen = PTXKernelGenerator(kernel)
        self.force = template
        self.template = None
        self.values: dict = {}      # IR value name -> register, for :meth:`_assign`

    def _assign(self, stmt) -> str:
        """Lower one ``Assign`` statement on its own into :attr:`gen`, the way the
        reference's op-table tests drive it (reference ``compile.py:2462-2594``): the
        operands are registers already named in :attr:`values`, the result register is
        stored under ``stmt.name`` and returned. An unknown operation raises
        ``NotImplementedError`` ("Unsupported unary/binary elementwise operation")."""
        from ..codegen import emit_op
        from ..ir import dtype_name, op_name
        op = stmt.op if isinstance(stmt.op, str) else getattr(stmt.op, "name", None)
        if not isinstance(op, str):
            op = op_name(stmt.op)
        dt = getattr(stmt, "dtype", None)
        dt = getattr(dt, "name", None) if dt is not None and not isinstance(dt, str) else dt
        if dt not in (None, "f32"):
            raise NotImplementedError(f"Unsupported elementwise dtype {dtype_name(dt)}")
        try:
            args = [self.values[a] for a in stmt.args]
        except KeyError as exc:
            raise ValueError(f"undefined elementwise input {exc.args[0]!r}") from None
        self.values[stmt.name] = emit_op(self.gen, op, args)
        return self.values[stmt.name]

    def _candidates(self):
        """(name, lift, emitter module) in dispatch order; a template module is imported
        only when its lift accepts the kernel, which keeps small compiles small."""
        k = self.kernel
        forced = self.force == "contraction"
        yield "contraction", (lambda: _fits_contraction(k, forced)), "matmul"
        yield "attention", (lambda: _fits_attention(k)), "attention"
        yield "attention_warp", (lambda: _fits_attention_warp(k)), "attention_warp"
        yield "rowreduce", (lambda: lift_rowreduce(k)), "reduce"
        yield "pointwise", (lambda: lift_pointwise(k)), "pointwise"

    def lower(self) -> str:
        _check_launch(self.kernel.launch)
        for name, lift, emit in self._candidates():
            if self.force and self.force not in (name, "auto"):
                continue
            plan = lift()
            if plan is None:
                continue
            module = importlib.import_module(f"{__name__}.{emit}")
            getattr(module, _EMITTERS[emit])(self.gen, self.kernel, plan)
            self.template = name
            return self.gen.render_module_decls() + self.gen.render_entry()
        from .walker import lower_general
        if self.force not in (None, "auto", "walker"):
            raise NotImplementedError(f"template {self.force!r} does not apply to this kernel")
        lower_general(self.gen, self.kernel)
        self.template = "walker"
        return self.gen.render_module_decls() + self.gen.render_entry()
