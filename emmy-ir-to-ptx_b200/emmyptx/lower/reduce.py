"""Reduction and fused-row templates for sm_100a.

One template serves the whole cooperative-reduction family the IR expresses
with ``StridedLoop -> WarpShuffle -> Smem -> TreeHalve`` (sum, mean, row sum,
RMSNorm, softmax, L2-norm; reference ``compile.py:2703-4856``). The IR's own
per-element program (including the online-softmax ``(max, sum)`` pair and its
combine rule) is evaluated literally; only the schedule is redesigned:

Full reduction (one scalar result)
    Every thread of the launch takes 16-byte chunks in a grid-stride loop,
    four chunks in flight per iteration. Partial states are folded by a
    ``shfl.sync.bfly`` ladder, then across warps through shared memory. Each
    CTA stores its partial to a module-scope ``.global`` array and takes a
    ticket with ``atom.acq_rel.gpu.inc`` (which wraps back to zero by itself);
    the CTA that draws the last ticket folds all partials in CTA order and
    writes the result. One launch, no workspace argument, and the result is
    deterministic for a given grid. The reference lowerer only accepts a
    single 128-thread CTA here (reference ``compile.py:2837-2854``).

Row operations (one CTA per row, grid-stride over rows)
    When the row is read twice (statistics, then the output pass) it is
    staged once into shared memory with ``cp.async.bulk`` completing on an
    ``mbarrier``; both passes then read shared memory, so HBM sees one read
    and one write per element. The reference reads the row from global
    memory two or three times (reference ``compile.py:3277-4856``).

Sums (a plain ``add`` accumulator and no fused output pass: the full sum and
mean, row sums) are accumulated in f64, so that every result is within 1e-5
relative of the exact sum even when its terms cancel: each f32 element is
widened (exactly) and added in f64, a thread of the full reduction keeps one
f64 accumulator per chunk in flight (short dependent chains), and the warp
ladder, the cross-warp tree and the cross-CTA fold add in f64; the result is
rounded to f32 once, before the IR's own scalar program (the mean's
division) runs. A full reduction whose launch gives each thread at most
``F32_LANE_LIMIT`` elements first adds them in f32 into 16 lane registers per
thread (at most 64 terms each) and widens those once (see ``_lower_full``). An f32 accumulation of n terms is off by about
2^-24 * sum|x| (times a factor that grows with n) whatever its order, and so
is Kahan's compensated loop (its bound is 2^-23 * sum|x|): both exceed
1e-5 * |sum x| when the sum is small next to sum|x|. Measured on B200 for the
2^26 sum (592 x 256 threads): plain f32 45.5 us per launch, f64 with four
accumulators 45.6 us (35.4 -> 35.9 us overlapped), the error-free TwoSum in
f32 59.8 us, eight chunks in flight 64-68 us in every form.

Every mbarrier wait is bounded: after the iteration limit the kernel sets
bit 0 of the module-scope word ``emmy_error`` and returns instead of
spinning forever.
"""

from __future__ import annotations

from ..analysis import ElemAccum, ElemLoad, ElemWrite
from ..codegen import emit_op, identity_literal, run_program
from .common import WAIT_LIMIT, aligned_predicate, load_pointers

SMEM_STAGE_LIMIT = 40 * 1024  # static shared memory we allow for staged rows
UNROLLED_CHUNKS = 8           # per-thread 16-byte chunks of a row handled without a loop
FULL_IN_FLIGHT = 4            # 16-byte loads a thread has in flight in a full reduction
F32_LANE_LIMIT = 1024         # exact sums: f32 lane registers up to this many elements/thread
EARLY_TRIGGER = (7, 8)        # overlapped launches: let the next kernel start past this share
FOLD_UNROLL = 8               # cross-CTA fold: partials per thread loaded in one batch


def _pow2_ceil(n):
    p = 1
    while p < n:
        p *= 2
    return p


def combine_identity_safe(plan) -> bool:
    """True when folding an identity state into a partial cannot change it (sum/max/min/prod)."""
    names = set(plan.states)
    for op in plan.combine:
        if op.name not in names or len(op.args) != 2:
            return False
        s = op.name
        if set(op.args) != {s, plan.partner[s]} or op.op != plan.state_ops[s]:
            return False
    return True


def exact_sum(plan) -> bool:
    """True for a pure sum: every state a plain ``add`` accumulator updated in place, the
    combine program the plain add, and no fused output pass (the full sum and mean, row
    sums). These get the compensated per-thread loop and the f64 fold."""
    if plan.pass2 is not None or not combine_identity_safe(plan):
        return False
    if any(plan.state_ops[s] != "add" for s in plan.states):
        return False
    for p in plan.pass1:
        if isinstance(p, ElemAccum) and (p.op != "add" or p.base not in (None, p.name)):
            return False
    return True


class _Reducer:
    """Emits the warp ladder, the cross-warp tree and partial-state bookkeeping."""

    def __init__(self, gen, plan, block, track_valid, f64=False):
        self.gen = gen
        self.plan = plan
        self.block = block
        self.nwarps = block // 32
        self.track = track_valid
        S = len(plan.states)
        if f64:
            gen.shared("emmy_red64", ".f64", length=S * 32, align=16)
            gen.shared("emmy_bcast64", ".f64", length=max(S, 1) + 1, align=16)
        else:
            gen.shared("emmy_red", ".f32", length=S * 32, align=16)
            gen.shared("emmy_bcast", ".f32", length=max(S, 1) + 1, align=16)
        if track_valid:
            gen.shared("emmy_redv", ".u32", length=32, align=16)

    # -- f64 sums (exact_sum plans) ------------------------------------------------
    def f64_sets(self, nsets):
        """``nsets`` sets of f64 accumulators (one per state), all zero."""
        sets = []
        for _ in range(nsets):
            regs = []
            for _ in self.plan.states:
                d = self.gen.register(".f64")
                self.gen.emit(f"mov.f64 {d}, 0d0000000000000000;")
                regs.append(d)
            sets.append(regs)
        return sets

    def f64_hook(self, sets, sel):
        """``run_program`` accumulate hook: widen the f32 value and add it in f64 to the
        state's accumulator in set ``sel[0]`` (the caller picks the set per chunk)."""
        gen = self.gen
        index = {name: i for i, name in enumerate(self.plan.states)}

        def accum(p, base, value, acc):
            d = sets[sel[0]][index[p.name]]
            w = gen.register(".f64")
            gen.emit(f"cvt.f64.f32 {w}, {value};")
            gen.emit(f"add.rn.f64 {d}, {d}, {w};")
        return accum

    def merge_sets(self, sets):
        """The sets added in order (set 0 + set 1 + ...): one f64 register per state."""
        out = list(sets[0])
        for st in sets[1:]:
            new = []
            for a, b in zip(out, st):
                r = self.gen.register(".f64")
                self.gen.emit(f"add.rn.f64 {r}, {a}, {b};")
                new.append(r)
            out = new
        return out

    def narrow(self, dregs):
        gen, out = self.gen, []
        for d in dregs:
            r = gen.register(".f32")
            gen.emit(f"cvt.rn.f32.f64 {r}, {d};")
            out.append(r)
        return out

    def _ladder64(self, regs, offsets):
        gen = self.gen
        for off in offsets:
            new = []
            for d in regs:
                lo, hi, lo2, hi2 = (gen.register(".b32") for _ in range(4))
                gen.emit(f"mov.b64 {{{lo}, {hi}}}, {d};")
                gen.emit(f"shfl.sync.bfly.b32 {lo2}, {lo}, {off}, 31, -1;")
                gen.emit(f"shfl.sync.bfly.b32 {hi2}, {hi}, {off}, 31, -1;")
                o, r = gen.register(".f64"), gen.register(".f64")
                gen.emit(f"mov.b64 {o}, {{{lo2}, {hi2}}};")
                gen.emit(f"add.rn.f64 {r}, {d}, {o};")
                new.append(r)
            regs = new
        return regs

    def block_reduce_f64(self, dregs, lane, warp, *, broadcast=True):
        """The f64 sum of ``dregs`` over the CTA: a butterfly ladder per warp, then warp 0
        over the warps' values in warp order. With ``broadcast`` every thread gets it,
        otherwise warp 0 holds it."""
        gen, S = self.gen, len(dregs)
        regs = self._ladder64(dregs, (16, 8, 4, 2, 1))
        if self.nwarps == 1:
            return regs
        p_lane0 = gen.register(".pred")
        gen.emit(f"setp.eq.u32 {p_lane0}, {lane}, 0;")
        wofs = gen.register(".u32")
        gen.emit(f"shl.b32 {wofs}, {warp}, 3;")
        base = gen.register(".u32")
        gen.emit(f"mov.u32 {base}, emmy_red64;")
        gen.emit(f"add.u32 {base}, {base}, {wofs};")
        for i, d in enumerate(regs):
            gen.emit(f"@{p_lane0} st.shared.f64 [{base}+{i * 256}], {d};")
        gen.emit("bar.sync 0;")
        L_skip = gen.new_label("w0skip64")
        p_w0 = gen.register(".pred")
        gen.emit(f"setp.ne.u32 {p_w0}, {warp}, 0;")
        out = [gen.register(".f64") for _ in range(S)]
        gen.emit(f"@{p_w0} bra {L_skip};")
        p_in = gen.register(".pred")
        gen.emit(f"setp.lt.u32 {p_in}, {lane}, {self.nwarps};")
        lofs = gen.register(".u32")
        gen.emit(f"shl.b32 {lofs}, {lane}, 3;")
        lb = gen.register(".u32")
        gen.emit(f"mov.u32 {lb}, emmy_red64;")
        gen.emit(f"add.u32 {lb}, {lb}, {lofs};")
        wregs = []
        for i in range(S):
            r = gen.register(".f64")
            gen.emit(f"mov.f64 {r}, 0d0000000000000000;")
            gen.emit(f"@{p_in} ld.shared.f64 {r}, [{lb}+{i * 256}];")
            wregs.append(r)
        offsets = []
        o = _pow2_ceil(self.nwarps) // 2
        while o >= 1:
            offsets.append(o)
            o //= 2
        wregs = self._ladder64(wregs, offsets)
        for d, r in zip(out, wregs):
            gen.emit(f"mov.f64 {d}, {r};")
        if broadcast:
            for i, r in enumerate(wregs):
                gen.emit(f"@{p_lane0} st.shared.f64 [emmy_bcast64+{i * 8}], {r};")
        gen.label(L_skip)
        if broadcast:
            gen.emit("bar.sync 0;")
            for i, d in enumerate(out):
                gen.emit(f"ld.shared.f64 {d}, [emmy_bcast64+{i * 8}];")
        return out

    def identity_states(self):
        regs = []
        for s in self.plan.states:
            r = self.gen.register(".f32")
            self.gen.emit(f"mov.f32 {r}, {identity_literal(self.plan.state_ops[s])};")
            regs.append(r)
        return regs

    def combine(self, mine, other, valid=None, ovalid=None):
        """Fold ``other`` into ``mine`` with the IR's combine program; returns new registers."""
        gen, plan = self.gen, self.plan
        env = {}
        for s, a, b in zip(plan.states, mine, other):
            env[s] = a
            env[plan.partner[s]] = b
        for op in plan.combine:
            env[op.name] = emit_op(gen, op.op, [env[a] for a in op.args])
        new = [env[s] for s in plan.states]
        if valid is None:
            return new
        out = []
        for n, a, b in zip(new, mine, other):
            t = gen.register(".f32")
            gen.emit(f"selp.f32 {t}, {n}, {a}, {ovalid};")
            r = gen.register(".f32")
            gen.emit(f"selp.f32 {r}, {t}, {b}, {valid};")
            out.append(r)
        return out

    def ladder(self, regs, valid, offsets):
        gen = self.gen
        for off in offsets:
            other = []
            for r in regs:
                o = gen.register(".f32")
                gen.emit(f"shfl.sync.bfly.b32 {o}, {r}, {off}, 31, -1;")
                other.append(o)
            if self.track:
                vu = gen.register(".u32")
                gen.emit(f"selp.u32 {vu}, 1, 0, {valid};")
                ov = gen.register(".u32")
                gen.emit(f"shfl.sync.bfly.b32 {ov}, {vu}, {off}, 31, -1;")
                pv = gen.register(".pred")
                gen.emit(f"setp.ne.u32 {pv}, {ov}, 0;")
                regs = self.combine(regs, other, valid, pv)
                nv = gen.register(".pred")
                gen.emit(f"or.pred {nv}, {valid}, {pv};")
                valid = nv
            else:
                regs = self.combine(regs, other)
        return regs, valid

    def block_reduce(self, regs, valid, tid, lane, warp, *, broadcast=True):
        """Fold the per-thread states of the CTA. With ``broadcast`` every thread gets
        the result (as ``TreeHalve`` specifies); otherwise only warp 0 lane 0 holds it."""
        gen, S = self.gen, len(self.plan.states)
        regs, valid = self.ladder(regs, valid, (16, 8, 4, 2, 1))
        if self.nwarps == 1:
            return regs, valid
        p_lane0 = gen.register(".pred")
        gen.emit(f"setp.eq.u32 {p_lane0}, {lane}, 0;")
        wofs = gen.register(".u32")
        gen.emit(f"shl.b32 {wofs}, {warp}, 2;")
        base = gen.register(".u32")
        gen.emit(f"mov.u32 {base}, emmy_red;")
        gen.emit(f"add.u32 {base}, {base}, {wofs};")
        for i, r in enumerate(regs):
            gen.emit(f"@{p_lane0} st.shared.f32 [{base}+{i * 128}], {r};")
        if self.track:
            vb = gen.register(".u32")
            gen.emit(f"mov.u32 {vb}, emmy_redv;")
            gen.emit(f"add.u32 {vb}, {vb}, {wofs};")
            vu = gen.register(".u32")
            gen.emit(f"selp.u32 {vu}, 1, 0, {valid};")
            gen.emit(f"@{p_lane0} st.shared.u32 [{vb}], {vu};")
        gen.emit("bar.sync 0;")
        L_skip = gen.new_label("w0skip")
        p_w0 = gen.register(".pred")
        gen.emit(f"setp.ne.u32 {p_w0}, {warp}, 0;")
        out = [gen.register(".f32") for _ in range(S)]
        outv = gen.register(".pred") if self.track else None
        gen.emit(f"@{p_w0} bra {L_skip};")
        p_in = gen.register(".pred")
        gen.emit(f"setp.lt.u32 {p_in}, {lane}, {self.nwarps};")
        lofs = gen.register(".u32")
        gen.emit(f"shl.b32 {lofs}, {lane}, 2;")
        lb = gen.register(".u32")
        gen.emit(f"mov.u32 {lb}, emmy_red;")
        gen.emit(f"add.u32 {lb}, {lb}, {lofs};")
        wregs = []
        for i, s in enumerate(self.plan.states):
            r = gen.register(".f32")
            gen.emit(f"mov.f32 {r}, {identity_literal(self.plan.state_ops[s])};")
            gen.emit(f"@{p_in} ld.shared.f32 {r}, [{lb}+{i * 128}];")
            wregs.append(r)
        wvalid = None
        if self.track:
            vb2 = gen.register(".u32")
            gen.emit(f"mov.u32 {vb2}, emmy_redv;")
            gen.emit(f"add.u32 {vb2}, {vb2}, {lofs};")
            vv = gen.register(".u32")
            gen.emit(f"mov.u32 {vv}, 0;")
            gen.emit(f"@{p_in} ld.shared.u32 {vv}, [{vb2}];")
            wvalid = gen.register(".pred")
            gen.emit(f"setp.ne.u32 {wvalid}, {vv}, 0;")
        offsets = []
        o = _pow2_ceil(self.nwarps) // 2
        while o >= 1:
            offsets.append(o)
            o //= 2
        wregs, wvalid = self.ladder(wregs, wvalid, offsets)
        for d, r in zip(out, wregs):
            gen.emit(f"mov.f32 {d}, {r};")
        if self.track:
            gen.emit(f"mov.pred {outv}, {wvalid};")
        if broadcast:
            for i, r in enumerate(wregs):
                gen.emit(f"@{p_lane0} st.shared.f32 [emmy_bcast+{i * 4}], {r};")
        gen.label(L_skip)
        if broadcast:
            gen.emit("bar.sync 0;")
            for i, d in enumerate(out):
                gen.emit(f"ld.shared.f32 {d}, [emmy_bcast+{i * 4}];")
        return out, outv


def _hoist_uniforms(gen, plan, ptrs):
    uniforms = {}
    for prog in (plan.pass1, plan.pass2 or [], plan.post, plan.final):
        for p in prog:
            if isinstance(p, ElemLoad) and p.kind == "uniform" and p.name not in uniforms:
                r = gen.register(".f32")
                gen.emit(f"ld.global.f32 {r}, [{ptrs[p.buffer]}+{p.offset * 4}];")
                uniforms[p.name] = r
    return uniforms


def _emit_wait(gen, mbar, phase):
    """Bounded ``mbarrier.try_wait.parity``; on timeout record the error and return."""
    it = gen.register(".u32")
    gen.emit(f"mov.u32 {it}, 0;")
    L_wait = gen.new_label("wait")
    L_ok = gen.new_label("waitok")
    p = gen.register(".pred")
    pl = gen.register(".pred")
    gen.label(L_wait)
    gen.emit(f"mbarrier.try_wait.parity.shared::cta.b64 {p}, [{mbar}], {phase};")
    gen.emit(f"@{p} bra {L_ok};")
    gen.emit(f"add.u32 {it}, {it}, 1;")
    gen.emit(f"setp.lt.u32 {pl}, {it}, {WAIT_LIMIT};")
    gen.emit(f"@{pl} bra {L_wait};")
    gen.emit("red.global.or.b32 [emmy_error], 1;")
    gen.emit("ret;")
    gen.label(L_ok)


def lower_rowreduce(gen, kernel, plan) -> None:
    launch = kernel.launch
    block = list(launch.get("block", [plan.threads, 1, 1]))
    grid = list(launch.get("grid", [1, 1, 1]))
    if block[1:] != [1, 1] or grid[1:] != [1, 1]:
        raise NotImplementedError("reduction template needs a 1-D launch")
    B = block[0]
    if B % 32 or not 32 <= B <= 1024:
        raise NotImplementedError("reduction template needs a whole number of warps")
    gen.maxntid = B
    gen.module_decl(".global .align 4 .u32 emmy_error;")
    if plan.full:
        _lower_full(gen, kernel, plan, B, max(grid[0], 1))
    else:
        _lower_rows(gen, kernel, plan, B)


# ---------------------------------------------------------------------------
# full reduction with single-pass cross-CTA finish
# ---------------------------------------------------------------------------

def _lower_full(gen, kernel, plan, B, G):
    L = plan.length
    S = len(plan.states)
    names = [a for a in kernel.arg_order]
    ptrs = load_pointers(gen, names)
    uniforms = _hoist_uniforms(gen, plan, ptrs)
    nthr = G * B
    NC = L // 4
    everyone_works = L >= 4 * nthr
    exact = exact_sum(plan)
    track = not combine_identity_safe(plan) and not everyone_works
    red = _Reducer(gen, plan, B, track, f64=exact)
    if exact:
        gen.module_decl(f".global .align 16 .f64 emmy_partials64[{G * S}];")
    else:
        gen.module_decl(f".global .align 16 .f32 emmy_partials[{G * S}];")
        gen.module_decl(f".global .align 16 .u32 emmy_pvalid[{G}];")
    gen.module_decl(".global .align 4 .u32 emmy_ticket;")
    gen.shared("emmy_last", ".u32", length=1, align=4)

    tid, cta, lane, warp = (gen.register(".u32") for _ in range(4))
    gen.emit(f"mov.u32 {tid}, %tid.x;")
    gen.emit(f"mov.u32 {cta}, %ctaid.x;")
    gen.emit(f"and.b32 {lane}, {tid}, 31;")
    gen.emit(f"shr.u32 {warp}, {tid}, 5;")
    # CTAs beyond the compiled grid take no part (keeps the ticket count exact)
    p_extra = gen.register(".pred")
    gen.emit(f"setp.ge.u32 {p_extra}, {cta}, {G};")
    gen.emit(f"@{p_extra} ret;")
    gtid = gen.register(".u32")
    gen.emit(f"mad.lo.u32 {gtid}, {cta}, {B}, {tid};")
    # set once this thread has executed griddepcontrol.launch_dependents (see below)
    p_trig = gen.register(".pred")
    gen.emit(f"setp.ne.u32 {p_trig}, 0, 0;")

    states = red.identity_states()
    # exact sums: one accumulator set per chunk in flight; ``sel`` picks the set
    sel = [0]
    sets = red.f64_sets(FULL_IN_FLIGHT) if exact else None
    hook = red.f64_hook(sets, sel) if exact else None
    # An exact sum widens every element to f64, unless the compiled launch gives each thread
    # at most F32_LANE_LIMIT elements: then its main loop adds them in f32 to 16 registers
    # (chunk u of a group, lane ln), at most F32_LANE_LIMIT / 16 = 64 terms each, and widens
    # those once after the loop. The error stays below 63 * 2^-24 (3.8e-6) of the sum of
    # the absolute values for any input, and per element the loop does one f32 add: widening
    # every element costs the overlapped stream 1.3-1.6 % at full clock and 10-13 % on a B200
    # whose power limit has lowered the clock.
    lane_acc = None
    if exact and -(-L // nthr) <= F32_LANE_LIMIT:
        index = {name: i for i, name in enumerate(plan.states)}
        lane_acc = [[[gen.register(".f32") for _ in plan.states] for _ in range(4)]
                    for _ in range(FULL_IN_FLIGHT)]
        for per_u in lane_acc:
            for per_ln in per_u:
                for r in per_ln:
                    gen.emit(f"mov.f32 {r}, 0f00000000;")
        lane_sel = [(0, 0)]

        def lane_hook(p, base, value, acc):
            u, ln = lane_sel[0]
            r = lane_acc[u][ln][index[p.name]]
            gen.emit(f"add.rn.f32 {r}, {r}, {value};")

        def flush_lanes():
            for u, per_u in enumerate(lane_acc):
                for per_ln in per_u:
                    for st, r in enumerate(per_ln):
                        w = gen.register(".f64")
                        gen.emit(f"cvt.f64.f32 {w}, {r};")
                        gen.emit(f"add.rn.f64 {sets[u][st]}, {sets[u][st]}, {w};")
    valid = None
    if track:
        valid = gen.register(".pred")
        gen.emit(f"setp.ne.u32 {valid}, 0, 0;")
    accum_regs = dict(zip(plan.states, states))
    elem_bufs = [p.buffer for p in plan.pass1 if isinstance(p, ElemLoad) and p.kind == "elem"]
    elem_bufs = list(dict.fromkeys(elem_bufs))

    def accumulate(lane_values, mark_valid=True, chunk=0, lane=None):
        sel[0] = chunk
        def load(p):
            if p.kind == "uniform":
                return uniforms[p.name]
            return lane_values[p.buffer]
        use = hook
        if lane is not None and lane_acc is not None:
            lane_sel[0] = (chunk, lane)
            use = lane_hook
        run_program(gen, plan.pass1, {}, load=load, accum_regs=accum_regs, accum=use)
        if track and mark_valid:
            gen.emit(f"setp.eq.u32 {valid}, 0, 0;")

    L_scalar = gen.new_label("scalar")
    L_reduce = gen.new_label("reduce")
    start = gen.register(".u32")
    if NC > 0:
        ok = aligned_predicate(gen, ptrs, elem_bufs)
        gen.emit(f"mov.u32 {start}, {gtid};")
        gen.emit(f"@!{ok} bra {L_scalar};")
        c = gen.register(".u32")
        gen.emit(f"mov.u32 {c}, {gtid};")
        UN = FULL_IN_FLIGHT
        # main loop: UN chunks per thread in flight
        if NC >= UN * nthr:
            L_main = gen.new_label("main")
            L_maindone = gen.new_label("maindone")
            pm = gen.register(".pred")
            gen.label(L_main)
            gen.emit(f"setp.gt.u32 {pm}, {c}, {NC - UN * nthr};")  # need c + (UN-1)*nthr < NC
            gen.emit(f"@{pm} bra {L_maindone};")
            # Overlapped launches: once this thread's position passes EARLY_TRIGGER of the
            # chunks, the next kernel on the stream may be scheduled. It starts at the front
            # of its input, which this kernel read more than an L2's worth of bytes ago when
            # the input is larger than L2, so the two kernels never read the same lines; it
            # just fills the SMs that finish streaming first.
            T = NC * EARLY_TRIGGER[0] // EARLY_TRIGGER[1]
            L_notrig = gen.new_label("notrig")
            pe = gen.register(".pred")
            gen.emit(f"@{p_trig} bra {L_notrig};")
            gen.emit(f"setp.lt.u32 {pe}, {c}, {T};")
            gen.emit(f"@{pe} bra {L_notrig};")
            gen.emit("griddepcontrol.launch_dependents;")
            gen.emit(f"setp.eq.u32 {p_trig}, 0, 0;")
            gen.label(L_notrig)
            loaded = []
            for u in range(UN):
                cu = gen.register(".u32")
                gen.emit(f"add.u32 {cu}, {c}, {u * nthr};")
                off = gen.register(".u64")
                gen.emit(f"mul.wide.u32 {off}, {cu}, 16;")
                vals = {}
                for b in elem_bufs:
                    a = gen.register(".u64")
                    gen.emit(f"add.s64 {a}, {ptrs[b]}, {off};")
                    regs = gen.registers(".f32", 4)
                    gen.emit(f"ld.global.nc.L1::no_allocate.v4.f32 {{{', '.join(regs)}}}, [{a}];")
                    vals[b] = regs
                loaded.append(vals)
            for u, vals in enumerate(loaded):
                for ln in range(4):
                    accumulate({b: vals[b][ln] for b in elem_bufs}, mark_valid=False, chunk=u,
                               lane=ln)
            if track:
                gen.emit(f"setp.eq.u32 {valid}, 0, 0;")
            gen.emit(f"add.u32 {c}, {c}, {UN * nthr};")
            gen.emit(f"bra.uni {L_main};")
            gen.label(L_maindone)
            if lane_acc is not None:
                flush_lanes()
        # remaining chunks (at most UN per thread: fewer than UN after the main loop, and
        # NC < UN * nthr when it never ran): one group of predicated loads, all issued
        # before any is accumulated, so the remainder costs one memory latency, not one each
        loaded = []
        for u in range(UN):
            cu, pu = gen.register(".u32"), gen.register(".pred")
            gen.emit(f"add.u32 {cu}, {c}, {u * nthr};")
            gen.emit(f"setp.lt.u32 {pu}, {cu}, {NC};")
            off = gen.register(".u64")
            gen.emit(f"mul.wide.u32 {off}, {cu}, 16;")
            vals = {}
            for b in elem_bufs:
                a = gen.register(".u64")
                gen.emit(f"add.s64 {a}, {ptrs[b]}, {off};")
                regs = gen.registers(".f32", 4)
                gen.emit(f"@{pu} ld.global.nc.L1::no_allocate.v4.f32 "
                         f"{{{', '.join(regs)}}}, [{a}];")
                vals[b] = regs
            loaded.append((pu, vals))
        for u, (pu, vals) in enumerate(loaded):
            L_skip = gen.new_label("remskip")
            gen.emit(f"@!{pu} bra {L_skip};")
            for ln in range(4):
                accumulate({b: vals[b][ln] for b in elem_bufs}, chunk=u)
            gen.label(L_skip)
        gen.emit(f"add.u32 {start}, {gtid}, {NC * 4};")
    else:
        gen.emit(f"mov.u32 {start}, {gtid};")
    # scalar tail (or everything, when misaligned)
    gen.label(L_scalar)
    e = gen.register(".u32")
    gen.emit(f"mov.u32 {e}, {start};")
    L_s = gen.new_label("s")
    ps = gen.register(".pred")
    gen.label(L_s)
    gen.emit(f"setp.ge.u32 {ps}, {e}, {L};")
    gen.emit(f"@{ps} bra {L_reduce};")
    off = gen.register(".u64")
    gen.emit(f"mul.wide.u32 {off}, {e}, 4;")
    sv = {}
    for b in elem_bufs:
        a = gen.register(".u64")
        gen.emit(f"add.s64 {a}, {ptrs[b]}, {off};")
        r = gen.register(".f32")
        gen.emit(f"ld.global.nc.f32 {r}, [{a}];")
        sv[b] = r
    accumulate(sv)
    gen.emit(f"add.u32 {e}, {e}, {nthr};")
    gen.emit(f"bra.uni {L_s};")
    gen.label(L_reduce)
    # Launched with programmatic stream serialization (no effect under a plain launch), the
    # next kernel may start once every CTA of this one has triggered: past EARLY_TRIGGER of
    # the input in the main loop, else here, when this thread has finished streaming. Every
    # global write (partials, ticket, result) waits for the previous kernel to finish.
    L_trigged = gen.new_label("trigged")
    gen.emit(f"@{p_trig} bra {L_trigged};")
    gen.emit("griddepcontrol.launch_dependents;")
    gen.label(L_trigged)
    gen.emit("griddepcontrol.wait;")

    # CTA partial -> global scratch, then the ticket
    if exact:
        part = red.block_reduce_f64(red.merge_sets(sets), lane, warp, broadcast=False)
        if G > 1:
            part = _cross_cta_fold_f64(gen, red, part, tid, cta, lane, warp, G, S, B)
        total = red.narrow(part)
    else:
        part, pvalid = red.block_reduce(states, valid, tid, lane, warp, broadcast=False)
        if G == 1:
            # one CTA (CTAs beyond the compiled grid return above): its partial is the result
            total = part
        else:
            total = _cross_cta_fold(gen, red, part, pvalid, tid, cta, lane, warp, G, S, B,
                                    track)
    p_w = gen.register(".pred")
    gen.emit(f"setp.ne.u32 {p_w}, {tid}, 0;")
    gen.emit(f"@{p_w} ret;")
    env = dict(zip(plan.states, total))

    def uload(p):
        return uniforms[p.name]

    run_program(gen, plan.post, env, load=uload)

    def fwrite(p, reg):
        gen.emit(f"st.global.f32 [{ptrs[p.buffer]}], {reg};")
    run_program(gen, plan.final, env, load=uload, write=fwrite)
    gen.emit("ret;")


# ---------------------------------------------------------------------------
# per-row reductions and fused row operations
# ---------------------------------------------------------------------------

def _lower_rows(gen, kernel, plan, B):
    L, R = plan.length, plan.rows
    S = len(plan.states)
    ptrs = load_pointers(gen, list(kernel.arg_order))
    # Launched with programmatic stream serialization (EMMY_RT_LAUNCH_OVERLAP; no effect under
    # a plain launch), the next kernel on the stream may be scheduled once every CTA of this
    # one has started, and this kernel touches global memory only after the previous one has
    # finished: a chain of launches keeps its order and only the launch latency overlaps
    # (the CTAs of the last wave are the last to trigger).
    gen.emit("griddepcontrol.launch_dependents;")
    gen.emit("griddepcontrol.wait;")
    uniforms = _hoist_uniforms(gen, plan, ptrs)
    NC = L // 4
    vec_ok = L % 4 == 0 and NC > 0
    everyone_works = (NC >= B) if vec_ok else (L >= B)
    exact = exact_sum(plan)
    track = not combine_identity_safe(plan) and not everyone_works
    red = _Reducer(gen, plan, B, track, f64=exact)

    pass2_elem = []
    if plan.pass2:
        pass2_elem = list(dict.fromkeys(p.buffer for p in plan.pass2
                                        if isinstance(p, ElemLoad) and p.kind == "elem"))
    pass1_elem = list(dict.fromkeys(p.buffer for p in plan.pass1
                                    if isinstance(p, ElemLoad) and p.kind == "elem"))
    staged = [b for b in pass1_elem if b in pass2_elem] if vec_ok else []
    if len(staged) * L * 4 > SMEM_STAGE_LIMIT:
        staged = []
    out_elem = [p.buffer for p in (plan.pass2 or []) if isinstance(p, ElemWrite)]
    col_bufs = plan.col_buffers
    row_bytes = L * 4

    tid, lane, warp, row, nrows_step = (gen.register(".u32") for _ in range(5))
    gen.emit(f"mov.u32 {tid}, %tid.x;")
    gen.emit(f"and.b32 {lane}, {tid}, 31;")
    gen.emit(f"shr.u32 {warp}, {tid}, 5;")
    gen.emit(f"mov.u32 {row}, %ctaid.x;")
    gen.emit(f"mov.u32 {nrows_step}, %nctaid.x;")

    align_bufs = list(dict.fromkeys(pass1_elem + pass2_elem + out_elem + col_bufs))
    p_vec = None
    if vec_ok:
        p_vec = aligned_predicate(gen, ptrs, align_bufs)
        if row_bytes % 16:
            raise AssertionError("vector rows must be 16-byte multiples")

    mbar = phase = None
    if staged:
        gen.shared("emmy_rows", ".b8", length=len(staged) * row_bytes, align=128)
        gen.shared("emmy_mbar", ".b64", length=1, align=8)
        mbar = gen.register(".u32")
        gen.emit(f"mov.u32 {mbar}, emmy_mbar;")
        phase = gen.register(".u32")
        gen.emit(f"mov.u32 {phase}, 0;")
        p_t0 = gen.register(".pred")
        gen.emit(f"setp.eq.u32 {p_t0}, {tid}, 0;")
        gen.emit(f"@{p_t0} mbarrier.init.shared::cta.b64 [{mbar}], 1;")
        gen.emit("fence.mbarrier_init.release.cluster;")
        gen.emit("bar.sync 0;")

    # column operands of the output pass (an RMSNorm weight) do not depend on the row: with
    # few chunks per thread they are loaded once, up front (read-only path; predicated on
    # the alignment check and the chunk bound), instead of after each chunk's output stores
    pre_cols = {}
    pass2_cols = [b for b in col_bufs if any(isinstance(p, ElemLoad) and p.kind == "col"
                                             and p.buffer == b for p in (plan.pass2 or []))]
    if vec_ok and pass2_cols and -(-NC // B) <= UNROLLED_CHUNKS \
            and not set(pass2_cols) & set(out_elem):
        for k in range(-(-NC // B)):
            c = gen.register(".u32")
            gen.emit(f"add.u32 {c}, {tid}, {k * B};")
            pk = gen.register(".pred")
            gen.emit(f"setp.lt.and.u32 {pk}, {c}, {NC}, {p_vec};")
            o = gen.register(".u64")
            gen.emit(f"mul.wide.u32 {o}, {c}, 16;")
            pre_cols[k] = {}
            for b in pass2_cols:
                a = gen.register(".u64")
                gen.emit(f"add.s64 {a}, {ptrs[b]}, {o};")
                regs = gen.registers(".f32", 4)
                gen.emit(f"@{pk} ld.global.nc.v4.f32 {{{', '.join(regs)}}}, [{a}];")
                pre_cols[k][b] = regs

    L_row = gen.new_label("row")
    L_done = gen.new_label("done")
    prow = gen.register(".pred")
    gen.label(L_row)
    gen.emit(f"setp.ge.u32 {prow}, {row}, {R};")
    gen.emit(f"@{prow} bra {L_done};")
    roff = gen.register(".u64")
    gen.emit(f"mul.wide.u32 {roff}, {row}, {row_bytes};")
    rowptr = {}
    for b in dict.fromkeys(pass1_elem + pass2_elem + out_elem):
        r = gen.register(".u64")
        gen.emit(f"add.s64 {r}, {ptrs[b]}, {roff};")
        rowptr[b] = r

    states = red.identity_states()
    sets = red.f64_sets(1) if exact else None
    hook = red.f64_hook(sets, [0]) if exact else None
    accum_regs = dict(zip(plan.states, states))
    valid = None
    if track:
        valid = gen.register(".pred")
        gen.emit(f"setp.ne.u32 {valid}, 0, 0;")

    def accumulate(values, colvals):
        def load(p):
            if p.kind == "uniform":
                return uniforms[p.name]
            if p.kind == "col":
                return colvals[p.buffer]
            return values[p.buffer]
        run_program(gen, plan.pass1, {}, load=load, accum_regs=accum_regs, accum=hook)
        if track:
            gen.emit(f"setp.eq.u32 {valid}, 0, 0;")

    L_scalar1 = gen.new_label("scalar1")
    L_stats = gen.new_label("stats")
    staged_ptr = {}
    if vec_ok:
        gen.emit(f"@!{p_vec} bra {L_scalar1};")
        if staged:
            base = gen.register(".u32")
            gen.emit(f"mov.u32 {base}, emmy_rows;")
            for k, b in enumerate(staged):
                sp = gen.register(".u32")
                gen.emit(f"add.u32 {sp}, {base}, {k * row_bytes};")
                staged_ptr[b] = sp
            p_t0 = gen.register(".pred")
            gen.emit(f"setp.eq.u32 {p_t0}, {tid}, 0;")
            L_noissue = gen.new_label("noissue")
            gen.emit(f"@!{p_t0} bra {L_noissue};")
            gen.emit(f"mbarrier.arrive.expect_tx.shared::cta.b64 _, [{mbar}], "
                     f"{len(staged) * row_bytes};")
            for b in staged:
                gen.emit(f"cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes "
                         f"[{staged_ptr[b]}], [{rowptr[b]}], {row_bytes}, [{mbar}];")
            gen.label(L_noissue)
            _emit_wait(gen, mbar, phase)
            gen.emit(f"xor.b32 {phase}, {phase}, 1;")
        # pass 1 over 16-byte chunks c = tid + k*B
        _chunk_loop(gen, tid, NC, B, lambda c, k: _accum_chunk(
            gen, c, pass1_elem, staged_ptr, rowptr, col_bufs, ptrs, accumulate))
        gen.emit(f"bra.uni {L_stats};")
    gen.label(L_scalar1)
    if True:
        e = gen.register(".u32")
        gen.emit(f"mov.u32 {e}, {tid};")
        L_s1 = gen.new_label("s1")
        ps = gen.register(".pred")
        gen.label(L_s1)
        gen.emit(f"setp.ge.u32 {ps}, {e}, {L};")
        gen.emit(f"@{ps} bra {L_stats};")
        eo = gen.register(".u64")
        gen.emit(f"mul.wide.u32 {eo}, {e}, 4;")
        vals, cols = {}, {}
        for b in pass1_elem:
            a = gen.register(".u64")
            gen.emit(f"add.s64 {a}, {rowptr[b]}, {eo};")
            r = gen.register(".f32")
            gen.emit(f"ld.global.f32 {r}, [{a}];")
            vals[b] = r
        for b in col_bufs:
            a = gen.register(".u64")
            gen.emit(f"add.s64 {a}, {ptrs[b]}, {eo};")
            r = gen.register(".f32")
            gen.emit(f"ld.global.nc.f32 {r}, [{a}];")
            cols[b] = r
        accumulate(vals, cols)
        gen.emit(f"add.u32 {e}, {e}, {B};")
        gen.emit(f"bra.uni {L_s1};")
    gen.label(L_stats)

    if exact:      # a row sum: only thread 0 writes, so no broadcast is needed
        total = red.narrow(red.block_reduce_f64(sets[0], lane, warp, broadcast=False))
    else:
        total, _ = red.block_reduce(states, valid, tid, lane, warp, broadcast=True)
    env = dict(zip(plan.states, total))

    def uload(p):
        return uniforms[p.name]
    run_program(gen, plan.post, env, load=uload)

    if plan.pass2:
        L_scalar2 = gen.new_label("scalar2")
        L_next = gen.new_label("next")
        if vec_ok:
            gen.emit(f"@!{p_vec} bra {L_scalar2};")
            _chunk_loop(gen, tid, NC, B, lambda c, k: _output_chunk(
                gen, c, plan, env, uniforms, pass2_elem, staged_ptr, rowptr, col_bufs, ptrs,
                pre_cols.get(k) if k is not None else None))
            gen.emit(f"bra.uni {L_next};")
        gen.label(L_scalar2)
        e2 = gen.register(".u32")
        gen.emit(f"mov.u32 {e2}, {tid};")
        L_s2 = gen.new_label("s2")
        ps2 = gen.register(".pred")
        gen.label(L_s2)
        gen.emit(f"setp.ge.u32 {ps2}, {e2}, {L};")
        gen.emit(f"@{ps2} bra {L_next};")
        eo2 = gen.register(".u64")
        gen.emit(f"mul.wide.u32 {eo2}, {e2}, 4;")

        def sload(p):
            if p.kind == "uniform":
                return uniforms[p.name]
            base_ptr = ptrs[p.buffer] if p.kind == "col" else rowptr[p.buffer]
            a = gen.register(".u64")
            gen.emit(f"add.s64 {a}, {base_ptr}, {eo2};")
            r = gen.register(".f32")
            gen.emit(f"ld.global.f32 {r}, [{a}];")
            return r

        def swrite(p, reg):
            a = gen.register(".u64")
            gen.emit(f"add.s64 {a}, {rowptr[p.buffer]}, {eo2};")
            gen.emit(f"st.global.f32 [{a}], {reg};")
        run_program(gen, plan.pass2, dict(env), load=sload, write=swrite)
        gen.emit(f"add.u32 {e2}, {e2}, {B};")
        gen.emit(f"bra.uni {L_s2};")
        gen.label(L_next)
    else:
        p_nt0 = gen.register(".pred")
        gen.emit(f"setp.ne.u32 {p_nt0}, {tid}, 0;")
        L_skipw = gen.new_label("skipw")
        gen.emit(f"@{p_nt0} bra {L_skipw};")
        fenv = dict(env)

        def rwrite(p, reg):
            a = gen.register(".u64")
            o = gen.register(".u64")
            gen.emit(f"mul.wide.u32 {o}, {row}, 4;")
            gen.emit(f"add.s64 {a}, {ptrs[p.buffer]}, {o};")
            gen.emit(f"st.global.f32 [{a}], {reg};")
        run_program(gen, plan.final, fenv, load=uload, write=rwrite)
        gen.label(L_skipw)
    # shared staging and the reduction scratch are reused by the next row
    gen.emit("bar.sync 0;")
    gen.emit(f"add.u32 {row}, {row}, {nrows_step};")
    gen.emit(f"bra.uni {L_row};")
    gen.label(L_done)
    gen.emit("ret;")


def _chunk_loop(gen, tid, NC, B, body):
    """Run ``body(c, k)`` for chunks ``c = tid + k*B < NC``; fully unrolled when short
    (``k`` is then the unrolled index, else None)."""
    per = -(-NC // B)
    if per <= UNROLLED_CHUNKS:
        for k in range(per):
            c = gen.register(".u32")
            gen.emit(f"add.u32 {c}, {tid}, {k * B};")
            if (k + 1) * B > NC:
                p = gen.register(".pred")
                skip = gen.new_label("cskip")
                gen.emit(f"setp.ge.u32 {p}, {c}, {NC};")
                gen.emit(f"@{p} bra {skip};")
                body(c, k)
                gen.label(skip)
            else:
                body(c, k)
        return
    c = gen.register(".u32")
    gen.emit(f"mov.u32 {c}, {tid};")
    L = gen.new_label("chunks")
    Ld = gen.new_label("chunksdone")
    p = gen.register(".pred")
    gen.label(L)
    gen.emit(f"setp.ge.u32 {p}, {c}, {NC};")
    gen.emit(f"@{p} bra {Ld};")
    body(c, None)
    gen.emit(f"add.u32 {c}, {c}, {B};")
    gen.emit(f"bra.uni {L};")
    gen.label(Ld)


def _vec_load(gen, c, base, shared):
    regs = gen.registers(".f32", 4)
    if shared:
        o = gen.register(".u32")
        gen.emit(f"shl.b32 {o}, {c}, 4;")
        a = gen.register(".u32")
        gen.emit(f"add.u32 {a}, {base}, {o};")
        gen.emit(f"ld.shared.v4.f32 {{{', '.join(regs)}}}, [{a}];")
    else:
        o = gen.register(".u64")
        gen.emit(f"mul.wide.u32 {o}, {c}, 16;")
        a = gen.register(".u64")
        gen.emit(f"add.s64 {a}, {base}, {o};")
        gen.emit(f"ld.global.v4.f32 {{{', '.join(regs)}}}, [{a}];")
    return regs


def _accum_chunk(gen, c, elem_bufs, staged_ptr, rowptr, col_bufs, ptrs, accumulate):
    vals = {}
    for b in elem_bufs:
        if b in staged_ptr:
            vals[b] = _vec_load(gen, c, staged_ptr[b], True)
        else:
            vals[b] = _vec_load(gen, c, rowptr[b], False)
    cols = {b: _vec_load(gen, c, ptrs[b], False) for b in col_bufs}
    for ln in range(4):
        accumulate({b: v[ln] for b, v in vals.items()}, {b: v[ln] for b, v in cols.items()})


def _output_chunk(gen, c, plan, env, uniforms, elem_bufs, staged_ptr, rowptr, col_bufs, ptrs,
                  pre=None):
    vals = {}
    for b in elem_bufs:
        if b in staged_ptr:
            vals[b] = _vec_load(gen, c, staged_ptr[b], True)
        else:
            vals[b] = _vec_load(gen, c, rowptr[b], False)
    used_cols = [b for b in col_bufs if any(isinstance(p, ElemLoad) and p.kind == "col"
                                            and p.buffer == b for p in plan.pass2)]
    cols = {b: (pre[b] if pre and b in pre else _vec_load(gen, c, ptrs[b], False))
            for b in used_cols}
    results = {}
    for ln in range(4):
        def load(p, ln=ln):
            if p.kind == "uniform":
                return uniforms[p.name]
            if p.kind == "col":
                return cols[p.buffer][ln]
            return vals[p.buffer][ln]

        def write(p, reg, ln=ln):
            results.setdefault(p.buffer, [None] * 4)[ln] = reg
        run_program(gen, plan.pass2, dict(env), load=load, write=write)
    for b, regs in results.items():
        o = gen.register(".u64")
        gen.emit(f"mul.wide.u32 {o}, {c}, 16;")
        a = gen.register(".u64")
        gen.emit(f"add.s64 {a}, {rowptr[b]}, {o};")
        gen.emit(f"st.global.v4.f32 [{a}], {{{', '.join(regs)}}};")


def _cross_cta_fold_f64(gen, red, part, tid, cta, lane, warp, G, S, B):
    """The cross-CTA finish of a compensated sum: as ``_cross_cta_fold`` with f64 partials
    (``emmy_partials64``); the last CTA adds them, each thread a fixed subset in CTA order,
    then the f64 block tree (deterministic for a given grid). Returns the f64 total in
    thread 0; other CTAs return."""
    p_t0 = gen.register(".pred")
    gen.emit(f"setp.eq.u32 {p_t0}, {tid}, 0;")
    L_not0 = gen.new_label("not0")
    gen.emit(f"@!{p_t0} bra {L_not0};")
    pa = gen.register(".u64")
    gen.emit(f"mov.u64 {pa}, emmy_partials64;")
    poff = gen.register(".u64")
    gen.emit(f"mul.wide.u32 {poff}, {cta}, 8;")
    gen.emit(f"add.s64 {pa}, {pa}, {poff};")
    for i, d in enumerate(part):
        gen.emit(f"st.global.f64 [{pa}+{i * G * 8}], {d};")
    old = gen.register(".u32")
    gen.emit(f"atom.acq_rel.gpu.global.inc.u32 {old}, [emmy_ticket], {G - 1};")
    last = gen.register(".u32")
    pl = gen.register(".pred")
    gen.emit(f"setp.eq.u32 {pl}, {old}, {G - 1};")
    gen.emit(f"selp.u32 {last}, 1, 0, {pl};")
    gen.emit(f"st.shared.u32 [emmy_last], {last};")
    gen.label(L_not0)
    gen.emit("bar.sync 0;")
    lastv = gen.register(".u32")
    gen.emit(f"ld.shared.u32 {lastv}, [emmy_last];")
    pnl = gen.register(".pred")
    gen.emit(f"setp.eq.u32 {pnl}, {lastv}, 0;")
    gen.emit(f"@{pnl} ret;")

    gen.emit("fence.acq_rel.gpu;")
    acc = []
    for _ in range(S):
        d = gen.register(".f64")
        gen.emit(f"mov.f64 {d}, 0d0000000000000000;")
        acc.append(d)
    rounds = -(-G // B)
    if rounds <= FOLD_UNROLL:
        # every partial this thread adds is requested before the first is added: one L2
        # round trip instead of one per partial (592 partials, 256 threads: 3 -> 1)
        base = gen.register(".u64")
        gen.emit(f"mov.u64 {base}, emmy_partials64;")
        off = gen.register(".u64")
        gen.emit(f"mul.wide.u32 {off}, {tid}, 8;")
        gen.emit(f"add.s64 {base}, {base}, {off};")
        loaded = []
        for r in range(rounds):
            pr = gen.register(".pred")
            gen.emit(f"setp.lt.u32 {pr}, {tid}, {G - r * B};")
            vals = []
            for k in range(S):
                v = gen.register(".f64")
                gen.emit(f"mov.f64 {v}, 0d0000000000000000;")
                gen.emit(f"@{pr} ld.relaxed.gpu.global.f64 {v}, "
                         f"[{base}+{(k * G + r * B) * 8}];")
                vals.append(v)
            loaded.append(vals)
        for vals in loaded:
            for k in range(S):
                gen.emit(f"add.rn.f64 {acc[k]}, {acc[k]}, {vals[k]};")
        return red.block_reduce_f64(acc, lane, warp, broadcast=False)
    i = gen.register(".u32")
    gen.emit(f"mov.u32 {i}, {tid};")
    L_f = gen.new_label("fold64")
    L_fd = gen.new_label("fold64done")
    pf = gen.register(".pred")
    gen.label(L_f)
    gen.emit(f"setp.ge.u32 {pf}, {i}, {G};")
    gen.emit(f"@{pf} bra {L_fd};")
    fa = gen.register(".u64")
    gen.emit(f"mov.u64 {fa}, emmy_partials64;")
    fo = gen.register(".u64")
    gen.emit(f"mul.wide.u32 {fo}, {i}, 8;")
    gen.emit(f"add.s64 {fa}, {fa}, {fo};")
    for k in range(S):
        r = gen.register(".f64")
        gen.emit(f"ld.relaxed.gpu.global.f64 {r}, [{fa}+{k * G * 8}];")
        gen.emit(f"add.rn.f64 {acc[k]}, {acc[k]}, {r};")
    gen.emit(f"add.u32 {i}, {i}, {B};")
    gen.emit(f"bra.uni {L_f};")
    gen.label(L_fd)
    return red.block_reduce_f64(acc, lane, warp, broadcast=False)


def _cross_cta_fold(gen, red, part, pvalid, tid, cta, lane, warp, G, S, B, track):
    """Single-pass cross-CTA finish: each CTA stores its partial (and validity), takes a
    ticket; the last CTA to arrive folds the G partials in CTA order (deterministic) and
    returns the block-reduced total in thread 0 (other CTAs return)."""
    p_t0 = gen.register(".pred")
    gen.emit(f"setp.eq.u32 {p_t0}, {tid}, 0;")
    L_not0 = gen.new_label("not0")
    gen.emit(f"@!{p_t0} bra {L_not0};")
    pa = gen.register(".u64")
    gen.emit(f"mov.u64 {pa}, emmy_partials;")
    poff = gen.register(".u64")
    gen.emit(f"mul.wide.u32 {poff}, {cta}, 4;")
    gen.emit(f"add.s64 {pa}, {pa}, {poff};")
    for i, r in enumerate(part):
        gen.emit(f"st.global.f32 [{pa}+{i * G * 4}], {r};")
    if track:
        va = gen.register(".u64")
        gen.emit(f"mov.u64 {va}, emmy_pvalid;")
        gen.emit(f"add.s64 {va}, {va}, {poff};")
        vu = gen.register(".u32")
        gen.emit(f"selp.u32 {vu}, 1, 0, {pvalid};")
        gen.emit(f"st.global.u32 [{va}], {vu};")
    old = gen.register(".u32")
    gen.emit(f"atom.acq_rel.gpu.global.inc.u32 {old}, [emmy_ticket], {G - 1};")
    last = gen.register(".u32")
    pl = gen.register(".pred")
    gen.emit(f"setp.eq.u32 {pl}, {old}, {G - 1};")
    gen.emit(f"selp.u32 {last}, 1, 0, {pl};")
    gen.emit(f"st.shared.u32 [emmy_last], {last};")
    gen.label(L_not0)
    gen.emit("bar.sync 0;")
    lastv = gen.register(".u32")
    gen.emit(f"ld.shared.u32 {lastv}, [emmy_last];")
    pnl = gen.register(".pred")
    gen.emit(f"setp.eq.u32 {pnl}, {lastv}, 0;")
    gen.emit(f"@{pnl} ret;")

    # last CTA: fold the G partials in CTA order
    gen.emit("fence.acq_rel.gpu;")
    fstates = red.identity_states()
    fvalid = None
    if track:
        fvalid = gen.register(".pred")
        gen.emit(f"setp.ne.u32 {fvalid}, 0, 0;")
    i = gen.register(".u32")
    gen.emit(f"mov.u32 {i}, {tid};")
    L_f = gen.new_label("fold")
    L_fd = gen.new_label("folddone")
    pf = gen.register(".pred")
    gen.label(L_f)
    gen.emit(f"setp.ge.u32 {pf}, {i}, {G};")
    gen.emit(f"@{pf} bra {L_fd};")
    fa = gen.register(".u64")
    gen.emit(f"mov.u64 {fa}, emmy_partials;")
    fo = gen.register(".u64")
    gen.emit(f"mul.wide.u32 {fo}, {i}, 4;")
    gen.emit(f"add.s64 {fa}, {fa}, {fo};")
    loaded = []
    for k in range(S):
        r = gen.register(".f32")
        gen.emit(f"ld.relaxed.gpu.global.f32 {r}, [{fa}+{k * G * 4}];")
        loaded.append(r)
    if track:
        fva = gen.register(".u64")
        gen.emit(f"mov.u64 {fva}, emmy_pvalid;")
        gen.emit(f"add.s64 {fva}, {fva}, {fo};")
        lv = gen.register(".u32")
        gen.emit(f"ld.relaxed.gpu.global.u32 {lv}, [{fva}];")
        plv = gen.register(".pred")
        gen.emit(f"setp.ne.u32 {plv}, {lv}, 0;")
        new = red.combine(fstates, loaded, fvalid, plv)
        gen.emit(f"or.pred {fvalid}, {fvalid}, {plv};")
    else:
        new = red.combine(fstates, loaded)
    for d, r in zip(fstates, new):
        gen.emit(f"mov.f32 {d}, {r};")
    gen.emit(f"add.u32 {i}, {i}, {B};")
    gen.emit(f"bra.uni {L_f};")
    gen.label(L_fd)
    total, _ = red.block_reduce(fstates, fvalid, tid, lane, warp, broadcast=False)
    return total
