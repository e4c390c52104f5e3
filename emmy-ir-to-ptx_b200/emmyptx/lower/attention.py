"""Attention template: O = softmax(q @ kt / c) @ v on tcgen05 with TMEM accumulators.

The IR expresses attention as a per-thread online softmax over the key axis
(reference ``problems/a01_attention``; lowered statement by statement by
reference ``compile.py:4858-5579``). This template keeps that computation and
schedules it flash-style for B200, one work item per (batch*head, 128 query
rows), 3xTF32 on both products (hi*hi + hi*lo + lo*hi, as the contraction
template) so that the result stays within 1e-4 of the fp64 attention.

Warp roles (256 threads):

* warps 0-3, one query row per thread (warp w owns TMEM lanes 32w..32w+31):
  split the Q row into TF32 hi/lo and store both into tensor memory with
  ``tcgen05.st`` (the S product reads A from TMEM); per key block read S with
  ``tcgen05.ld``, run the online softmax in registers (base-2 exponentials,
  log2(e) folded into the scale, one FFMA + ``ex2`` per score), and write
  P_hi / P_lo to tensor memory with ``tcgen05.st`` (D = 32, 64, 128), or to shared memory
  in the K-major SWIZZLE_128B layout where tensor memory has no room for it
  (D = 96). The output accumulator
  O stays in tensor memory; the running maximum is only raised when a row's
  block maximum exceeds it by more than 2^8 (then that warp rescales its O rows
  in TMEM), so most blocks need no correction at all. The next work item's Q
  rows are fetched during the last key block and stored as soon as the last S
  product has landed. Finally O / l is stored;
* warp 4: one ``elect.sync`` lane issues S_j = Q K_j^T (A in TMEM, B in shared
  memory) into one of two S buffers and O += P_j V_j (A = P in tensor or shared
  memory, B in shared memory); S runs one block ahead of P*V so the tensor core
  overlaps the softmax;
* warps 5-7: fill the kt and v tiles of each key block, MN-major in
  SWIZZLE_128B_BASE32B (the TF32 MN-major layout). When the runtime has written
  tensor maps for the launch's kt and v pointers, warp 5 copies each raw tile
  with ``cp.async.bulk.tensor`` (the raw f32 words serve as the hi operand: the
  MMA reads their top 19 bits) and warps 6-7 write the lo tile from it; with one
  buffer per tile (D = 96, or a launch whose shared memory holds only one) the
  MMA warp issues the products that read only the raw tile (hi x hi, lo x hi) as
  soon as the copy lands and the hi x lo products once the lo tile is written.
  Otherwise all three warps load the tiles with 16-byte loads (the next kt tile in
  flight while the v tile waits for its buffer), split them and store hi and lo.
  Both paths give the same bits.

Hand-offs use mbarriers (loads -> MMA, MMA commit -> softmax, softmax -> MMA);
every wait is bounded and warp-uniform; on expiry it sets bit 3 of
``emmy_error`` and leaves through the common exit, which waits (bounded) for
the issued MMAs and frees the tensor memory.
"""

from __future__ import annotations

from math import gcd

from . import tmap
from .common import WAIT_LIMIT, pack2, tf32_split_pairs, unpack2

TQ = 128
# keys per block. At D = 128, 32-key blocks let P live in tensor memory (Q hi/lo 256 + two S
# buffers 64 + O 128 + P hi/lo 64 = 512 columns), which leaves the shared memory room for two
# kt and two v buffers: with TMA-fed tiles and one barrier wait per product they ran 7.6 %
# faster than 64-key blocks with one buffer each (interleaved on a B200); with register-staged
# tiles and more hand-offs per block they had been slower (1.151 against 1.08 ms)
BKV_FOR_D = {32: 64, 64: 64, 96: 64, 128: 32}
THREADS = 256
NLOAD = 96                 # loader threads: warps 5-7
NWORK = 64                 # TMA path: lo-tile workers, warps 6-7 (warp 5 issues the copies)
RESCALE_BITS = "0f41000000"   # 8.0: raise the running maximum only past 2^8 of growth


def _p_in_tmem(D, BKV):
    return 3 * D + 4 * BKV <= 512


def smem_bytes_needed(D, nbuf=1):
    """Dynamic shared memory of the template: ``nbuf`` kt and v tile pairs (hi and lo each),
    plus P hi/lo when P does not fit in tensor memory."""
    BKV = BKV_FOR_D[D]
    tiles = nbuf * 2 * (D * BKV * 4) * 2
    return tiles + (0 if _p_in_tmem(D, BKV) else 2 * (TQ * BKV * 4))


def tile_buffers(D, smem):
    """kt/v tile buffers: two when the launch's shared memory holds them (a tile can then be
    stored while the tensor core still reads the other), else one; always one at D = 96, whose
    P takes shared memory too."""
    return 2 if D != 96 and smem >= smem_bytes_needed(D, 2) else 1


def fits(plan, launch):
    block = list(launch.get("block", [1, 1, 1]))
    grid = list(launch.get("grid", [1, 1, 1]))
    if block != [THREADS, 1, 1] or grid[1:] != [1, 1]:
        return False
    if plan.D not in BKV_FOR_D or plan.Dv != plan.D:
        return False
    if plan.Sq % TQ or plan.Skv % BKV_FOR_D[plan.D]:
        return False
    return int(launch.get("smem_bytes", 0) or 0) >= smem_bytes_needed(plan.D)


class _Wait:
    """Bounded, warp-uniform ``mbarrier.try_wait.parity`` loops.

    Every wait in this template is executed by whole warps; the lanes vote on
    the result so that they leave the loop together (on success or on expiry)
    and the warp stays converged for the ``.sync.aligned`` tensor-memory
    instructions that follow. On expiry bit 3 of ``emmy_error`` is set and the
    warp jumps to ``exit_label`` (or falls through when it is None)."""

    def __init__(self, gen, exit_label):
        self.gen, self.exit = gen, exit_label

    def __call__(self, mbar, parity, exit_label="default"):
        gen = self.gen
        target = self.exit if exit_label == "default" else exit_label
        it = gen.register(".u32")
        p, pa, pl = gen.register(".pred"), gen.register(".pred"), gen.register(".pred")
        top, ok = gen.new_label("aw"), gen.new_label("awok")
        gen.emit(f"mov.u32 {it}, 0;")
        gen.label(top)
        gen.emit(f"mbarrier.try_wait.parity.shared::cta.b64 {p}, [{mbar}], {parity};")
        gen.emit(f"vote.sync.all.pred {pa}, {p}, -1;")
        gen.emit(f"@{pa} bra.uni {ok};")
        gen.emit(f"add.u32 {it}, {it}, 1;")
        gen.emit(f"setp.lt.u32 {pl}, {it}, {WAIT_LIMIT};")
        gen.emit(f"@{pl} bra.uni {top};")
        gen.emit("red.global.or.b32 [emmy_error], 8;")
        if target is not None:
            gen.emit(f"bra.uni {target};")
        gen.label(ok)


def _mn32_offset(gen, krow, ncol4, sbo, lbo=512):
    """Byte offset of the 16-byte chunk (k = krow, n = 4*ncol4 .. +3) in an MN-major
    SWIZZLE_128B_BASE32B tile: 32 n x 4 k atoms of 512 bytes, ``lbo`` bytes apart along n and
    ``sbo`` bytes apart along k (4-row groups), the 32-byte units of each 128-byte k row
    permuted by XOR with k % 4. With ``lbo`` = rows x 128 and ``sbo`` = 512 each 32-wide
    column strip is one contiguous run of 128-byte rows: the layout a TMA box of 32 columns
    writes with the 128-byte swizzle of 32-byte atoms."""
    j, c8, unit, half, k4, kq, off = (gen.register(".u32") for _ in range(7))
    gen.emit(f"shr.u32 {j}, {ncol4}, 3;")
    gen.emit(f"and.b32 {c8}, {ncol4}, 7;")
    gen.emit(f"shr.u32 {unit}, {c8}, 1;")
    gen.emit(f"and.b32 {half}, {c8}, 1;")
    gen.emit(f"and.b32 {k4}, {krow}, 3;")
    gen.emit(f"shr.u32 {kq}, {krow}, 2;")
    gen.emit(f"mul.lo.u32 {off}, {kq}, {sbo};")
    gen.emit(f"mad.lo.u32 {off}, {j}, {lbo}, {off};")
    gen.emit(f"mad.lo.u32 {off}, {k4}, 128, {off};")
    gen.emit(f"xor.b32 {unit}, {unit}, {k4};")
    gen.emit(f"mad.lo.u32 {off}, {unit}, 32, {off};")
    gen.emit(f"mad.lo.u32 {off}, {half}, 16, {off};")
    return off


class _TileCopy:
    """One loader thread's share of a rows x cols f32 tile (row-major in global memory,
    ``row_stride`` floats per row) copied into hi/lo MN-major SWIZZLE_128B_BASE32B tiles.

    Thread ``lt`` owns the 16-byte chunks lt, lt + 96, lt + 192, ...; 96 is a multiple of
    the chunks per row, so its column group is fixed and its rows advance by ``rstep``.
    Global offsets are then immediates, and shared-memory offsets repeat with period
    ``P`` (rows mod 4) up to an immediate: both are set up once per kernel."""

    def __init__(self, gen, lt, *, rows, cols, row_stride, sbo, base, lbo=512):
        per_row = cols // 4
        assert NLOAD % per_row == 0
        self.gen, self.rows, self.sbo = gen, rows, sbo
        self.rstep = NLOAD // per_row
        self.iters = -(-(rows * per_row) // NLOAD)
        self.P = 4 // gcd(self.rstep, 4)
        self.gstep = self.rstep * row_stride * 4
        r0, cn = gen.register(".u32"), gen.register(".u32")
        gen.emit(f"div.u32 {r0}, {lt}, {per_row};")
        gen.emit(f"rem.u32 {cn}, {lt}, {per_row};")
        e = gen.register(".u32")
        gen.emit(f"mul.lo.u32 {e}, {r0}, {row_stride};")
        gen.emit(f"mad.lo.u32 {e}, {cn}, 4, {e};")
        self.goff = gen.register(".u64")
        gen.emit(f"mul.wide.u32 {self.goff}, {e}, 4;")
        self.bases = []
        for t in range(min(self.P, self.iters)):
            rt = gen.register(".u32")
            gen.emit(f"add.u32 {rt}, {r0}, {self.rstep * t};")
            off = _mn32_offset(gen, rt, cn, sbo, lbo)
            gen.emit(f"add.u32 {off}, {off}, {base};")
            self.bases.append(off)
        self.pv = None
        if self.iters * NLOAD > rows * per_row:
            self.pv = gen.register(".pred")
            rl = gen.register(".u32")
            gen.emit(f"add.u32 {rl}, {r0}, {self.rstep * (self.iters - 1)};")
            gen.emit(f"setp.lt.u32 {self.pv}, {rl}, {rows};")

    def load(self, tile, into=None):
        """Issue the loads of the tile starting at global address ``tile`` (u64 register)."""
        gen = self.gen
        out = into if into is not None else [gen.registers(".f32", 4) for _ in range(self.iters)]
        a = gen.register(".u64")
        gen.emit(f"add.s64 {a}, {tile}, {self.goff};")
        for i, regs in enumerate(out):
            pred = f"@{self.pv} " if (self.pv and i == self.iters - 1) else ""
            gen.emit(f"{pred}ld.global.nc.v4.f32 {{{', '.join(regs)}}}, [{a}+{i * self.gstep}];")
        return out

    def store(self, regs, hi, lo, shift=None):
        """Split and store the loaded tile; ``shift`` (a register, bytes) selects the buffer."""
        gen = self.gen
        step = (self.rstep * self.P // 4) * self.sbo
        bases = self.bases
        if shift is not None:
            bases = []
            for b in self.bases:
                r = gen.register(".u32")
                gen.emit(f"add.u32 {r}, {b}, {shift};")
                bases.append(r)
        for i, four in enumerate(regs):
            b = bases[i % self.P]
            imm = (i // self.P) * step
            his, los = tf32_split_pairs(gen, four)
            pred = f"@{self.pv} " if (self.pv and i == self.iters - 1) else ""
            gen.emit(f"{pred}st.shared.v4.b32 [{b}+{imm + hi}], {{{', '.join(his)}}};")
            gen.emit(f"{pred}st.shared.v4.b32 [{b}+{imm + lo}], {{{', '.join(los)}}};")


def _item_loop(gen, cta, ncta, nitems, hint):
    """Open a grid-stride loop over work items; returns (item register, close callback)."""
    item = gen.register(".u32")
    gen.emit(f"mov.u32 {item}, {cta};")
    top, done = gen.new_label(hint), gen.new_label(hint + "done")
    p = gen.register(".pred")
    gen.label(top)
    gen.emit(f"setp.ge.u32 {p}, {item}, {nitems};")
    gen.emit(f"@{p} bra.uni {done};")

    def close():
        gen.emit(f"add.u32 {item}, {item}, {ncta};")
        gen.emit(f"bra.uni {top};")
        gen.label(done)
    return item, close


def _counted_loop(gen, count, hint):
    """Open ``for j in range(count)`` (count a Python int); returns (j register, close)."""
    j = gen.register(".u32")
    gen.emit(f"mov.u32 {j}, 0;")
    top, done = gen.new_label(hint), gen.new_label(hint + "done")
    p = gen.register(".pred")
    gen.label(top)
    gen.emit(f"setp.ge.u32 {p}, {j}, {count};")
    gen.emit(f"@{p} bra.uni {done};")

    def close():
        gen.emit(f"add.u32 {j}, {j}, 1;")
        gen.emit(f"bra.uni {top};")
        gen.label(done)
    return j, close


def _parity(gen, counter, shift=0, minus=0):
    """((counter >> shift) - minus) & 1 in a fresh register."""
    r = gen.register(".u32")
    src = counter
    if shift:
        gen.emit(f"shr.u32 {r}, {src}, {shift};")
        src = r
    if minus:
        gen.emit(f"sub.u32 {r}, {src}, {minus};")
        src = r
    gen.emit(f"and.b32 {r}, {src}, 1;")
    return r


def _tree3(gen, op, regs):
    """Reduction of ``regs`` with the three-input f32 ``min``/``max`` (``op`` is
    ``max.f32`` or ``min.f32``): about half the instructions of a pairwise tree."""
    level = list(regs)
    while len(level) > 1:
        nxt = []
        i = 0
        while i < len(level):
            chunk = level[i:i + 3]
            if len(chunk) == 1:
                nxt.append(chunk[0])
            else:
                t = gen.register(".f32")
                gen.emit(f"{op} {t}, {', '.join(chunk)};")
                nxt.append(t)
            i += 3
        level = nxt
    return level[0]


def _sum_pairs(gen, regs):
    """Sum of an even number of f32 registers: a pairwise tree over packed pairs
    (``add.rn.f32x2``), then one add of the two lanes."""
    level = [pack2(gen, a, b) for a, b in zip(regs[0::2], regs[1::2])]
    while len(level) > 1:
        nxt = []
        for a, b in zip(level[0::2], level[1::2]):
            t = gen.register(".b64")
            gen.emit(f"add.rn.f32x2 {t}, {a}, {b};")
            nxt.append(t)
        if len(level) % 2:
            nxt.append(level[-1])
        level = nxt
    x, y = unpack2(gen, level[0])
    t = gen.register(".f32")
    gen.emit(f"add.rn.f32 {t}, {x}, {y};")
    return t


def _tree(gen, op, regs):
    """Pairwise reduction of ``regs`` with the binary f32 instruction ``op``."""
    level = list(regs)
    while len(level) > 1:
        nxt = []
        for a, b in zip(level[0::2], level[1::2]):
            t = gen.register(".f32")
            gen.emit(f"{op} {t}, {a}, {b};")
            nxt.append(t)
        if len(level) % 2:
            nxt.append(level[-1])
        level = nxt
    return level[0]


def _block_before(gen, J, k):
    """J - k in a fresh register (a block index k blocks back)."""
    r = gen.register(".u32")
    gen.emit(f"sub.u32 {r}, {J}, {k};")
    return r


def _wait_pair(wait, gen, B, first, block, **kw):
    """Wait until barrier pair ``first`` has completed the phase of block ``block``."""
    wait(_pair_barrier(gen, B, first, block), _parity(gen, block, shift=1), **kw)


def _pair_barrier(gen, B, first, counter):
    """Address of barrier ``first`` + (counter & 1) (the two barriers are adjacent)."""
    r = gen.register(".u32")
    gen.emit(f"and.b32 {r}, {counter}, 1;")
    gen.emit(f"mad.lo.u32 {r}, {r}, 8, {B['_base']};")
    gen.emit(f"add.u32 {r}, {r}, {8 * B['_index'][first]};")
    return r


def lower_attention(gen, kernel, plan):
    D = plan.D
    BKV = BKV_FOR_D[D]
    c = dict(D=D, BKV=BKV, NB=plan.Skv // BKV, NQB=plan.Sq // TQ, Sq=plan.Sq, Skv=plan.Skv)
    c["NITEMS"] = plan.G * c["NQB"]
    # tensor memory columns: Q_hi, Q_lo, two S buffers, the O accumulator
    c.update(QHI=0, QLO=D, S0=2 * D, O=2 * D + 2 * BKV)
    TMEM_COLS = 512
    # P in tensor memory when it fits (D = 64: Q 128 + S 128 + O 64 + P hi/lo 128 columns;
    # D = 128 with 32-key blocks: 256 + 64 + 128 + 64): the softmax writes it with tcgen05.st
    # and P*V reads A from TMEM; otherwise (D = 96) P goes through shared memory in the
    # K-major SWIZZLE_128B layout
    c["P_TMEM"] = _p_in_tmem(D, BKV)
    c.update(PTHI=3 * D + 2 * BKV, PTLO=3 * D + 3 * BKV)
    # dynamic shared memory (1024-aligned): NBUF x (kt hi, kt lo), NBUF x (v hi, v lo), P hi/lo
    NBUF = tile_buffers(D, int(kernel.launch.get("smem_bytes", 0) or 0))
    # one buffer per tile: split each product around the lo pass (see the barriers below)
    c["SPLIT"] = NBUF == 1
    K_BYTES, V_BYTES, P_BYTES = D * BKV * 4, BKV * D * 4, TQ * BKV * 4
    VBASE = NBUF * 2 * K_BYTES
    PBASE = VBASE + NBUF * 2 * V_BYTES
    c.update(NBUF=NBUF, KHI=0, KLO=K_BYTES, KSTEP=2 * K_BYTES, VHI=VBASE, VLO=VBASE + V_BYTES,
             VSTEP=2 * V_BYTES, PHI=PBASE, PLO=PBASE + P_BYTES)
    NEED = c["PHI"] if c["P_TMEM"] else c["PLO"] + P_BYTES
    # kt [K = D rows, N = keys] and v [K = keys, N = D] tiles, MN-major SWIZZLE_128B_BASE32B:
    # each 32-wide column strip is a contiguous run of 128-byte rows (4-row groups 512 B apart,
    # strips rows x 128 B apart)
    c.update(SBO_K=512, LBO_K=D * 128, SBO_V=512, LBO_V=BKV * 128)
    gen.maxntid = THREADS

    gen.module_decl(".global .align 4 .u32 emmy_error;")
    gen.module_decl(".extern .shared .align 1024 .b8 emmy_dsmem[];")
    # Barrier pairs are indexed by the block's parity, their phase by (block >> 1) & 1.
    # Every wait costs the MMA warp (which sets the pace when the tiles come by TMA) well over
    # a hundred cycles even when the phase has long completed, so each product waits on one
    # barrier that gathers all it needs:
    # SGO[b]: S of the next block using TMEM S buffer b may start (its kt tile is stored, 96
    #         loader arrivals, and the softmax has read the buffer's previous S, 128 arrivals);
    # SFULL[b]: that S has completed (tcgen05.commit) -- also frees its kt tile for the loader;
    # PVGO[b]: P*V of the block may start (P written, 128 softmax arrivals; its v tile stored,
    #          96 loader arrivals -- the loader may be a block ahead with two tile buffers);
    # PVDONE[b]: P*V of the block has completed -- frees P and its v tile, and O may be read
    #            or rescaled.
    # On the TMA path the producer lane arrives for its warp once it has issued a tile's copy,
    # and KRAW[b] / VRAW[b] complete when the raw kt / v tile has landed (expect_tx); the
    # workers arrive on SGO / PVGO once the lo tile is written. With one buffer per tile
    # (D = 96) the copies are on the critical path: the producer then arrives for all 96 on
    # SGO / PVGO, the MMA warp issues the products that read only the raw tile (hi x hi,
    # lo x hi) after KRAW / VRAW and the hi x lo products after KLO[b] / VLO[b] (64 worker
    # arrivals once the lo tile is written).
    names = ["SGO0", "SGO1", "SFULL0", "SFULL1", "PVGO0", "PVGO1", "PVDONE0", "PVDONE1",
             "QREADY", "DRAIN", "KRAW0", "KRAW1", "VRAW0", "VRAW1", "KLO0", "KLO1", "VLO0",
             "VLO1"]
    gen.shared("emmy_bar", ".b64", length=len(names), align=8)
    gen.shared("emmy_tmem_slot", ".b32", length=1, align=4)

    # tensor maps of kt [G, D, Skv] and v [G, Skv, D] (innermost first), boxes of 32
    # columns: one box fills one column strip of a tile buffer
    tmap.declare(gen, [
        tmap.record(kernel.arg_order.index(plan.kt), [plan.Skv, D, plan.G],
                    [plan.Skv * 4, D * plan.Skv * 4], [32, D, 1]),
        tmap.record(kernel.arg_order.index(plan.v), [D, plan.Skv, plan.G],
                    [D * 4, plan.Skv * D * 4], [32, BKV, 1]),
    ])

    ptr, raw_ptr = {}, {}
    for name in kernel.arg_order:
        raw, g = gen.register(".u64"), gen.register(".u64")
        gen.emit(f"ld.param.u64 {raw}, [{gen.parameter(name)}];")
        gen.emit(f"cvta.to.global.u64 {g}, {raw};")
        ptr[name], raw_ptr[name] = g, raw

    tid, warp, lane = (gen.register(".u32") for _ in range(3))
    gen.emit(f"mov.u32 {tid}, %tid.x;")
    gen.emit(f"shr.u32 {warp}, {tid}, 5;")
    gen.emit(f"and.b32 {lane}, {tid}, 31;")
    base = gen.register(".u32")
    gen.emit(f"mov.u32 {base}, emmy_dsmem;")
    gen.emit(f"add.u32 {base}, {base}, 1023;")
    gen.emit(f"and.b32 {base}, {base}, -1024;")
    dsz, used = gen.register(".u32"), gen.register(".u32")
    gen.emit(f"mov.u32 {dsz}, %dynamic_smem_size;")
    gen.emit(f"mov.u32 {used}, emmy_dsmem;")
    gen.emit(f"sub.u32 {used}, {base}, {used};")
    gen.emit(f"add.u32 {used}, {used}, {NEED};")
    p_small = gen.register(".pred")
    gen.emit(f"setp.gt.u32 {p_small}, {used}, {dsz};")
    L_fit = gen.new_label("fits")
    gen.emit(f"@!{p_small} bra {L_fit};")
    gen.emit("red.global.or.b32 [emmy_error], 4;")
    gen.emit("ret;")
    gen.label(L_fit)

    bar = gen.register(".u32")
    gen.emit(f"mov.u32 {bar}, emmy_bar;")
    B = {n: f"{bar}+{8 * i}" for i, n in enumerate(names)}
    B["_base"] = bar
    B["_index"] = {n: i for i, n in enumerate(names)}

    p_t0 = gen.register(".pred")
    gen.emit(f"setp.eq.u32 {p_t0}, {tid}, 0;")
    L_noinit = gen.new_label("noinit")
    gen.emit(f"@!{p_t0} bra {L_noinit};")
    counts = {"SGO0": NLOAD + 128, "SGO1": NLOAD + 128, "PVGO0": NLOAD + 128,
              "PVGO1": NLOAD + 128, "QREADY": 128, "KLO0": NWORK, "KLO1": NWORK,
              "VLO0": NWORK, "VLO1": NWORK}
    for n in names:
        gen.emit(f"mbarrier.init.shared::cta.b64 [{B[n]}], {counts.get(n, 1)};")
    gen.emit("fence.mbarrier_init.release.cluster;")
    gen.label(L_noinit)

    p_mw = gen.register(".pred")
    gen.emit(f"setp.eq.u32 {p_mw}, {warp}, 4;")
    L_noalloc = gen.new_label("noalloc")
    gen.emit(f"@!{p_mw} bra {L_noalloc};")
    slot = gen.register(".u32")
    gen.emit(f"mov.u32 {slot}, emmy_tmem_slot;")
    gen.emit(f"tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [{slot}], {TMEM_COLS};")
    gen.emit("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;")
    gen.emit("tcgen05.fence::before_thread_sync;")
    gen.label(L_noalloc)
    gen.emit("bar.sync 0;")
    gen.emit("tcgen05.fence::after_thread_sync;")
    tmem = gen.register(".u32")
    gen.emit(f"ld.shared.b32 {tmem}, [emmy_tmem_slot];")
    cta, ncta = gen.register(".u32"), gen.register(".u32")
    gen.emit(f"mov.u32 {cta}, %ctaid.x;")
    gen.emit(f"mov.u32 {ncta}, %nctaid.x;")

    # the TMA path when the runtime has written maps for exactly these kt and v pointers
    p_tma = tmap.keys_match(gen, [raw_ptr[plan.kt], raw_ptr[plan.v]])
    L_exit = gen.new_label("exit")
    wait = _Wait(gen, L_exit)
    L_mma, L_load = gen.new_label("mma_role"), gen.new_label("load_role")
    gen.emit(f"@{p_mw} bra {L_mma};")
    p_ld = gen.register(".pred")
    gen.emit(f"setp.ge.u32 {p_ld}, {warp}, 5;")
    gen.emit(f"@{p_ld} bra {L_load};")

    _softmax_role(gen, ptr, plan, tid, warp, tmem, base, B, wait, cta, ncta, c)
    gen.emit(f"bra {L_exit};")
    gen.label(L_mma)
    _mma_role(gen, tmem, base, B, wait, cta, ncta, lane, c, p_tma)
    gen.emit(f"bra {L_exit};")
    gen.label(L_load)
    _load_role(gen, ptr, p_tma, plan, tid, base, B, wait, cta, ncta, c)

    gen.label(L_exit)
    L_nodrain = gen.new_label("nodrain")
    gen.emit(f"@!{p_mw} bra {L_nodrain};")
    p_el2, el2 = gen.register(".pred"), gen.register(".u32")
    gen.emit(f"elect.sync {el2}|{p_el2}, -1;")
    gen.emit(f"@{p_el2} tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 "
             f"[{B['DRAIN']}];")
    wait(B["DRAIN"], 0, exit_label=None)
    gen.label(L_nodrain)
    gen.emit("tcgen05.fence::before_thread_sync;")
    gen.emit("barrier.sync 0;")
    gen.emit("tcgen05.fence::after_thread_sync;")
    L_nodealloc = gen.new_label("nodealloc")
    gen.emit(f"@!{p_mw} bra {L_nodealloc};")
    gen.emit("bar.warp.sync -1;")
    gen.emit(f"tcgen05.dealloc.cta_group::1.sync.aligned.b32 {tmem}, {TMEM_COLS};")
    gen.label(L_nodealloc)
    gen.emit("ret;")


# ------------------------------------------------------------------ softmax warps 0-3

def _softmax_role(gen, ptr, plan, tid, warp, tmem, base, B, wait, cta, ncta, c):
    BKV = c["BKV"]
    D, NB, NQB = c["D"], c["NB"], c["NQB"]
    lane_field = gen.register(".u32")
    gen.emit(f"shl.b32 {lane_field}, {warp}, 21;")
    trow = gen.register(".u32")
    gen.emit(f"add.u32 {trow}, {tmem}, {lane_field};")
    # the IR scales the scores by reciprocal(c); log2(e) is folded in for ex2
    cval = gen.register(".f32")
    gen.emit(f"ld.global.f32 {cval}, [{ptr[plan.scale_buf]}];")
    scale = gen.register(".f32")
    gen.emit(f"rcp.rn.f32 {scale}, {cval};")
    gen.emit(f"mul.rn.f32 {scale}, {scale}, 0f3FB8AA3B;")
    p_neg = gen.register(".pred")
    gen.emit(f"setp.lt.f32 {p_neg}, {scale}, 0f00000000;")
    scale2 = pack2(gen, scale, scale)
    # P row base addresses for the 8 swizzle phases: row*128 + ((k/4 % 8) ^ row % 8) * 16
    r8, prow = gen.register(".u32"), gen.register(".u32")
    gen.emit(f"and.b32 {r8}, {tid}, 7;")
    gen.emit(f"shl.b32 {prow}, {tid}, 7;")
    gen.emit(f"add.u32 {prow}, {prow}, {base};")
    pofs = []
    for k in range(8):
        t = gen.register(".u32")
        gen.emit(f"xor.b32 {t}, {r8}, {k};")
        gen.emit(f"mad.lo.u32 {t}, {t}, 16, {prow};")
        pofs.append(t)

    def row_of(item):
        g, qb, grow = (gen.register(".u32") for _ in range(3))
        gen.emit(f"div.u32 {g}, {item}, {NQB};")
        gen.emit(f"rem.u32 {qb}, {item}, {NQB};")
        gen.emit(f"mad.lo.u32 {grow}, {g}, {c['Sq']}, {tid};")
        gen.emit(f"mad.lo.u32 {grow}, {qb}, {TQ}, {grow};")
        off = gen.register(".u64")
        gen.emit(f"mul.wide.u32 {off}, {grow}, {D * 4};")
        return off

    def q_load(item):
        a = gen.register(".u64")
        gen.emit(f"add.s64 {a}, {ptr[plan.q]}, {row_of(item)};")
        regs = []
        for v4 in range(D // 4):
            r = gen.registers(".f32", 4)
            gen.emit(f"ld.global.nc.v4.f32 {{{', '.join(r)}}}, [{a}+{v4 * 16}];")
            regs += r
        return regs

    def q_store(regs):
        for cb in range(D // 32):
            his, los = tf32_split_pairs(gen, regs[cb * 32:cb * 32 + 32])
            gen.emit(f"tcgen05.st.sync.aligned.32x32b.x32.b32 [{trow}+{c['QHI'] + cb * 32}], "
                     f"{{{', '.join(his)}}};")
            gen.emit(f"tcgen05.st.sync.aligned.32x32b.x32.b32 [{trow}+{c['QLO'] + cb * 32}], "
                     f"{{{', '.join(los)}}};")
        gen.emit("tcgen05.wait::st.sync.aligned;")
        gen.emit("tcgen05.fence::before_thread_sync;")
        gen.emit(f"mbarrier.arrive.shared::cta.b64 _, [{B['QREADY']}];")

    J = gen.register(".u32")
    gen.emit(f"mov.u32 {J}, 0;")
    # neither TMEM S buffer holds an unread S yet: count those reads as done
    for b in ("SGO0", "SGO1"):
        gen.emit(f"mbarrier.arrive.shared::cta.b64 _, [{B[b]}];")
    # Q rows of the first work item
    p_any = gen.register(".pred")
    gen.emit(f"setp.lt.u32 {p_any}, {cta}, {c['NITEMS']};")
    L_noq = gen.new_label("noq")
    gen.emit(f"@!{p_any} bra.uni {L_noq};")
    q_store(q_load(cta))
    gen.label(L_noq)

    m_used, lsum, negm = gen.register(".f32"), gen.register(".f32"), gen.register(".f32")
    item, close_item = _item_loop(gen, cta, ncta, c["NITEMS"], "sitem")
    orow = gen.register(".u64")
    gen.emit(f"add.s64 {orow}, {ptr[plan.out]}, {row_of(item)};")
    gen.emit(f"mov.f32 {m_used}, 0fFF800000;")
    gen.emit(f"mov.f32 {lsum}, 0f00000000;")

    def block(first, last):
        """One key block. ``first``: True/False, or a predicate register true on block 0."""
        sfull = _pair_barrier(gen, B, "SFULL0", J)
        sphase = _parity(gen, J, shift=1)
        if last:
            # fetch the next item's Q rows while the last S product runs; once it has
            # landed, Q's tensor-memory columns are free. Load, wait and store share one
            # branch so the Q registers are live only inside it.
            nxt, p_has = gen.register(".u32"), gen.register(".pred")
            gen.emit(f"add.u32 {nxt}, {item}, {ncta};")
            gen.emit(f"setp.lt.u32 {p_has}, {nxt}, {c['NITEMS']};")
            L_plain, L_joined = gen.new_label("noqnext"), gen.new_label("qjoined")
            gen.emit(f"@!{p_has} bra.uni {L_plain};")
            qnext = q_load(nxt)
            wait(sfull, sphase)
            gen.emit("tcgen05.fence::after_thread_sync;")
            q_store(qnext)
            gen.emit(f"bra.uni {L_joined};")
            gen.label(L_plain)
            wait(sfull, sphase)
            gen.emit("tcgen05.fence::after_thread_sync;")
            gen.label(L_joined)
        else:
            wait(sfull, sphase)
            gen.emit("tcgen05.fence::after_thread_sync;")
        scol = gen.register(".u32")
        gen.emit(f"and.b32 {scol}, {J}, 1;")
        gen.emit(f"mad.lo.u32 {scol}, {scol}, {BKV}, {trow};")
        s = []
        for cb in range(BKV // 32):
            regs = gen.registers(".f32", 32)
            gen.emit(f"tcgen05.ld.sync.aligned.32x32b.x32.b32 {{{', '.join(regs)}}}, "
                     f"[{scol}+{c['S0'] + cb * 32}];")
            s += regs
        gen.emit("tcgen05.wait::ld.sync.aligned;")
        gen.emit("tcgen05.fence::before_thread_sync;")
        gen.emit(f"mbarrier.arrive.shared::cta.b64 _, [{_pair_barrier(gen, B, 'SGO0', J)}];")
        # block maximum of the scaled scores (scale < 0 flips max and min)
        mx = gen.register(".f32")
        L_min, L_mx = gen.new_label("smin"), gen.new_label("smx")
        gen.emit(f"@{p_neg} bra.uni {L_min};")
        gen.emit(f"mov.f32 {mx}, {_tree3(gen, 'max.f32', s)};")
        gen.emit(f"bra.uni {L_mx};")
        gen.label(L_min)
        gen.emit(f"mov.f32 {mx}, {_tree3(gen, 'min.f32', s)};")
        gen.label(L_mx)
        gen.emit(f"mul.rn.f32 {mx}, {mx}, {scale};")
        thr, need, anyneed = gen.register(".f32"), gen.register(".pred"), gen.register(".pred")
        gen.emit(f"add.rn.f32 {thr}, {m_used}, {RESCALE_BITS};")
        gen.emit(f"setp.gt.f32 {need}, {mx}, {thr};")
        gen.emit(f"vote.sync.any.pred {anyneed}, {need}, -1;")
        L_keep = gen.new_label("keepmax")
        gen.emit(f"@!{anyneed} bra.uni {L_keep};")
        m_new, alpha = gen.register(".f32"), gen.register(".f32")
        gen.emit(f"selp.f32 {m_new}, {mx}, {m_used}, {need};")
        gen.emit(f"sub.rn.f32 {alpha}, {m_used}, {m_new};")
        gen.emit(f"ex2.approx.ftz.f32 {alpha}, {alpha};")
        gen.emit(f"mul.rn.f32 {lsum}, {lsum}, {alpha};")
        gen.emit(f"mov.f32 {m_used}, {m_new};")
        if first is not True:
            # rescale this warp's O rows once P*V of the previous block is done
            L_norescale = gen.new_label("noresc")
            if first is not False:
                gen.emit(f"@{first} bra.uni {L_norescale};")
            _wait_pair(wait, gen, B, "PVDONE0", _block_before(gen, J, 1))
            gen.emit("tcgen05.fence::after_thread_sync;")
            for cb in range(D // 16):
                regs = gen.registers(".f32", 16)
                col = c["O"] + cb * 16
                gen.emit(f"tcgen05.ld.sync.aligned.32x32b.x16.b32 {{{', '.join(regs)}}}, "
                         f"[{trow}+{col}];")
                gen.emit("tcgen05.wait::ld.sync.aligned;")
                for r in regs:
                    gen.emit(f"mul.rn.f32 {r}, {r}, {alpha};")
                gen.emit(f"tcgen05.st.sync.aligned.32x32b.x16.b32 [{trow}+{col}], "
                         f"{{{', '.join(regs)}}};")
            gen.emit("tcgen05.wait::st.sync.aligned;")
            gen.label(L_norescale)
        gen.label(L_keep)
        # p = 2^(s * scale - m), row sum
        gen.emit(f"neg.f32 {negm}, {m_used};")
        # ex2 without subnormal handling: arguments are at most 8 (the lazy maximum), and a
        # score below 2^-126 of the row's maximum weighs nothing next to it
        # two scores per fma.rn.f32x2 (each lane rounded as fma.rn.f32 would)
        negm2 = pack2(gen, negm, negm)
        p = []
        for x, y in zip(s[0::2], s[1::2]):
            t2 = gen.register(".b64")
            gen.emit(f"fma.rn.f32x2 {t2}, {pack2(gen, x, y)}, {scale2}, {negm2};")
            for t in unpack2(gen, t2):
                gen.emit(f"ex2.approx.ftz.f32 {t}, {t};")
                p.append(t)
        gen.emit(f"add.rn.f32 {lsum}, {lsum}, {_sum_pairs(gen, p)};")
        # P -> shared memory once P*V of the previous block has released it
        L_nopw = gen.new_label("nopw")
        pz = gen.register(".pred")
        gen.emit(f"setp.eq.u32 {pz}, {J}, 0;")
        gen.emit(f"@{pz} bra.uni {L_nopw};")
        _wait_pair(wait, gen, B, "PVDONE0", _block_before(gen, J, 1))
        gen.label(L_nopw)
        if c["P_TMEM"]:
            for cb in range(BKV // 32):
                his, los = tf32_split_pairs(gen, p[cb * 32:cb * 32 + 32])
                for col, regs in ((c["PTHI"], his), (c["PTLO"], los)):
                    gen.emit(f"tcgen05.st.sync.aligned.32x32b.x32.b32 [{trow}+{col + cb * 32}], "
                             f"{{{', '.join(regs)}}};")
            gen.emit("tcgen05.wait::st.sync.aligned;")
        else:
            for k4 in range(BKV // 4):
                halves = tf32_split_pairs(gen, p[4 * k4:4 * k4 + 4])
                atom = (4 * k4) // 32
                for nm, regs in zip(("PHI", "PLO"), halves):
                    gen.emit(f"st.shared.v4.b32 [{pofs[k4 % 8]}+{c[nm] + atom * TQ * 128}], "
                             f"{{{', '.join(regs)}}};")
            gen.emit("fence.proxy.async.shared::cta;")
        gen.emit("tcgen05.fence::before_thread_sync;")
        gen.emit(f"mbarrier.arrive.shared::cta.b64 _, [{_pair_barrier(gen, B, 'PVGO0', J)}];")
        gen.emit(f"add.u32 {J}, {J}, 1;")

    if NB > 1:
        j, close_j = _counted_loop(gen, NB - 1, "sblk")
        pfirst = gen.register(".pred")
        gen.emit(f"setp.eq.u32 {pfirst}, {j}, 0;")
        block(pfirst, False)
        close_j()
    block(NB == 1, True)
    # epilogue: O / l once the last P*V has landed
    _wait_pair(wait, gen, B, "PVDONE0", _block_before(gen, J, 1))
    gen.emit("tcgen05.fence::after_thread_sync;")
    inv = gen.register(".f32")
    gen.emit(f"rcp.rn.f32 {inv}, {lsum};")
    for cb in range(D // 32):
        regs = gen.registers(".f32", 32)
        gen.emit(f"tcgen05.ld.sync.aligned.32x32b.x32.b32 {{{', '.join(regs)}}}, "
                 f"[{trow}+{c['O'] + cb * 32}];")
        gen.emit("tcgen05.wait::ld.sync.aligned;")
        for r in regs:
            gen.emit(f"mul.rn.f32 {r}, {r}, {inv};")
        for v4 in range(8):
            gen.emit(f"st.global.v4.f32 [{orow}+{(cb * 32 + v4 * 4) * 4}], "
                     f"{{{', '.join(regs[v4 * 4:v4 * 4 + 4])}}};")
    close_item()


# ------------------------------------------------------------------ MMA warp 4

def _mma_role(gen, tmem, base, B, wait, cta, ncta, lane, c, p_tma):
    BKV = c["BKV"]
    D, NB = c["D"], c["NB"]
    p_el, el = gen.register(".pred"), gen.register(".u32")
    gen.emit(f"elect.sync {el}|{p_el}, -1;")
    p_true, p_false = gen.register(".pred"), gen.register(".pred")
    gen.emit(f"setp.eq.u32 {p_true}, {lane}, {lane};")
    gen.emit(f"setp.ne.u32 {p_false}, {lane}, {lane};")
    # instruction descriptors: f32 accumulate, TF32 A and B, B MN-major, M = 128
    common = (1 << 4) | (2 << 7) | (2 << 10) | (1 << 16) | ((TQ >> 4) << 24)
    r_is, r_io = gen.register(".u32"), gen.register(".u32")
    gen.emit(f"mov.u32 {r_is}, {common | ((BKV >> 3) << 17)};")
    gen.emit(f"mov.u32 {r_io}, {common | ((D >> 3) << 17)};")
    # shared-memory descriptor high words: SBO, version 1, layout
    hi_k, hi_v, hi_p = (gen.register(".u32") for _ in range(3))
    gen.emit(f"mov.u32 {hi_k}, {(c['SBO_K'] >> 4) | (1 << 14) | (1 << 29)};")
    gen.emit(f"mov.u32 {hi_v}, {(c['SBO_V'] >> 4) | (1 << 14) | (1 << 29)};")
    lbo_k, lbo_v = (c["LBO_K"] >> 4) << 16, (c["LBO_V"] >> 4) << 16

    def tile_shift(block, step):
        """Shared-memory descriptor offset (16-byte units) of block ``block``'s tile buffer."""
        if c["NBUF"] == 1:
            return None
        r = gen.register(".u32")
        gen.emit(f"and.b32 {r}, {block}, 1;")
        gen.emit(f"mul.lo.u32 {r}, {r}, {step >> 4};")
        return r
    gen.emit(f"mov.u32 {hi_p}, {(1024 >> 4) | (1 << 14) | (2 << 29)};")
    sb4 = gen.register(".u32")
    gen.emit(f"shr.u32 {sb4}, {base}, 4;")

    def desc(lo_const, hi_reg, shift=None):
        lo = gen.register(".u32")
        gen.emit(f"add.u32 {lo}, {sb4}, {lo_const};")
        if shift is not None:
            gen.emit(f"add.u32 {lo}, {lo}, {shift};")
        d = gen.register(".b64")
        gen.emit(f"mov.b64 {d}, {{{lo}, {hi_reg}}};")
        return d

    def commit(bar_addr):
        gen.emit(f"@{p_el} tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 "
                 f"[{bar_addr}];")

    def tma_wait(first, block):
        """On the TMA path only: wait for barrier pair ``first`` of block ``block``."""
        L = gen.new_label("notma")
        gen.emit(f"@!{p_tma} bra.uni {L};")
        _wait_pair(wait, gen, B, first, block)
        gen.emit("tcgen05.fence::after_thread_sync;")
        gen.label(L)

    J, icount = gen.register(".u32"), gen.register(".u32")
    gen.emit(f"mov.u32 {J}, 0;")
    gen.emit(f"mov.u32 {icount}, 0;")

    def issue_s():
        wait(_pair_barrier(gen, B, "SGO0", J), _parity(gen, J, shift=1))
        gen.emit("tcgen05.fence::after_thread_sync;")
        dcol = gen.register(".u32")
        gen.emit(f"and.b32 {dcol}, {J}, 1;")
        gen.emit(f"mad.lo.u32 {dcol}, {dcol}, {BKV}, {tmem};")
        gen.emit(f"add.u32 {dcol}, {dcol}, {c['S0']};")
        kshift = tile_shift(J, c["KSTEP"])
        if c["SPLIT"]:
            tma_wait("KRAW0", J)
        lo_products = []
        for ks in range(D // 8):
            a_hi, a_lo = gen.register(".u32"), gen.register(".u32")
            gen.emit(f"add.u32 {a_hi}, {tmem}, {c['QHI'] + ks * 8};")
            gen.emit(f"add.u32 {a_lo}, {tmem}, {c['QLO'] + ks * 8};")
            kadv = (2 * c["SBO_K"] * ks) >> 4
            b_hi = desc(((c["KHI"] >> 4) + kadv) | lbo_k, hi_k, kshift)
            b_lo = desc(((c["KLO"] >> 4) + kadv) | lbo_k, hi_k, kshift)
            acc = p_false if ks == 0 else p_true
            for a, b, en in ((a_hi, b_hi, acc), (a_lo, b_hi, p_true)):
                gen.emit(f"@{p_el} tcgen05.mma.cta_group::1.kind::tf32 [{dcol}], [{a}], {b}, "
                         f"{r_is}, {en};")
            lo_products.append((a_hi, b_lo))
        if c["SPLIT"]:
            tma_wait("KLO0", J)
        for a, b in lo_products:
            gen.emit(f"@{p_el} tcgen05.mma.cta_group::1.kind::tf32 [{dcol}], [{a}], {b}, "
                     f"{r_is}, {p_true};")
        commit(_pair_barrier(gen, B, "SFULL0", J))

    def issue_pv(Jp, first):
        """O (+)= P_Jp V_Jp; ``first``: True/False or a predicate true on an item's block 0."""
        _wait_pair(wait, gen, B, "PVGO0", Jp)
        gen.emit("tcgen05.fence::after_thread_sync;")
        vshift = tile_shift(Jp, c["VSTEP"])
        if first is True:
            acc0 = p_false
        elif first is False:
            acc0 = p_true
        else:
            acc0 = gen.register(".pred")
            gen.emit(f"not.pred {acc0}, {first};")
        dcol = gen.register(".u32")
        gen.emit(f"add.u32 {dcol}, {tmem}, {c['O']};")
        if c["SPLIT"]:
            tma_wait("VRAW0", Jp)
        lo_products = []
        for ks in range(BKV // 8):
            if c["P_TMEM"]:                  # A = P from tensor memory, 8 columns per step
                a_hi, a_lo = gen.register(".u32"), gen.register(".u32")
                gen.emit(f"add.u32 {a_hi}, {tmem}, {c['PTHI'] + ks * 8};")
                gen.emit(f"add.u32 {a_lo}, {tmem}, {c['PTLO'] + ks * 8};")
                a_hi, a_lo = f"[{a_hi}]", f"[{a_lo}]"
            else:
                patom, pin = (ks * 8) // 32, ((ks * 8) % 32) * 4
                a_hi = desc(((c["PHI"] + patom * TQ * 128 + pin) >> 4) | (1 << 16), hi_p)
                a_lo = desc(((c["PLO"] + patom * TQ * 128 + pin) >> 4) | (1 << 16), hi_p)
            vadv = (2 * c["SBO_V"] * ks) >> 4
            b_hi = desc(((c["VHI"] >> 4) + vadv) | lbo_v, hi_v, vshift)
            b_lo = desc(((c["VLO"] >> 4) + vadv) | lbo_v, hi_v, vshift)
            acc = acc0 if ks == 0 else p_true
            for a, b, en in ((a_hi, b_hi, acc), (a_lo, b_hi, p_true)):
                gen.emit(f"@{p_el} tcgen05.mma.cta_group::1.kind::tf32 [{dcol}], {a}, {b}, "
                         f"{r_io}, {en};")
            lo_products.append((a_hi, b_lo))
        if c["SPLIT"]:
            tma_wait("VLO0", Jp)
        for a, b in lo_products:
            gen.emit(f"@{p_el} tcgen05.mma.cta_group::1.kind::tf32 [{dcol}], {a}, {b}, "
                     f"{r_io}, {p_true};")
        commit(_pair_barrier(gen, B, "PVDONE0", Jp))

    item, close_item = _item_loop(gen, cta, ncta, c["NITEMS"], "mitem")
    wait(B["QREADY"], _parity(gen, icount))
    gen.emit("tcgen05.fence::after_thread_sync;")
    j, close_j = _counted_loop(gen, NB, "mblk")
    issue_s()
    L_nopv = gen.new_label("nopv")
    pz, p1 = gen.register(".pred"), gen.register(".pred")
    gen.emit(f"setp.eq.u32 {pz}, {j}, 0;")
    gen.emit(f"@{pz} bra.uni {L_nopv};")
    gen.emit(f"setp.eq.u32 {p1}, {j}, 1;")
    Jm = gen.register(".u32")
    gen.emit(f"sub.u32 {Jm}, {J}, 1;")
    issue_pv(Jm, p1)
    gen.label(L_nopv)
    gen.emit(f"add.u32 {J}, {J}, 1;")
    close_j()
    Jl = gen.register(".u32")
    gen.emit(f"sub.u32 {Jl}, {J}, 1;")
    issue_pv(Jl, NB == 1)
    gen.emit(f"add.u32 {icount}, {icount}, 1;")
    close_item()


# ------------------------------------------------------------------ loader warps 5-7

def _load_role(gen, ptr, p_tma, plan, tid, base, B, wait, cta, ncta, c):
    """Warps 5-7: the TMA path when the runtime has written tensor maps for this launch's kt
    and v pointers, else the register-staged path. Bit 0 of ``emmy_path`` records a CTA on
    the TMA path, bit 1 one on the register path."""
    L_tma, L_done = gen.new_label("ld_tma"), gen.new_label("ld_done")
    gen.emit(f"@{p_tma} bra.uni {L_tma};")
    _load_lsu(gen, ptr, plan, tid, base, B, wait, cta, ncta, c)
    gen.emit(f"bra.uni {L_done};")
    gen.label(L_tma)
    _load_tma(gen, plan, tid, base, B, wait, cta, ncta, c)
    gen.label(L_done)


def _after(gen, wait, B, block, k, first, hint, **kw):
    """Wait for barrier pair ``first`` of block ``block - k`` unless block < k."""
    p = gen.register(".pred")
    gen.emit(f"setp.lt.u32 {p}, {block}, {k};")
    L = gen.new_label(hint)
    gen.emit(f"@{p} bra.uni {L};")
    _wait_pair(wait, gen, B, first, _block_before(gen, block, k), **kw)
    gen.label(L)


def _buf_shift(gen, c, block, step):
    """Byte offset of block ``block``'s tile buffer (None with one buffer)."""
    if c["NBUF"] == 1:
        return None
    r = gen.register(".u32")
    gen.emit(f"and.b32 {r}, {block}, 1;")
    gen.emit(f"mul.lo.u32 {r}, {r}, {step};")
    return r


def _load_lsu(gen, ptr, plan, tid, base, B, wait, cta, ncta, c):
    """kt and v tiles of each key block -> hi/lo MN-major tiles in shared memory.

    The tensor core runs S_j, PV_(j-1), S_(j+1), PV_j, ... The kt tile of block j + 1 is
    stored a block ahead of the v tile of block j. With NBUF tile buffers, the kt tile of block
    X goes to buffer X % NBUF once S_(X - NBUF) has released it, and the v tile of block X
    once PV_(X - NBUF) has: with two buffers a tile is stored while the tensor core still
    reads the other one. The global loads of each tile are issued a step before its buffer
    wait, so L2 latency overlaps the tensor-core work."""
    D, NB, NQB, BKV, NBUF = c["D"], c["NB"], c["NQB"], c["BKV"], c["NBUF"]
    lt = gen.register(".u32")
    gen.emit(f"sub.u32 {lt}, {tid}, 160;")
    p_l0 = gen.register(".pred")
    gen.emit(f"setp.eq.u32 {p_l0}, {lt}, 0;")
    gen.emit(f"@{p_l0} red.global.or.b32 [emmy_path], 2;")
    ktc = _TileCopy(gen, lt, rows=D, cols=BKV, row_stride=c["Skv"], sbo=c["SBO_K"], base=base,
                    lbo=c["LBO_K"])
    vc = _TileCopy(gen, lt, rows=BKV, cols=D, row_stride=D, sbo=c["SBO_V"], base=base,
                   lbo=c["LBO_V"])
    J = gen.register(".u32")
    gen.emit(f"mov.u32 {J}, 0;")
    item, close_item = _item_loop(gen, cta, ncta, c["NITEMS"], "litem")
    g = gen.register(".u32")
    gen.emit(f"div.u32 {g}, {item}, {NQB};")
    kt_t, v_t = gen.register(".u64"), gen.register(".u64")
    gen.emit(f"mul.wide.u32 {kt_t}, {g}, {D * c['Skv'] * 4};")
    gen.emit(f"add.s64 {v_t}, {ptr[plan.v]}, {kt_t};")
    gen.emit(f"add.s64 {kt_t}, {ptr[plan.kt]}, {kt_t};")
    kregs = ktc.load(kt_t)
    vregs = vc.load(v_t)

    def buf_shift(block, step):
        return _buf_shift(gen, c, block, step)

    def after(block, k, first, hint):
        _after(gen, wait, B, block, k, first, hint)

    def put_k(block):
        """kt tile (in kregs) of global block ``block`` -> its buffer, once S of the block
        NBUF earlier has released it; counts toward SGO."""
        after(block, NBUF, "SFULL0", "kfree")
        ktc.store(kregs, c["KHI"], c["KLO"], buf_shift(block, c["KSTEP"]))
        gen.emit("fence.proxy.async.shared::cta;")
        gen.emit(f"mbarrier.arrive.shared::cta.b64 _, [{_pair_barrier(gen, B, 'SGO0', block)}];")

    put_k(J)                                        # kt of this item's first block
    if NB > 1:
        gen.emit(f"add.s64 {kt_t}, {kt_t}, {BKV * 4};")
        ktc.load(kt_t, into=kregs)
    j, close_j = _counted_loop(gen, NB, "lblk")
    # kt of block J + 1
    pk = gen.register(".pred")
    gen.emit(f"setp.lt.u32 {pk}, {j}, {NB - 1};")
    L_nok = gen.new_label("nonextk")
    gen.emit(f"@!{pk} bra.uni {L_nok};")
    jn = gen.register(".u32")
    gen.emit(f"add.u32 {jn}, {J}, 1;")
    put_k(jn)
    pk2 = gen.register(".pred")
    gen.emit(f"setp.lt.u32 {pk2}, {j}, {NB - 2};")
    L_nok2 = gen.new_label("nok2")
    gen.emit(f"@!{pk2} bra.uni {L_nok2};")
    gen.emit(f"add.s64 {kt_t}, {kt_t}, {BKV * 4};")
    ktc.load(kt_t, into=kregs)
    gen.label(L_nok2)
    gen.label(L_nok)
    # v of block J, once P*V of the block NBUF earlier has released its buffer
    after(J, NBUF, "PVDONE0", "vfree")
    vc.store(vregs, c["VHI"], c["VLO"], buf_shift(J, c["VSTEP"]))
    gen.emit("fence.proxy.async.shared::cta;")
    gen.emit(f"mbarrier.arrive.shared::cta.b64 _, [{_pair_barrier(gen, B, 'PVGO0', J)}];")
    L_nov = gen.new_label("nonextv")
    gen.emit(f"@!{pk} bra.uni {L_nov};")
    gen.emit(f"add.s64 {v_t}, {v_t}, {BKV * D * 4};")
    vc.load(v_t, into=vregs)
    gen.label(L_nov)
    gen.emit(f"add.u32 {J}, {J}, 1;")
    close_j()
    close_item()


def _lo_pass(gen, wt, base, shift, src, dst, nbytes):
    """Workers (64 threads): the lo part ``x - (x & 0xFFFFE000)`` of every f32 of the raw tile
    at ``src`` into the same offsets at ``dst``. The raw tile stays in place as the hi operand:
    a ``kind::tf32`` MMA reads only the top 19 bits of each f32 word, so the raw word and its
    masked hi part give the same products. Thread ``wt`` owns the 16-byte chunks wt, wt + 64,
    ...: each warp instruction covers 512 contiguous bytes (no bank conflicts), and the lo
    tile has the hi tile's swizzled layout because the offsets are the same."""
    cpt = nbytes // 16 // 64
    assert cpt * 16 * 64 == nbytes
    a = gen.register(".u32")
    gen.emit(f"mad.lo.u32 {a}, {wt}, 16, {base};")
    if shift is not None:
        gen.emit(f"add.u32 {a}, {a}, {shift};")
    for g0 in range(0, cpt, 8):
        group = []
        for i in range(g0, min(cpt, g0 + 8)):
            regs = gen.registers(".b32", 4)
            gen.emit(f"ld.shared.v4.b32 {{{', '.join(regs)}}}, [{a}+{src + i * 1024}];")
            group.append((i, regs))
        for i, regs in group:
            _, los = tf32_split_pairs(gen, regs)
            gen.emit(f"st.shared.v4.b32 [{a}+{dst + i * 1024}], {{{', '.join(los)}}};")


def _load_tma(gen, plan, tid, base, B, wait, cta, ncta, c):
    """TMA path. Warp 5 is the producer: once a tile buffer is free (S or P*V of the block
    NBUF earlier has completed), its elected lane copies the block's raw kt or v tile into the
    hi buffer with ``cp.async.bulk.tensor`` (one box per 32-column strip, completing on the
    KRAW / VRAW barrier pair; no multicast, the maps cover this GPU's buffers only) and
    arrives for its warp on SGO / PVGO (for all 96 loader threads when the products are split
    around the lo pass: one buffer per tile, D = 96). Warps 6-7 wait for the copy, write the lo tile and arrive on
    SGO / PVGO (KLO / VLO when split). The tile order is the register path's: kt of block
    J + 1 before v of block J.
    On an expired wait the producer waits (bounded) for the copies it has in flight before it
    leaves, so none lands in shared memory after the CTA has exited."""
    D, NB, NQB, BKV = c["D"], c["NB"], c["NQB"], c["BKV"]
    K_BYTES, V_BYTES = D * BKV * 4, BKV * D * 4
    lt = gen.register(".u32")
    gen.emit(f"sub.u32 {lt}, {tid}, 160;")
    p_prod = gen.register(".pred")
    gen.emit(f"setp.lt.u32 {p_prod}, {lt}, 32;")
    L_work, L_end = gen.new_label("tma_work"), gen.new_label("tma_end")
    gen.emit(f"@!{p_prod} bra.uni {L_work};")

    # ---- producer (warp 5)
    p_el, el = gen.register(".pred"), gen.register(".u32")
    gen.emit(f"elect.sync {el}|{p_el}, -1;")
    tk, tv = tmap.map_address(gen, 0), tmap.map_address(gen, 1)
    gen.emit(f"@{p_el} fence.proxy.tensormap::generic.acquire.gpu [{tk}], 128;")
    gen.emit(f"@{p_el} fence.proxy.tensormap::generic.acquire.gpu [{tv}], 128;")
    gen.emit(f"@{p_el} red.global.or.b32 [emmy_path], 1;")
    L_drain = gen.new_label("tma_drain")
    J, nk, nv, zero = (gen.register(".u32") for _ in range(4))
    for r in (J, nk, nv, zero):
        gen.emit(f"mov.u32 {r}, 0;")

    def issue(X, key0, g, *, free, raw, go, step, hi, nbytes, lbo, strips, tm, coords, share):
        _after(gen, wait, B, X, c["NBUF"], free, "pfree", exit_label=L_drain)
        bar = _pair_barrier(gen, B, raw, X)
        shift = _buf_shift(gen, c, X, step)
        gen.emit(f"@{p_el} mbarrier.arrive.expect_tx.shared::cta.b64 _, [{bar}], {nbytes};")
        for s in range(strips):
            dst = gen.register(".u32")
            gen.emit(f"add.u32 {dst}, {base}, {hi + s * lbo};")
            if shift is not None:
                gen.emit(f"add.u32 {dst}, {dst}, {shift};")
            x, y = coords(s, key0)
            gen.emit(f"@{p_el} cp.async.bulk.tensor.3d.shared::cluster.global.tile"
                     f".mbarrier::complete_tx::bytes [{dst}], [{tm}, {{{x}, {y}, {g}}}], [{bar}];")
        gen.emit(f"@{p_el} mbarrier.arrive.shared::cta.b64 _, "
                 f"[{_pair_barrier(gen, B, go, X)}], {share};")

    def strip_x(s):
        if s == 0:
            return zero
        r = gen.register(".u32")
        gen.emit(f"mov.u32 {r}, {32 * s};")
        return r

    def kcoords(s, key0):
        if s == 0:
            return key0, zero
        x = gen.register(".u32")
        gen.emit(f"add.u32 {x}, {key0}, {32 * s};")
        return x, zero

    def vcoords(s, key0):
        return strip_x(s), key0

    def issue_k(X, key0, g):
        issue(X, key0, g, free="SFULL0", raw="KRAW0", go="SGO0", step=c["KSTEP"], hi=c["KHI"],
              nbytes=K_BYTES, lbo=c["LBO_K"], strips=BKV // 32, tm=tk, coords=kcoords,
              share=NLOAD if c["SPLIT"] else NLOAD - NWORK)
        gen.emit(f"add.u32 {nk}, {X}, 1;")

    def issue_v(X, key0, g):
        issue(X, key0, g, free="PVDONE0", raw="VRAW0", go="PVGO0", step=c["VSTEP"],
              hi=c["VHI"], nbytes=V_BYTES, lbo=c["LBO_V"], strips=D // 32, tm=tv,
              coords=vcoords, share=NLOAD if c["SPLIT"] else NLOAD - NWORK)
        gen.emit(f"add.u32 {nv}, {X}, 1;")

    item, close_item = _item_loop(gen, cta, ncta, c["NITEMS"], "pitem")
    g = gen.register(".u32")
    gen.emit(f"div.u32 {g}, {item}, {NQB};")
    issue_k(J, zero, g)
    j, close_j = _counted_loop(gen, NB, "pblk")
    pk = gen.register(".pred")
    gen.emit(f"setp.lt.u32 {pk}, {j}, {NB - 1};")
    L_nok = gen.new_label("pnok")
    gen.emit(f"@!{pk} bra.uni {L_nok};")
    jn, kn = gen.register(".u32"), gen.register(".u32")
    gen.emit(f"add.u32 {jn}, {J}, 1;")
    gen.emit(f"mad.lo.u32 {kn}, {j}, {BKV}, {BKV};")
    issue_k(jn, kn, g)
    gen.label(L_nok)
    kc = gen.register(".u32")
    gen.emit(f"mul.lo.u32 {kc}, {j}, {BKV};")
    issue_v(J, kc, g)
    gen.emit(f"add.u32 {J}, {J}, 1;")
    close_j()
    close_item()
    gen.label(L_drain)
    for cnt, raw in ((nk, "KRAW0"), (nv, "VRAW0")):
        for back in (1, 2):
            p = gen.register(".pred")
            gen.emit(f"setp.lt.u32 {p}, {cnt}, {back};")
            L = gen.new_label("pdrain")
            gen.emit(f"@{p} bra.uni {L};")
            _wait_pair(wait, gen, B, raw, _block_before(gen, cnt, back), exit_label=None)
            gen.label(L)
    gen.emit(f"bra.uni {L_end};")

    # ---- lo workers (warps 6-7)
    gen.label(L_work)
    wt = gen.register(".u32")
    gen.emit(f"sub.u32 {wt}, {lt}, 32;")
    W = gen.register(".u32")
    gen.emit(f"mov.u32 {W}, 0;")

    def lo(X, *, free, raw, go, step, hi, lo_, nbytes, hint):
        _after(gen, wait, B, X, c["NBUF"], free, hint)
        _wait_pair(wait, gen, B, raw, X)
        _lo_pass(gen, wt, base, _buf_shift(gen, c, X, step), hi, lo_, nbytes)
        gen.emit("fence.proxy.async.shared::cta;")
        gen.emit(f"mbarrier.arrive.shared::cta.b64 _, [{_pair_barrier(gen, B, go, X)}];")

    def lo_k(X):
        lo(X, free="SFULL0", raw="KRAW0", go="KLO0" if c["SPLIT"] else "SGO0",
           step=c["KSTEP"], hi=c["KHI"],
           lo_=c["KLO"], nbytes=K_BYTES, hint="wkfree")

    def lo_v(X):
        lo(X, free="PVDONE0", raw="VRAW0", go="VLO0" if c["SPLIT"] else "PVGO0",
           step=c["VSTEP"], hi=c["VHI"],
           lo_=c["VLO"], nbytes=V_BYTES, hint="wvfree")

    witem, wclose_item = _item_loop(gen, cta, ncta, c["NITEMS"], "witem")
    lo_k(W)
    wj, wclose_j = _counted_loop(gen, NB, "wblk")
    wpk = gen.register(".pred")
    gen.emit(f"setp.lt.u32 {wpk}, {wj}, {NB - 1};")
    L_wnok = gen.new_label("wnok")
    gen.emit(f"@!{wpk} bra.uni {L_wnok};")
    wn = gen.register(".u32")
    gen.emit(f"add.u32 {wn}, {W}, 1;")
    lo_k(wn)
    gen.label(L_wnok)
    lo_v(W)
    gen.emit(f"add.u32 {W}, {W}, 1;")
    wclose_j()
    wclose_item()
    gen.label(L_end)
