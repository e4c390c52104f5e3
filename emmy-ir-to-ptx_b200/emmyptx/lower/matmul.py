"""Contraction template: C (+)= A @ B in f32 on the 5th-generation tensor cores.

The IR describes matmul as a per-thread FMA schedule over a ``cp.async``
ring (reference ``problems/m01_matmul_512``, ``m02_matmul_rect``; lowered
statement by statement by reference ``compile.py:4858-5579``). On B200 the
template keeps only the contraction and computes it with
``tcgen05.mma.kind::tf32`` (``cta_group::1``, or ``::2`` for CTA pairs) into a
tensor-memory accumulator.

f32 accuracy with TF32 inputs (3xTF32, Ootomo & Yokota 2022): each operand
x is split into ``hi`` (x with its 13 low mantissa bits cleared, an integer
``and`` so the conversion unit stays free) and ``lo = x - hi``; the three
products ``hi*hi + hi*lo + lo*hi`` are accumulated in f32, which leaves an
error of order 2^-19 relative per product instead of 2^-11.

CTA tile 128 x BN (BN <= 256), K step 32 (one 128-byte swizzle atom of f32):

* loader warps (all warps but the last) read A and B tiles with 16-byte
  global loads, split them, and store hi and lo into shared memory in the
  canonical layouts the MMA reads: A K-major SWIZZLE_128B (8 rows x 128 B
  atoms); B[K, N] row-major stays MN-major in SWIZZLE_128B_BASE32B (32 n x
  4 k atoms), the one MN-major layout TF32 operands accept -- declared in
  the plain SWIZZLE_128B layout they multiply as zeros on B200;
* the last warp runs the issue loop converged and one ``elect.sync`` lane
  issues 3 x 4 MMAs per K step, handing the stage back with
  ``tcgen05.commit`` on the stage's "empty" mbarrier;
* warps 0-3 drain the 128 x BN accumulator with ``tcgen05.ld.32x32b``
  (warp w owns TMEM lanes 32w..32w+31, one output row per thread) and store
  it (``red.global.add.f32`` when the IR's write is atomic).

CTA pairs (even grid, M % 256 = 0, dynamic shared memory for two stages: the
benchmark shapes): the PTX declares clusters of two CTAs, each loading 128 rows
of A and half of the B tile's columns; the leader issues
``tcgen05.mma.cta_group::2`` with M = 256, which reads both CTAs' shared memory
and writes each CTA's rows into its own tensor memory, so each SM stages half of
B. The first ``SM_COUNT / 2`` clusters walk 256 x BN tiles; the tiles of an
incomplete last round run as half-width units. Ragged M, N and K (multiples of 4)
are masked: chunks outside the matrix are zero-filled, stores stop at its edge.

Stages ``S`` and ``BN`` are chosen from the shared memory the launch provides
(``meta.json`` ``smem_bytes`` is dynamic shared memory; without it the stages
live in static shared memory, 48 KiB at most). Tiles are distributed over the
launched CTAs in a grid-stride loop, so any grid is correct.

Every mbarrier wait is bounded; on expiry the kernel sets ``emmy_error`` bit 1
and leaves through the common exit, which waits (bounded) for issued MMAs and
frees its tensor memory.
"""

from __future__ import annotations

from .common import WAIT_LIMIT, tf32_split

BM = 128
BK = 32
SM_COUNT = 148                   # B200: CTA pairs that run at once = SM_COUNT / 2


def _bn_choices(N):
    """Tile widths to try for N columns, widest first: the widths that divide N, else
    (ragged N, the last tile masked) every width from the narrowest power of two that covers
    N (at most 256) down to 32."""
    exact = [bn for bn in (256, 128, 64, 32) if N % bn == 0]
    if exact:
        return exact
    return [bn for bn in (256, 128, 64, 32) if bn < 2 * N or bn == 32]


def ragged_ok(M, N, K):
    """Shapes the template takes with masked tile edges: any M, N and K multiples of 4 (rows
    of A, B and C start on 16-byte boundaries, and a 16-byte chunk is all in or all out)."""
    return M > 0 and N > 0 and K > 0 and N % 4 == 0 and K % 4 == 0


def plan_tiles(M, N, K, dyn_smem, threads):
    """(BN, stages, smem placement) for this launch, or None if the template does not fit.
    M need not be a multiple of 128, nor N and K of the tile (``ragged_ok``): the edge tiles
    load zeros past the matrix and store only what lies inside it."""
    if not ragged_ok(M, N, K) or threads < 160 or threads % 32 or threads > 1024:
        return None
    budget_dyn = dyn_smem if dyn_smem else 0
    for bn in _bn_choices(N):
        stage = 2 * BM * BK * 4 + 2 * BK * bn * 4
        if budget_dyn >= 2 * stage:
            return bn, min(budget_dyn // stage, 4), "dynamic"
    for bn in _bn_choices(N):
        stage = 2 * BM * BK * 4 + 2 * BK * bn * 4
        if budget_dyn >= stage:
            return bn, 1, "dynamic"
        if stage + 1024 + 512 <= 48 * 1024:
            return bn, 1, "static"
    return None


def plan_pair(M, N, K, dyn_smem, threads, grid):
    """(BN, stages) of the CTA-pair variant, or None: two CTAs of a cluster share one
    256 x BN tile with ``tcgen05.mma.cta_group::2``; each holds 128 rows of A and BN/2
    columns of B, so per SM the B loads and stores (and the tensor core's B reads) halve.
    Needs an even grid (clusters of 2), M % 256, and dynamic shared memory for two stages;
    N and K may be ragged (``ragged_ok``)."""
    if (grid % 2 or M % (2 * BM) or not ragged_ok(M, N, K) or threads < 160 or threads % 32
            or threads > 1024 or not dyn_smem):
        return None
    for bn in _bn_choices(N):
        if bn < 64:
            continue
        stage = 2 * BM * BK * 4 + 2 * BK * (bn // 2) * 4
        if dyn_smem >= 2 * stage:
            return bn, min(dyn_smem // stage, 4)
    return None


class _Wait:
    """Emit bounded ``mbarrier.try_wait.parity`` loops that jump to ``exit_label`` on expiry."""

    def __init__(self, gen, exit_label, scope="cta"):
        self.gen = gen
        self.exit = exit_label
        # cluster scope: the barrier also receives arrivals from the peer CTA of a pair
        self.sem = ".acquire.cluster" if scope == "cluster" else ""

    def __call__(self, mbar_addr, parity):
        gen = self.gen
        it = gen.register(".u32")
        p = gen.register(".pred")
        pl = gen.register(".pred")
        top, ok = gen.new_label("mw"), gen.new_label("mwok")
        gen.emit(f"mov.u32 {it}, 0;")
        gen.label(top)
        gen.emit(f"mbarrier.try_wait.parity{self.sem}.shared::cta.b64 {p}, [{mbar_addr}], "
                 f"{parity};")
        gen.emit(f"@{p} bra {ok};")
        gen.emit(f"add.u32 {it}, {it}, 1;")
        gen.emit(f"setp.lt.u32 {pl}, {it}, {WAIT_LIMIT};")
        gen.emit(f"@{pl} bra {top};")
        gen.emit("red.global.or.b32 [emmy_error], 2;")
        gen.emit(f"bra {self.exit};")
        gen.label(ok)


def emit_contraction(gen, kernel, a_buf, b_buf, c_buf, M, N, K, atomic):
    launch = kernel.launch
    block = list(launch.get("block", [256, 1, 1]))
    if block[1:] != [1, 1] or list(launch.get("grid", [1, 1, 1]))[1:] != [1, 1]:
        raise NotImplementedError("contraction template needs a 1-D launch")
    T = block[0]
    dyn = int(launch.get("smem_bytes", 0) or 0)
    grid = int(list(launch.get("grid", [1, 1, 1]))[0])
    pp = plan_pair(M, N, K, dyn, T, grid)
    if pp is not None:
        BN, S = pp
        place, pair = "dynamic", True
    else:
        plan = plan_tiles(M, N, K, dyn, T)
        if plan is None:
            raise NotImplementedError("contraction shape or launch outside the tcgen05 template")
        BN, S, place = plan
        pair = False
    BNH = BN // 2 if pair else BN        # columns of B this CTA loads (half of the tile's)
    NW = T // 32
    NL = T - 32                          # loader threads: every warp but the last
    QA = BM * BK // 4                    # 16-byte chunks of an A tile
    QB = BK * BNH // 4                   # 16-byte chunks of this CTA's B tile
    A_BYTES = BM * BK * 4
    B_BYTES = BK * BNH * 4
    STAGE = 2 * A_BYTES + 2 * B_BYTES
    SBO_B = 16 * BNH                     # stride between 4-row K groups of the B tile
    KB = -(-K // BK)
    NT_N = -(-N // BN)
    MT = 2 * BM if pair else BM          # rows of C one unit covers
    NTILES = -(-M // MT) * NT_N
    # ragged edges (masked): rows of A and C past M, columns of B and C past N, the K tail
    RAG_M, RAG_N, RAG_K = M % MT != 0, N % BN != 0, K % BK != 0
    # two accumulators of BN columns: the MMAs of a unit run while the epilogue drains the
    # previous unit's
    TMEM_COLS = 32
    while TMEM_COLS < 2 * BN:
        TMEM_COLS *= 2
    CG = "cta_group::2" if pair else "cta_group::1"
    # Pairs: only the first P clusters work (one per SM pair), over NUNITS units: F full tiles
    # (F a multiple of P), then the R = NTILES % P remaining tiles as 2R half-width units
    # (256 x BN/2, disjoint columns) when 2R <= P, so the last round takes half a tile's time
    # instead of a whole one with most SM pairs idle. Needs BN/2 >= 64 (half of a CTA's B
    # still a whole 32-column atom). Without pairs: tiles grid-stride over all CTAs.
    P = F = H = 0
    NUNITS = NTILES
    if pair:
        P = max(1, min(grid // 2, SM_COUNT // 2))
        R = NTILES % P
        F, H = (NTILES - R, 2 * R) if (R and 2 * R <= P and BNH >= 64) else (NTILES, 0)
        NUNITS = F + H
    gen.maxntid = T
    if pair:
        gen.cluster = 2

    gen.module_decl(".global .align 4 .u32 emmy_error;")
    if place == "dynamic":
        gen.module_decl(".extern .shared .align 1024 .b8 emmy_dsmem[];")
    else:
        gen.shared("emmy_stage", ".b8", length=S * STAGE + 1024, align=1024)
    gen.shared("emmy_bar", ".b64", length=2 * S + 5, align=8)
    gen.shared("emmy_tmem_slot", ".b32", length=1, align=4)

    ptrs = {}
    for name in kernel.arg_order:
        raw, g = gen.register(".u64"), gen.register(".u64")
        gen.emit(f"ld.param.u64 {raw}, [{gen.parameter(name)}];")
        gen.emit(f"cvta.to.global.u64 {g}, {raw};")
        ptrs[name] = g
    A, B, C = ptrs[a_buf], ptrs[b_buf], ptrs[c_buf]

    tid, warp, lane = gen.register(".u32"), gen.register(".u32"), gen.register(".u32")
    gen.emit(f"mov.u32 {tid}, %tid.x;")
    gen.emit(f"shr.u32 {warp}, {tid}, 5;")
    gen.emit(f"and.b32 {lane}, {tid}, 31;")
    if pair and grid // 2 > P:
        # clusters beyond the P that work leave before any barrier (both CTAs of a cluster)
        cid0, p_idle = gen.register(".u32"), gen.register(".pred")
        gen.emit(f"mov.u32 {cid0}, %clusterid.x;")
        gen.emit(f"setp.ge.u32 {p_idle}, {cid0}, {P};")
        gen.emit(f"@{p_idle} ret;")

    # ---- shared memory bases ------------------------------------------------------------
    base = gen.register(".u32")
    gen.emit(f"mov.u32 {base}, {'emmy_dsmem' if place == 'dynamic' else 'emmy_stage'};")
    gen.emit(f"add.u32 {base}, {base}, 1023;")
    gen.emit(f"and.b32 {base}, {base}, -1024;")
    if place == "dynamic":
        # the stages need S*STAGE bytes from the 1024-aligned base; leave (error bit 2) if the
        # launch's dynamic shared memory does not cover them
        dsz, used = gen.register(".u32"), gen.register(".u32")
        gen.emit(f"mov.u32 {dsz}, %dynamic_smem_size;")
        gen.emit(f"mov.u32 {used}, emmy_dsmem;")
        gen.emit(f"sub.u32 {used}, {base}, {used};")
        gen.emit(f"add.u32 {used}, {used}, {S * STAGE};")
        p_small = gen.register(".pred")
        gen.emit(f"setp.gt.u32 {p_small}, {used}, {dsz};")
        L_fit = gen.new_label("fits")
        gen.emit(f"@!{p_small} bra {L_fit};")
        gen.emit("red.global.or.b32 [emmy_error], 4;")
        gen.emit("ret;")
        gen.label(L_fit)
    bar = gen.register(".u32")
    gen.emit(f"mov.u32 {bar}, emmy_bar;")
    # barrier k: full[s] = bar + 8s, empty[s] = bar + 8(S+s), acc_full, acc_empty, drain
    full = lambda s: f"{bar}+{8 * s}"             # noqa: E731
    empty = lambda s: f"{bar}+{8 * (S + s)}"      # noqa: E731
    # acc_full[b] = bar + 8(2S+b), acc_empty[b] = bar + 8(2S+2+b), b the accumulator
    AF0, AE0 = 8 * (2 * S), 8 * (2 * S + 2)
    DRAIN = f"{bar}+{8 * (2 * S + 4)}"

    L_exit = gen.new_label("exit")
    wait = _Wait(gen, L_exit, "cluster" if pair else "cta")

    rank = None
    full_count = NL
    if pair:
        # each CTA's loaders arrive on their own "full" barriers; in the peer (rank 1) its
        # last warp forwards each completed phase to the leader's, which counts NL + 1
        rank = gen.register(".u32")
        gen.emit(f"mov.u32 {rank}, %cluster_ctarank;")
        full_count = gen.register(".u32")
        p_lead = gen.register(".pred")
        gen.emit(f"setp.eq.u32 {p_lead}, {rank}, 0;")
        gen.emit(f"selp.u32 {full_count}, {NL + 1}, {NL}, {p_lead};")
    p_t0 = gen.register(".pred")
    gen.emit(f"setp.eq.u32 {p_t0}, {tid}, 0;")
    L_noinit = gen.new_label("noinit")
    gen.emit(f"@!{p_t0} bra {L_noinit};")
    # in a pair, "acc_empty" of the leader CTA (rank 0) counts both CTAs' epilogue threads
    for s in range(S):
        gen.emit(f"mbarrier.init.shared::cta.b64 [{full(s)}], {full_count};")
        gen.emit(f"mbarrier.init.shared::cta.b64 [{empty(s)}], 1;")
    for b in range(2):
        gen.emit(f"mbarrier.init.shared::cta.b64 [{bar}+{AF0 + 8 * b}], 1;")
        gen.emit(f"mbarrier.init.shared::cta.b64 [{bar}+{AE0 + 8 * b}], {256 if pair else 128};")
    gen.emit(f"mbarrier.init.shared::cta.b64 [{DRAIN}], 1;")
    gen.emit("fence.mbarrier_init.release.cluster;")
    gen.label(L_noinit)

    # ---- tensor memory: the last warp allocates the accumulator columns -----------------
    p_mw = gen.register(".pred")
    gen.emit(f"setp.eq.u32 {p_mw}, {warp}, {NW - 1};")
    L_noalloc = gen.new_label("noalloc")
    gen.emit(f"@!{p_mw} bra {L_noalloc};")
    slot = gen.register(".u32")
    gen.emit(f"mov.u32 {slot}, emmy_tmem_slot;")
    # (in a pair the last warp of both CTAs allocates: the same columns in both)
    gen.emit(f"tcgen05.alloc.{CG}.sync.aligned.shared::cta.b32 [{slot}], {TMEM_COLS};")
    gen.emit(f"tcgen05.relinquish_alloc_permit.{CG}.sync.aligned;")
    gen.emit("tcgen05.fence::before_thread_sync;")
    gen.label(L_noalloc)
    if pair:
        # both CTAs' barriers are initialised before any thread of the pair uses them
        gen.emit("barrier.cluster.arrive.release;")
        gen.emit("barrier.cluster.wait.acquire;")
    else:
        gen.emit("bar.sync 0;")
    gen.emit("tcgen05.fence::after_thread_sync;")
    tmem = gen.register(".u32")
    gen.emit(f"ld.shared.b32 {tmem}, [emmy_tmem_slot];")

    cta, ncta = gen.register(".u32"), gen.register(".u32")
    lead_bar = None
    if pair:
        # tiles are walked per cluster; rank 0 (the leader) issues the pair's MMAs
        gen.emit(f"mov.u32 {cta}, %clusterid.x;")
        gen.emit(f"mov.u32 {ncta}, {P};")
        lead_bar = gen.register(".u32")             # the leader's barriers, cluster address
        gen.emit(f"mapa.shared::cluster.u32 {lead_bar}, {bar}, 0;")
    else:
        gen.emit(f"mov.u32 {cta}, %ctaid.x;")
        gen.emit(f"mov.u32 {ncta}, %nctaid.x;")

    L_mma_role = gen.new_label("mma_role")
    gen.emit(f"@{p_mw} bra {L_mma_role};")

    # =================================== loader / epilogue warps ==========================
    # per-thread chunk offsets (global byte offset within a tile, shared byte offset)
    a_chunks, b_chunks = [], []
    a_edge = []                        # per A chunk: (row in the tile, K column in the step)
    for i in range(-(-QA // NL)):
        q = gen.register(".u32")
        gen.emit(f"add.u32 {q}, {tid}, {i * NL};")
        pv = None
        if (i + 1) * NL > QA:
            pv = gen.register(".pred")
            gen.emit(f"setp.lt.u32 {pv}, {q}, {QA};")
        row, c, r8 = gen.register(".u32"), gen.register(".u32"), gen.register(".u32")
        gen.emit(f"shr.u32 {row}, {q}, 3;")
        gen.emit(f"and.b32 {c}, {q}, 7;")
        gen.emit(f"and.b32 {r8}, {row}, 7;")
        goff = gen.register(".u64")
        t32 = gen.register(".u32")
        gen.emit(f"mad.lo.u32 {t32}, {row}, {K}, 0;")
        gen.emit(f"shl.b32 {c}, {c}, 2;")
        gen.emit(f"add.u32 {t32}, {t32}, {c};")
        gen.emit(f"mul.wide.u32 {goff}, {t32}, 4;")
        soff = gen.register(".u32")
        sw = gen.register(".u32")
        kcol = gen.register(".u32")              # the chunk's first K column in the step
        gen.emit(f"mov.u32 {kcol}, {c};")
        gen.emit(f"shr.u32 {c}, {c}, 2;")
        gen.emit(f"xor.b32 {sw}, {c}, {r8};")
        gen.emit(f"shl.b32 {sw}, {sw}, 4;")
        gen.emit(f"shl.b32 {soff}, {row}, 7;")
        gen.emit(f"add.u32 {soff}, {soff}, {sw};")
        a_chunks.append((goff, soff, pv))
        a_edge.append((row, kcol))
    # B[K, N] row-major is N-contiguous, so it is stored MN-major in the SWIZZLE_128B_BASE32B
    # layout (the only MN-major layout TF32 operands support): atoms of 32 n x 4 k (512 B), the
    # BN/32 atoms of a 4-row K group side by side (LBO 512 B), K groups SBO_B = 16*BN bytes apart;
    # within a 128-byte row the 32-byte unit (n%32)/8 is XORed with k%4.
    def b_chunk_list(cols):
        """This thread's chunks of a B tile ``cols`` columns wide (chunks tid + i*NL), in the
        layout of a BNH-wide tile: a narrower tile fills the first cols/32 atoms of each K
        group, so the MMA reads it with the same descriptors and a smaller N."""
        QBc = BK * cols // 4
        out, edge = [], []
        for i in range(-(-QBc // NL)):
            q = gen.register(".u32")
            gen.emit(f"add.u32 {q}, {tid}, {i * NL};")
            pv = None
            if (i + 1) * NL > QBc:
                pv = gen.register(".pred")
                gen.emit(f"setp.lt.u32 {pv}, {q}, {QBc};")
            k, cn = gen.register(".u32"), gen.register(".u32")
            gen.emit(f"shr.u32 {k}, {q}, {(cols // 4).bit_length() - 1};")
            gen.emit(f"and.b32 {cn}, {q}, {cols // 4 - 1};")        # 16-byte chunk along n
            t32 = gen.register(".u32")
            gen.emit(f"mul.lo.u32 {t32}, {k}, {N};")
            n4 = gen.register(".u32")
            gen.emit(f"shl.b32 {n4}, {cn}, 2;")
            gen.emit(f"add.u32 {t32}, {t32}, {n4};")
            goff = gen.register(".u64")
            gen.emit(f"mul.wide.u32 {goff}, {t32}, 4;")
            j, c8, u32b, half, k4, kq = (gen.register(".u32") for _ in range(6))
            gen.emit(f"shr.u32 {j}, {cn}, 3;")                     # n / 32
            gen.emit(f"and.b32 {c8}, {cn}, 7;")                    # (n % 32) / 4
            gen.emit(f"shr.u32 {u32b}, {c8}, 1;")                  # 32-byte unit
            gen.emit(f"and.b32 {half}, {c8}, 1;")
            gen.emit(f"and.b32 {k4}, {k}, 3;")
            gen.emit(f"shr.u32 {kq}, {k}, 2;")
            soff = gen.register(".u32")
            gen.emit(f"mul.lo.u32 {soff}, {kq}, {SBO_B};")
            gen.emit(f"mad.lo.u32 {soff}, {j}, 512, {soff};")
            gen.emit(f"mad.lo.u32 {soff}, {k4}, 128, {soff};")
            gen.emit(f"xor.b32 {u32b}, {u32b}, {k4};")
            gen.emit(f"mad.lo.u32 {soff}, {u32b}, 32, {soff};")
            gen.emit(f"mad.lo.u32 {soff}, {half}, 16, {soff};")
            out.append((goff, soff, pv))
            edge.append((k, n4))             # (K row in the step, column in the tile)
        return out, edge

    b_chunks, b_edge = b_chunk_list(BNH)
    b_chunks_half, b_edge_half = b_chunk_list(BNH // 2) if H else (None, None)

    def unit_tile(u):
        """(tile index, which half, is-half predicate) of work unit ``u``: units below F are
        whole tiles, the H after them halves of the last tiles (two per tile)."""
        if not H:
            return u, None, None
        ph = gen.register(".pred")
        gen.emit(f"setp.ge.u32 {ph}, {u}, {F};")
        h, t, hs = gen.register(".u32"), gen.register(".u32"), gen.register(".u32")
        gen.emit(f"sub.u32 {h}, {u}, {F};")
        gen.emit(f"shr.u32 {t}, {h}, 1;")
        gen.emit(f"add.u32 {t}, {t}, {F};")
        gen.emit(f"selp.u32 {t}, {t}, {u}, {ph};")
        gen.emit(f"and.b32 {hs}, {h}, 1;")
        gen.emit(f"selp.u32 {hs}, {hs}, 0, {ph};")
        return t, hs, ph

    it = gen.register(".u32")          # global K-step counter (ring position)
    tcount = gen.register(".u32")      # tiles finished by this CTA
    tile = gen.register(".u32")
    gen.emit(f"mov.u32 {it}, 0;")
    gen.emit(f"mov.u32 {tcount}, 0;")
    gen.emit(f"mov.u32 {tile}, {cta};")
    p_epi = gen.register(".pred")
    gen.emit(f"setp.lt.u32 {p_epi}, {warp}, 4;")

    L_tile = gen.new_label("ltile")
    L_tiles_done = gen.new_label("ltilesdone")
    pt = gen.register(".pred")
    gen.label(L_tile)
    gen.emit(f"setp.ge.u32 {pt}, {tile}, {NUNITS};")
    gen.emit(f"@{pt} bra {L_tiles_done};")
    tt, hsel, p_half = unit_tile(tile)
    mb, nb = gen.register(".u32"), gen.register(".u32")
    gen.emit(f"div.u32 {mb}, {tt}, {NT_N};")
    gen.emit(f"rem.u32 {nb}, {tt}, {NT_N};")
    a_tile = gen.register(".u64")            # A + m0*K*4
    m0 = gen.register(".u32")
    if pair:                                 # this CTA's 128 rows of the 256-row pair tile
        gen.emit(f"mad.lo.u32 {m0}, {mb}, {2 * BM}, 0;")
        rk = gen.register(".u32")
        gen.emit(f"mul.lo.u32 {rk}, {rank}, {BM};")
        gen.emit(f"add.u32 {m0}, {m0}, {rk};")
    else:
        gen.emit(f"mul.lo.u32 {m0}, {mb}, {BM};")
    tmp64 = gen.register(".u64")
    gen.emit(f"mul.wide.u32 {tmp64}, {m0}, {K * 4};")
    gen.emit(f"add.s64 {a_tile}, {A}, {tmp64};")
    b_tile = gen.register(".u64")            # B + (n0 + this CTA's half)*4
    n0 = gen.register(".u32")                # the tile's first column (of C)
    gen.emit(f"mul.lo.u32 {n0}, {nb}, {BN};")
    if H:                                    # second half of a split tile: BN/2 further
        gen.emit(f"mad.lo.u32 {n0}, {hsel}, {BN // 2}, {n0};")
    nb0 = n0
    if pair:                                 # this CTA's columns: half of the unit's width
        nb0 = gen.register(".u32")
        if H:
            wdt = gen.register(".u32")
            gen.emit(f"selp.u32 {wdt}, {BNH // 2}, {BNH}, {p_half};")
            gen.emit(f"mad.lo.u32 {nb0}, {rank}, {wdt}, {n0};")
        else:
            gen.emit(f"mad.lo.u32 {nb0}, {rank}, {BNH}, {n0};")
    gen.emit(f"mul.wide.u32 {tmp64}, {nb0}, 4;")
    gen.emit(f"add.s64 {b_tile}, {B}, {tmp64};")

    # ragged edges: per unit, which of this thread's chunks lie inside M (A rows) and N (B
    # columns); the K tail is checked per step in issue_loads
    tile_ok = {}
    if RAG_M:
        tile_ok["a"] = []
        for row, _ in a_edge:
            t, q = gen.register(".u32"), gen.register(".pred")
            gen.emit(f"add.u32 {t}, {m0}, {row};")
            gen.emit(f"setp.lt.u32 {q}, {t}, {M};")
            tile_ok["a"].append(q)
    if RAG_N:
        for key, edge in (("b", b_edge), ("bh", b_edge_half)):
            if edge is None:
                continue
            tile_ok[key] = []
            for _, n4 in edge:
                t, q = gen.register(".u32"), gen.register(".pred")
                gen.emit(f"add.u32 {t}, {nb0}, {n4};")
                gen.emit(f"setp.lt.u32 {q}, {t}, {N};")
                tile_ok[key].append(q)

    def issue_loads(kb, regs=None, bch=b_chunks):
        """Global loads of K step ``kb`` (a register or an int) into ``regs`` (new if None).
        With ragged edges a chunk outside the matrix is zeroed instead of loaded."""
        a_k, b_k = gen.register(".u64"), gen.register(".u64")
        kk = None
        if isinstance(kb, int):
            gen.emit(f"add.s64 {a_k}, {a_tile}, {kb * BK * 4};")
            gen.emit(f"add.s64 {b_k}, {b_tile}, {kb * BK * N * 4};")
            if RAG_K:
                kk = gen.register(".u32")
                gen.emit(f"mov.u32 {kk}, {kb * BK};")
        else:
            gen.emit(f"mul.wide.u32 {tmp64}, {kb}, {BK * 4};")
            gen.emit(f"add.s64 {a_k}, {a_tile}, {tmp64};")
            gen.emit(f"mul.wide.u32 {tmp64}, {kb}, {BK * N * 4};")
            gen.emit(f"add.s64 {b_k}, {b_tile}, {tmp64};")
            if RAG_K:
                kk = gen.register(".u32")
                gen.emit(f"mul.lo.u32 {kk}, {kb}, {BK};")
        out = regs if regs is not None else [gen.registers(".f32", 4)
                                             for _ in range(len(a_chunks) + len(bch))]
        nA = len(a_chunks)
        bkey = "b" if bch is b_chunks else "bh"
        bedge = b_edge if bch is b_chunks else b_edge_half
        for idx, (goff, soff, pv) in enumerate(a_chunks + bch):
            addr = gen.register(".u64")
            gen.emit(f"add.s64 {addr}, {a_k if idx < nA else b_k}, {goff};")
            conds = [pv] if pv else []
            if idx < nA and "a" in tile_ok:
                conds.append(tile_ok["a"][idx])
            if idx >= nA and bkey in tile_ok:
                conds.append(tile_ok[bkey][idx - nA])
            if RAG_K:
                kpos = a_edge[idx][1] if idx < nA else bedge[idx - nA][0]
                t, q = gen.register(".u32"), gen.register(".pred")
                gen.emit(f"add.u32 {t}, {kk}, {kpos};")
                gen.emit(f"setp.lt.u32 {q}, {t}, {K};")
                conds.append(q)
            masked = len(conds) > (1 if pv else 0)
            if masked:                       # zeros where the chunk lies outside the matrix
                for r in out[idx]:
                    gen.emit(f"mov.f32 {r}, 0f00000000;")
            pred = ""
            if conds:
                q = conds[0]
                for extra in conds[1:]:
                    t = gen.register(".pred")
                    gen.emit(f"and.pred {t}, {q}, {extra};")
                    q = t
                pred = f"@{q} "
            gen.emit(f"{pred}ld.global.nc.L1::no_allocate.v4.f32 {{{', '.join(out[idx])}}}, "
                     f"[{addr}];")
        return out

    def split_store(hi_base, lo_base, soff, values, pv):
        his, los = [], []
        for x in values:
            h, lo = tf32_split(gen, x)
            his.append(h)
            los.append(lo)
        pred = f"@{pv} " if pv else ""
        ah, al = gen.register(".u32"), gen.register(".u32")
        gen.emit(f"add.u32 {ah}, {hi_base}, {soff};")
        gen.emit(f"add.u32 {al}, {lo_base}, {soff};")
        gen.emit(f"{pred}st.shared.v4.b32 [{ah}], {{{', '.join(his)}}};")
        gen.emit(f"{pred}st.shared.v4.b32 [{al}], {{{', '.join(los)}}};")

    def store_step(vals, bch=b_chunks):
        """Wait until the MMA has released the ring slot of step ``it`` (skipped for the first
        S steps), split and store the loaded values, hand the slot to the MMA warp."""
        s_reg, ph = gen.register(".u32"), gen.register(".u32")
        gen.emit(f"rem.u32 {s_reg}, {it}, {S};")
        gen.emit(f"div.u32 {ph}, {it}, {S};")
        gen.emit(f"and.b32 {ph}, {ph}, 1;")
        L_nowait = gen.new_label("nowait")
        p_first = gen.register(".pred")
        gen.emit(f"setp.lt.u32 {p_first}, {it}, {S};")
        gen.emit(f"@{p_first} bra {L_nowait};")
        emp = gen.register(".u32")
        gen.emit(f"mad.lo.u32 {emp}, {s_reg}, 8, {bar};")
        gen.emit(f"add.u32 {emp}, {emp}, {8 * S};")
        php = gen.register(".u32")
        gen.emit(f"xor.b32 {php}, {ph}, 1;")
        wait(emp, php)
        gen.label(L_nowait)
        sbase = gen.register(".u32")
        gen.emit(f"mad.lo.u32 {sbase}, {s_reg}, {STAGE}, {base};")
        bases = {"ahi": sbase}
        for nm, off in (("alo", A_BYTES), ("bhi", 2 * A_BYTES), ("blo", 2 * A_BYTES + B_BYTES)):
            r = gen.register(".u32")
            gen.emit(f"add.u32 {r}, {sbase}, {off};")
            bases[nm] = r
        nA = len(a_chunks)
        for idx, ((goff, soff, pv), regs) in enumerate(zip(a_chunks + bch, vals)):
            if idx < nA:
                split_store(bases["ahi"], bases["alo"], soff, regs, pv)
            else:
                split_store(bases["bhi"], bases["blo"], soff, regs, pv)
        gen.emit("fence.proxy.async.shared::cta;")
        fb = gen.register(".u32")
        gen.emit(f"mad.lo.u32 {fb}, {s_reg}, 8, {bar};")
        gen.emit(f"mbarrier.arrive.shared::cta.b64 _, [{fb}];")
        gen.emit(f"add.u32 {it}, {it}, 1;")

    def k_loop(bch):
        """The K steps of one unit with B chunk list ``bch``."""
        kb = gen.register(".u32")
        gen.emit(f"mov.u32 {kb}, 0;")
        L_k = gen.new_label("lk")
        L_kdone = gen.new_label("lkdone")
        pk = gen.register(".pred")
        if KB % 2 == 0:
            # software pipelined by two register sets: the loads of step kb + 1 are in flight
            # while step kb waits for its ring slot and is stored
            X = issue_loads(0, bch=bch)
            gen.label(L_k)
            gen.emit(f"setp.ge.u32 {pk}, {kb}, {KB};")
            gen.emit(f"@{pk} bra {L_kdone};")
            k1 = gen.register(".u32")
            gen.emit(f"add.u32 {k1}, {kb}, 1;")
            Y = issue_loads(k1, bch=bch)
            store_step(X, bch)
            k2 = gen.register(".u32")
            gen.emit(f"add.u32 {k2}, {kb}, 2;")
            p2 = gen.register(".pred")
            gen.emit(f"setp.lt.u32 {p2}, {k2}, {KB};")
            L_nox = gen.new_label("nox")
            gen.emit(f"@!{p2} bra {L_nox};")
            issue_loads(k2, X, bch=bch)
            gen.label(L_nox)
            store_step(Y, bch)
            gen.emit(f"add.u32 {kb}, {kb}, 2;")
            gen.emit(f"bra.uni {L_k};")
        else:
            gen.label(L_k)
            gen.emit(f"setp.ge.u32 {pk}, {kb}, {KB};")
            gen.emit(f"@{pk} bra {L_kdone};")
            store_step(issue_loads(kb, bch=bch), bch)
            gen.emit(f"add.u32 {kb}, {kb}, 1;")
            gen.emit(f"bra.uni {L_k};")
        gen.label(L_kdone)

    if H:
        L_khalf, L_kend = gen.new_label("khalf"), gen.new_label("kend")
        gen.emit(f"@{p_half} bra {L_khalf};")
        k_loop(b_chunks)
        gen.emit(f"bra.uni {L_kend};")
        gen.label(L_khalf)
        k_loop(b_chunks_half)
        gen.label(L_kend)
    else:
        k_loop(b_chunks)

    # ---- epilogue (warps 0-3): TMEM -> registers -> C ------------------------------------
    L_noepi = gen.new_label("noepi")
    gen.emit(f"@!{p_epi} bra {L_noepi};")
    ab, tph, afb = gen.register(".u32"), gen.register(".u32"), gen.register(".u32")
    gen.emit(f"and.b32 {ab}, {tcount}, 1;")             # this unit's accumulator
    gen.emit(f"shr.u32 {tph}, {tcount}, 1;")
    gen.emit(f"and.b32 {tph}, {tph}, 1;")
    gen.emit(f"mad.lo.u32 {afb}, {ab}, 8, {bar};")
    gen.emit(f"add.u32 {afb}, {afb}, {AF0};")
    wait(afb, tph)
    gen.emit("tcgen05.fence::after_thread_sync;")
    row = gen.register(".u32")
    gen.emit(f"shl.b32 {row}, {warp}, 5;")
    gen.emit(f"add.u32 {row}, {row}, {lane};")
    grow = gen.register(".u32")
    gen.emit(f"add.u32 {grow}, {m0}, {row};")
    crow = gen.register(".u64")
    t32 = gen.register(".u32")
    gen.emit(f"mad.lo.u32 {t32}, {grow}, {N}, {n0};")
    gen.emit(f"mul.wide.u32 {crow}, {t32}, 4;")
    gen.emit(f"add.s64 {crow}, {C}, {crow};")
    lane_field = gen.register(".u32")
    gen.emit(f"shl.b32 {lane_field}, {warp}, 21;")        # (32*warp) << 16
    gen.emit(f"mad.lo.u32 {lane_field}, {ab}, {BN}, {lane_field};")   # + accumulator columns
    gen.emit("bar.warp.sync -1;")
    width = 64 if BN >= 64 else 32
    # ragged edges: rows past M and 4-column chunks past N are not stored
    p_rowok = ncols_left = None
    if RAG_M:
        p_rowok = gen.register(".pred")
        gen.emit(f"setp.lt.u32 {p_rowok}, {grow}, {M};")
    if RAG_N:
        ncols_left = gen.register(".s32")
        gen.emit(f"sub.s32 {ncols_left}, {N}, {n0};")
    L_cols_done = gen.new_label("colsdone")
    for cb in range(BN // width):
        if H and cb == (BN // 2) // width:
            gen.emit(f"@{p_half} bra {L_cols_done};")       # a half unit has BN/2 columns
        regs = gen.registers(".b32", width)
        ta = gen.register(".u32")
        gen.emit(f"add.u32 {ta}, {tmem}, {lane_field};")
        gen.emit(f"add.u32 {ta}, {ta}, {cb * width};")
        gen.emit(f"tcgen05.ld.sync.aligned.32x32b.x{width}.b32 {{{', '.join(regs)}}}, [{ta}];")
        gen.emit("tcgen05.wait::ld.sync.aligned;")
        for v in range(width // 4):
            four = regs[4 * v:4 * v + 4]
            off = 4 * (cb * width + 4 * v)
            pred = ""
            if RAG_N:
                q = gen.register(".pred")
                gen.emit(f"setp.gt.s32 {q}, {ncols_left}, {cb * width + 4 * v};")
                if p_rowok is not None:
                    gen.emit(f"and.pred {q}, {q}, {p_rowok};")
                pred = f"@{q} "
            elif p_rowok is not None:
                pred = f"@{p_rowok} "
            if atomic:
                for e, r in enumerate(four):
                    f = gen.register(".f32")
                    gen.emit(f"mov.b32 {f}, {r};")
                    gen.emit(f"{pred}red.global.add.f32 [{crow}+{off + 4 * e}], {f};")
            else:
                gen.emit(f"{pred}st.global.v4.b32 [{crow}+{off}], {{{', '.join(four)}}};")
    gen.label(L_cols_done)
    gen.emit("tcgen05.fence::before_thread_sync;")
    aeb = gen.register(".u32")
    if pair:                               # both CTAs' epilogues free the pair's accumulator
        gen.emit(f"mad.lo.u32 {aeb}, {ab}, 8, {lead_bar};")
        gen.emit(f"mbarrier.arrive.release.cluster.shared::cluster.b64 _, [{aeb}+{AE0}];")
    else:
        gen.emit(f"mad.lo.u32 {aeb}, {ab}, 8, {bar};")
        gen.emit(f"mbarrier.arrive.shared::cta.b64 _, [{aeb}+{AE0}];")
    gen.label(L_noepi)
    gen.emit(f"add.u32 {tcount}, {tcount}, 1;")
    gen.emit(f"add.u32 {tile}, {tile}, {ncta};")
    gen.emit(f"bra.uni {L_tile};")
    gen.label(L_tiles_done)
    gen.emit(f"bra.uni {L_exit};")

    # =================================== MMA warp ===========================================
    gen.label(L_mma_role)
    # The whole warp runs the issue loop converged; one elected lane issues each tcgen05.mma
    # and tcgen05.commit (their operands are read as warp-uniform values).
    L_mma_done = gen.new_label("mmadone")
    peer_bar = None
    p_el = gen.register(".pred")
    el_r = gen.register(".u32")
    gen.emit(f"elect.sync {el_r}|{p_el}, -1;")
    if pair:
        # Only the leader issues. The peer's last warp forwards each completed phase of its
        # own "full" barriers to the leader's with one cluster-scope release arrive: the
        # loaders arrive locally (a CTA-scope release does not wait for their prefetched
        # global loads, a cluster-scope one would), and release is cumulative, so the
        # peer's stored tiles are visible to the leader's MMA once it sees the phase.
        L_lead = gen.new_label("lead")
        gen.emit(f"setp.eq.u32 {p_lead}, {rank}, 0;")
        gen.emit(f"@{p_lead} bra {L_lead};")
        fit, ftile = gen.register(".u32"), gen.register(".u32")
        gen.emit(f"mov.u32 {fit}, 0;")
        gen.emit(f"mov.u32 {ftile}, {cta};")
        L_ft, L_fk, L_fkd = gen.new_label("ft"), gen.new_label("fk"), gen.new_label("fkd")
        pf = gen.register(".pred")
        gen.label(L_ft)
        gen.emit(f"setp.ge.u32 {pf}, {ftile}, {NUNITS};")
        gen.emit(f"@{pf} bra {L_exit};")
        fkb = gen.register(".u32")
        gen.emit(f"mov.u32 {fkb}, 0;")
        gen.label(L_fk)
        gen.emit(f"setp.ge.u32 {pf}, {fkb}, {KB};")
        gen.emit(f"@{pf} bra {L_fkd};")
        fs, fph, fb2 = gen.register(".u32"), gen.register(".u32"), gen.register(".u32")
        gen.emit(f"rem.u32 {fs}, {fit}, {S};")
        gen.emit(f"div.u32 {fph}, {fit}, {S};")
        gen.emit(f"and.b32 {fph}, {fph}, 1;")
        gen.emit(f"mad.lo.u32 {fb2}, {fs}, 8, {bar};")
        wait(fb2, fph)
        gen.emit(f"mad.lo.u32 {fb2}, {fs}, 8, {lead_bar};")
        gen.emit(f"@{p_el} mbarrier.arrive.release.cluster.shared::cluster.b64 _, [{fb2}];")
        gen.emit(f"add.u32 {fit}, {fit}, 1;")
        gen.emit(f"add.u32 {fkb}, {fkb}, 1;")
        gen.emit(f"bra.uni {L_fk};")
        gen.label(L_fkd)
        gen.emit(f"add.u32 {ftile}, {ftile}, {ncta};")
        gen.emit(f"bra.uni {L_ft};")
        gen.label(L_lead)
        peer_bar = gen.register(".u32")             # the peer's barriers, cluster address
        gen.emit(f"mapa.shared::cluster.u32 {peer_bar}, {bar}, 1;")
    MM = 2 * BM if pair else BM          # rows of one MMA (a pair spans both CTAs)
    idesc = (1 << 4) | (2 << 7) | (2 << 10) | (1 << 16) | ((BN >> 3) << 17) | ((MM >> 4) << 24)
    idesc_half = (idesc & ~(0x3F << 17)) | (((BN // 2) >> 3) << 17)
    a_hi_word = (1024 >> 4) | (1 << 14) | (2 << 29)        # SBO 1024 B, version 1, SWIZZLE_128B
    b_hi_word = (SBO_B >> 4) | (1 << 14) | (1 << 29)        # SWIZZLE_128B_BASE32B
    a_lo_word = 1 << 16                                     # LBO 16 B (unused by swizzled K-major)
    b_lo_word = (512 >> 4) << 16                            # LBO 512 B between N atoms
    r_idesc = gen.register(".u32")
    gen.emit(f"mov.u32 {r_idesc}, {idesc};")
    a_hi = gen.register(".u32")
    gen.emit(f"mov.u32 {a_hi}, {a_hi_word};")
    b_hi = gen.register(".u32")
    gen.emit(f"mov.u32 {b_hi}, {b_hi_word};")
    p_true = gen.register(".pred")
    gen.emit(f"setp.eq.u32 {p_true}, {lane}, {lane};")

    def commit(offset):
        """Arrive on this CTA's barrier at ``bar + offset`` (a register or an int) when this
        thread's MMAs so far are done; in a pair also on the same barrier of the peer CTA
        (one commit each: the peer's loaders and epilogue wait on their own barriers)."""
        for base_reg in ([bar, peer_bar] if pair else [bar]):
            a = gen.register(".u32")
            gen.emit(f"add.u32 {a}, {base_reg}, {offset};")
            gen.emit(f"@{p_el} tcgen05.commit.{CG}.mbarrier::arrive::one.shared::cluster.b64 "
                     f"[{a}];")

    mit, mt, mtile = gen.register(".u32"), gen.register(".u32"), gen.register(".u32")
    gen.emit(f"mov.u32 {mit}, 0;")
    gen.emit(f"mov.u32 {mt}, 0;")
    gen.emit(f"mov.u32 {mtile}, {cta};")
    L_mt = gen.new_label("mt")
    pmt = gen.register(".pred")
    gen.label(L_mt)
    gen.emit(f"setp.ge.u32 {pmt}, {mtile}, {NUNITS};")
    gen.emit(f"@{pmt} bra {L_mma_done};")
    # accumulator mt % 2: wait until the epilogue has drained it (units mt - 2, ...)
    mab, dacc = gen.register(".u32"), gen.register(".u32")
    gen.emit(f"and.b32 {mab}, {mt}, 1;")
    gen.emit(f"mad.lo.u32 {dacc}, {mab}, {BN}, {tmem};")
    L_skipe = gen.new_label("skipe")
    p_t1 = gen.register(".pred")
    gen.emit(f"setp.lt.u32 {p_t1}, {mt}, 2;")
    gen.emit(f"@{p_t1} bra {L_skipe};")
    eph, aeb_m = gen.register(".u32"), gen.register(".u32")
    gen.emit(f"shr.u32 {eph}, {mt}, 1;")
    gen.emit(f"sub.u32 {eph}, {eph}, 1;")
    gen.emit(f"and.b32 {eph}, {eph}, 1;")
    gen.emit(f"mad.lo.u32 {aeb_m}, {mab}, 8, {bar};")
    gen.emit(f"add.u32 {aeb_m}, {aeb_m}, {AE0};")
    wait(aeb_m, eph)
    gen.label(L_skipe)
    gen.emit("tcgen05.fence::after_thread_sync;")
    if H:                                  # a half unit multiplies N = BN/2
        ph_m = gen.register(".pred")
        gen.emit(f"setp.ge.u32 {ph_m}, {mtile}, {F};")
        gen.emit(f"selp.u32 {r_idesc}, {idesc_half}, {idesc}, {ph_m};")
    mkb = gen.register(".u32")
    gen.emit(f"mov.u32 {mkb}, 0;")
    L_mk = gen.new_label("mk")
    L_mkdone = gen.new_label("mkdone")
    pmk = gen.register(".pred")
    gen.label(L_mk)
    gen.emit(f"setp.ge.u32 {pmk}, {mkb}, {KB};")
    gen.emit(f"@{pmk} bra {L_mkdone};")
    ms, mph = gen.register(".u32"), gen.register(".u32")
    gen.emit(f"rem.u32 {ms}, {mit}, {S};")
    gen.emit(f"div.u32 {mph}, {mit}, {S};")
    gen.emit(f"and.b32 {mph}, {mph}, 1;")
    fbar = gen.register(".u32")
    gen.emit(f"mad.lo.u32 {fbar}, {ms}, 8, {bar};")
    wait(fbar, mph)
    gen.emit("tcgen05.fence::after_thread_sync;")
    sb = gen.register(".u32")
    gen.emit(f"mad.lo.u32 {sb}, {ms}, {STAGE}, {base};")
    addr_of = {}
    for nm, off in (("ahi", 0), ("alo", A_BYTES), ("bhi", 2 * A_BYTES),
                    ("blo", 2 * A_BYTES + B_BYTES)):
        r = gen.register(".u32")
        gen.emit(f"add.u32 {r}, {sb}, {off};")
        gen.emit(f"shr.u32 {r}, {r}, 4;")
        addr_of[nm] = r
    p_acc = gen.register(".pred")
    first = gen.register(".pred")
    gen.emit(f"setp.ne.u32 {first}, {mkb}, 0;")
    for ks in range(BK // 8):
        descs = {}
        for nm in ("ahi", "alo", "bhi", "blo"):
            lo = gen.register(".u32")
            # next K step of 8: A advances 32 B inside its swizzle row, B two K groups
            step = (32 >> 4) * ks if nm[0] == "a" else ((2 * SBO_B) >> 4) * ks
            low_word = a_lo_word if nm[0] == "a" else b_lo_word
            gen.emit(f"add.u32 {lo}, {addr_of[nm]}, {step + low_word};")
            d = gen.register(".b64")
            gen.emit(f"mov.b64 {d}, {{{lo}, {a_hi if nm[0] == 'a' else b_hi}}};")
            descs[nm] = d
        gen.emit(f"mov.pred {p_acc}, {first if ks == 0 else p_true};")
        gen.emit(f"@{p_el} tcgen05.mma.{CG}.kind::tf32 [{dacc}], {descs['ahi']}, "
                 f"{descs['bhi']}, {r_idesc}, {p_acc};")
        gen.emit(f"@{p_el} tcgen05.mma.{CG}.kind::tf32 [{dacc}], {descs['ahi']}, "
                 f"{descs['blo']}, {r_idesc}, {p_true};")
        gen.emit(f"@{p_el} tcgen05.mma.{CG}.kind::tf32 [{dacc}], {descs['alo']}, "
                 f"{descs['bhi']}, {r_idesc}, {p_true};")
    eoff = gen.register(".u32")                   # empty[ms], from the barrier base
    gen.emit(f"mad.lo.u32 {eoff}, {ms}, 8, {8 * S};")
    commit(eoff)
    gen.emit(f"add.u32 {mit}, {mit}, 1;")
    gen.emit(f"add.u32 {mkb}, {mkb}, 1;")
    gen.emit(f"bra.uni {L_mk};")
    gen.label(L_mkdone)
    afo = gen.register(".u32")
    gen.emit(f"mad.lo.u32 {afo}, {mab}, 8, {AF0};")
    commit(afo)
    gen.emit(f"add.u32 {mt}, {mt}, 1;")
    gen.emit(f"add.u32 {mtile}, {mtile}, {ncta};")
    gen.emit(f"bra.uni {L_mt};")
    gen.label(L_mma_done)
    # drain: wait for every MMA this thread issued before tensor memory is freed
    gen.emit(f"@{p_el} tcgen05.commit.{CG}.mbarrier::arrive::one.shared::cluster.b64 "
             f"[{DRAIN}];")
    wait(DRAIN, 0)

    # =================================== common exit ========================================
    gen.label(L_exit)
    gen.emit("tcgen05.fence::before_thread_sync;")
    if pair:
        # every thread of both CTAs: the leader's MMAs have drained and no thread of the pair
        # touches the other's shared or tensor memory after this point
        gen.emit("barrier.cluster.arrive.release;")
        gen.emit("barrier.cluster.wait.acquire;")
    else:
        gen.emit("barrier.sync 0;")
    gen.emit("tcgen05.fence::after_thread_sync;")
    L_nodealloc = gen.new_label("nodealloc")
    gen.emit(f"@!{p_mw} bra {L_nodealloc};")
    gen.emit("bar.warp.sync -1;")
    gen.emit(f"tcgen05.dealloc.{CG}.sync.aligned.b32 {tmem}, {TMEM_COLS};")
    gen.label(L_nodealloc)
    gen.emit("ret;")
    return {"BN": BN, "stages": S, "smem": place, "tiles": NTILES, "pair": pair}


def lower_contraction(gen, kernel, plan):
    return emit_contraction(gen, kernel, plan.a, plan.b, plan.c, plan.M, plan.N, plan.K,
                            plan.atomic)
