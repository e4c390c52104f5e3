"""The cross-GPU fold (emmy_rt_fold_f32) on one GPU, and on two GPUs when the box has them.

On one GPU the other ranks are emulated without a second kernel: their mailbox entries are
written by the host before the launch (a flag that is already up), so the only kernel that
waits is this rank's, and it waits on nothing another kernel must set. The bounded wait is
exercised with a flag that nothing sets: the kernel gives up after about a second, sets the
error word and leaves the output untouched, and the context stays usable.
With two or more GPUs, two processes (one per GPU) exchange mailbox handles over a gloo
group and fold through peer stores; each must get the same bits, the rank-order sum.
"""

import os
import socket
import time

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

OVERLAP = 1
SENTINEL = np.float32(-12345.0)


def _entry_bytes(vals, epoch):
    e = np.zeros(8, np.uint32)
    e[:4] = np.frombuffer(np.array(list(vals) + [0.0] * (4 - len(vals)), np.float32).tobytes(),
                          np.uint32)
    e[4] = epoch
    return e


class _Fold:
    """Buffers for one emulated rank: its mailbox and the other ranks' mailboxes (all local)."""

    def __init__(self, rt, world):
        from emmyptx.fold import box_bytes
        self.rt, self.world = rt, world
        self.boxes = [rt.DeviceBuffer(box_bytes(world)) for _ in range(world)]
        for b in self.boxes:
            b.zero()
        self.ptrs = rt.DeviceBuffer.from_array(np.array([b.ptr for b in self.boxes], np.uint64))
        self.vals = rt.DeviceBuffer(16)
        self.out = rt.DeviceBuffer(16)
        self.err = rt.DeviceBuffer(4)
        self.err.zero()

    def box_words(self, r):
        return self.boxes[r].download(np.zeros(16 * self.world, np.uint32)).reshape(-1, 8)

    def plant(self, r_box, sender, vals, epoch):
        """Host-side: rank `sender`'s entry for `epoch`, flag up, in mailbox `r_box`."""
        words = self.box_words(r_box)
        words[(epoch & 1) * self.world + sender] = _entry_bytes(vals, epoch)
        self.boxes[r_box].upload(words.reshape(-1))

    def run(self, rank, vals, epoch, flags=0, nvals=None):
        nv = len(vals) if nvals is None else nvals
        self.vals.upload(np.array(list(vals) + [0.0] * (4 - len(vals)), np.float32))
        self.out.upload(np.full(4, SENTINEL, np.float32))
        L = self.rt.lib()
        rc = L.emmy_rt_fold_f32(self.vals.ptr, nv, self.ptrs.ptr, rank, self.world, epoch,
                                self.out.ptr, self.err.ptr, 0, flags)
        assert rc == 0, L.emmy_rt_last_error()
        self.rt.sync()
        return self.out.download(np.zeros(4, np.float32))

    def error(self):
        return int(self.err.download(np.zeros(1, np.uint32))[0])

    def free(self):
        for b in self.boxes + [self.ptrs, self.vals, self.out, self.err]:
            b.free()


def test_fold_single_rank_is_identity(gpu_runtime):
    f = _Fold(gpu_runtime, 1)
    rng = np.random.default_rng(3)
    for epoch in range(1, 6):
        v = rng.standard_normal(4).astype(np.float32)
        out = f.run(0, v, epoch, flags=OVERLAP if epoch % 2 else 0)
        assert out.tobytes() == v.tobytes()
    out = f.run(0, [1.5, 2.5], 6)
    assert out[:2].tolist() == [1.5, 2.5] and out[2] == SENTINEL and out[3] == SENTINEL
    assert f.error() == 0
    f.free()


@pytest.mark.parametrize("world,rank", [(2, 0), (2, 1), (4, 2), (8, 7)])
def test_fold_emulated_ranks_rank_order_sum(gpu_runtime, world, rank):
    f = _Fold(gpu_runtime, world)
    rng = np.random.default_rng(world * 10 + rank)
    for epoch in range(1, 5):                       # both entry sets, twice
        vals = rng.standard_normal((world, 2)).astype(np.float32) * 1e3
        for s in range(world):
            if s != rank:
                f.plant(rank, s, vals[s], epoch)
        out = f.run(rank, vals[rank], epoch)
        want = np.zeros(2, np.float32)
        for s in range(world):                      # rank order, f32 adds from zero
            want = (want + vals[s]).astype(np.float32)
        assert out[:2].tobytes() == want.tobytes(), (epoch, out, want)
        # this rank's entry, with its flag, went into every mailbox of this epoch's set
        for r in range(world):
            e = f.box_words(r)[(epoch & 1) * world + rank]
            assert e[4] == epoch
            assert e[:2].tobytes() == vals[rank].tobytes()
    assert f.error() == 0
    f.free()


def test_fold_wait_is_bounded(gpu_runtime):
    """Rank 1 never arrives: the kernel returns after about a second with bit 0 set."""
    f = _Fold(gpu_runtime, 2)
    t0 = time.perf_counter()
    out = f.run(0, [1.0, 2.0], 1)
    dt = time.perf_counter() - t0
    assert f.error() == 1
    assert np.all(out == SENTINEL)
    assert 0.5 < dt < 10.0, dt
    # while the error word is set, a call returns at once without writing out
    f.plant(0, 1, [3.0, 4.0], 2)
    t0 = time.perf_counter()
    out = f.run(0, [1.0, 2.0], 2)
    assert np.all(out == SENTINEL) and time.perf_counter() - t0 < 0.5 and f.error() == 1
    # the context is still usable: cleared, the same epoch with rank 1's entry planted completes
    f.err.zero()
    f.plant(0, 1, [3.0, 4.0], 2)
    out = f.run(0, [1.0, 2.0], 2)
    assert out[:2].tolist() == [4.0, 6.0] and f.error() == 0
    f.free()


def test_fold_overlapped_behind_emitted_sum(gpu_runtime):
    """Overlapped behind the emitted sum kernel, the fold reads the sum's result only after
    the sum completed (griddepcontrol.wait)."""
    from emmyptx import workloads
    from emmyptx.emit import compile_payload
    rt = gpu_runtime
    n = (1 << 24) + 5
    x = np.random.default_rng(5).uniform(-1, 1, n).astype(np.float32)
    xb = rt.DeviceBuffer.from_array(x)
    payload, meta = workloads.full_reduce(n, "sum", grid=592)
    ptx, _, _ = compile_payload(payload, meta)
    k = meta["kernels"][0]
    mod = rt.Module(ptx, k["entry"])
    f = _Fold(rt, 1)
    L = rt.lib()
    outs = []
    for epoch in range(1, 9):
        f.vals.upload(np.zeros(4, np.float32))
        f.out.upload(np.full(4, SENTINEL, np.float32))
        mod.launch(k["grid"], k["block"], 0, [xb.ptr, f.vals.ptr], overlap=True)
        rc = L.emmy_rt_fold_f32(f.vals.ptr, 1, f.ptrs.ptr, 0, 1, epoch, f.out.ptr, f.err.ptr,
                                0, OVERLAP)
        assert rc == 0, L.emmy_rt_last_error()
        rt.sync()
        outs.append(float(f.out.download(np.zeros(4, np.float32))[0]))
    want = float(x.astype(np.float64).sum())
    assert abs(outs[0] - want) <= 1e-5 * abs(want) + 1e-5 * n ** 0.5
    assert len(set(outs)) == 1
    assert mod.error_word() == 0 and f.error() == 0
    mod.close()
    f.free()
    xb.free()


def test_fold_on_its_own_stream_behind_the_reductions(gpu_runtime):
    """The benchmark's exchange pattern: overlapped sum -> mean launches on one stream, each
    step's fold on a second stream after an event recorded behind that step's mean, every step
    writing its own result slot. Each folded pair equals the pair the kernels wrote (so no fold
    read a slot before its mean completed), and the sum matches fp64."""
    import torch
    from emmyptx import workloads
    from emmyptx.emit import compile_payload
    rt = gpu_runtime
    dev = torch.device("cuda", 0)
    n = (1 << 22) + 3
    g = torch.Generator(device=dev).manual_seed(3)
    x = torch.empty(n, device=dev, dtype=torch.float32).uniform_(-1, 1, generator=g)
    cnt = torch.tensor([float(n)], device=dev, dtype=torch.float32)
    mods = []
    for op in ("sum", "mean"):
        payload, meta = workloads.full_reduce(n, op, grid=592)
        ptx, _, _ = compile_payload(payload, meta)
        k = meta["kernels"][0]
        mods.append((rt.Module(ptx, k["entry"]), k))
    (ms, ks), (mm, km) = mods
    assert [a["name"] for a in km["args"]] == ["x", "mean_keepdim_count", "mean"]
    f = _Fold(rt, 1)
    L = rt.lib()
    steps = 12
    res = torch.zeros(steps, 2, device=dev, dtype=torch.float32)
    tot = torch.full((steps, 2), float(SENTINEL), device=dev, dtype=torch.float32)
    main, side = torch.cuda.Stream(device=dev), torch.cuda.Stream(device=dev)
    evs = [torch.cuda.Event() for _ in range(steps)]
    torch.cuda.synchronize()
    for i in range(steps):
        ms.launch(ks["grid"], ks["block"], 0, [x.data_ptr(), res[i].data_ptr()],
                  main.cuda_stream, overlap=i > 0)
        mm.launch(km["grid"], km["block"], 0, [x.data_ptr(), cnt.data_ptr(), res[i].data_ptr() + 4],
                  main.cuda_stream, overlap=True)
        evs[i].record(main)
        side.wait_event(evs[i])
        rc = L.emmy_rt_fold_f32(res[i].data_ptr(), 2, f.ptrs.ptr, 0, 1, i + 1, tot[i].data_ptr(),
                                f.err.ptr, side.cuda_stream, 0)
        assert rc == 0, L.emmy_rt_last_error()
    torch.cuda.synchronize()
    got, wrote = tot.cpu().numpy(), res.cpu().numpy()
    assert np.array_equal(got, wrote)
    assert np.all(got == got[0])
    want = float(x.double().sum())
    assert abs(float(got[0, 0]) - want) <= 1e-5 * abs(want) + 1e-5 * n ** 0.5
    assert abs(float(got[0, 1]) - want / n) <= 1e-5 * abs(want / n) + 1e-5 / n ** 0.5
    assert ms.error_word() == 0 and mm.error_word() == 0 and f.error() == 0
    ms.close()
    mm.close()
    f.free()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _two_gpu_worker(rank, world, port, q):
    import datetime

    import torch.distributed as dist
    from emmyptx import runtime
    from emmyptx.fold import PeerFold
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60))
    try:
        runtime.init(rank)

        def gather(obj):
            out = [None] * world
            dist.all_gather_object(out, obj)
            return out
        fold = PeerFold(rank, world, gather)
        vals = runtime.DeviceBuffer(8)
        out = runtime.DeviceBuffer(8)
        got = []
        rng = np.random.default_rng(99)
        table = rng.standard_normal((20, world, 2)).astype(np.float32)
        for step in range(20):
            vals.upload(table[step, rank])
            fold.launch(vals.ptr, 2, out.ptr, 0, overlap=bool(step % 2))
            runtime.sync()
            got.append(out.download(np.zeros(2, np.float32)).tobytes())
        err = fold.error_word()
        dist.barrier()              # no rank unmaps a mailbox a peer may still write
        fold.close()
        want = []
        for step in range(20):
            acc = np.zeros(2, np.float32)
            for s in range(world):
                acc = (acc + table[step, s]).astype(np.float32)
            want.append(acc.tobytes())
        q.put((rank, err, got == want))
    finally:
        dist.destroy_process_group()


def test_fold_two_gpus_peer_stores():
    import torch
    import torch.multiprocessing as mp
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_two_gpu_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=180)
    res = sorted(q.get(timeout=5) for _ in range(2))
    assert [r[1] for r in res] == [0, 0], res
    assert all(r[2] for r in res), res
    assert all(p.exitcode == 0 for p in procs)
