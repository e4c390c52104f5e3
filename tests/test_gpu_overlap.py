"""Overlapped launches (``emmy_rt_launch_ex`` with EMMY_RT_LAUNCH_OVERLAP) of the full sum and
mean kernels give the same bits as plain launches.

Each overlapped kernel may start while its predecessor on the stream is still finishing and
orders its global writes (CTA partials, the ticket, the result) behind that predecessor with
``griddepcontrol.wait``. Consecutive launches of one module share its partials and ticket, so
any ordering gap shows up as a wrong or differing result; the fold runs in CTA order, so a
correct result is bit-identical to the plain launch's.
"""

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _modules(n, grid):
    from emmyptx import runtime, workloads
    from emmyptx.emit import compile_payload
    mods = []
    for op in ("sum", "mean"):
        payload, meta = workloads.full_reduce(n, op, grid=grid)
        ptx, template, _ = compile_payload(payload, meta)
        assert template == "rowreduce"
        k = meta["kernels"][0]
        mods.append((runtime.Module(ptx, k["entry"]), k))
    return mods


@pytest.mark.parametrize("n,grid", [(1 << 22, 592), (1 << 20 | 12345, 148), ((1 << 24) + 4, 1184)])
def test_overlapped_sum_mean_match_plain_launches(n, grid):
    from emmyptx import runtime
    runtime.init(0)
    rng = np.random.default_rng(n)
    x = rng.uniform(-1, 1, n).astype(np.float32)
    xb = runtime.DeviceBuffer.from_array(x)
    cb = runtime.DeviceBuffer.from_array(np.array([float(n)], np.float32))
    reps = 20
    out = runtime.DeviceBuffer(4 * 2 * (reps + 1))
    out.zero()
    (ms, ks), (mm, km) = _modules(n, grid)
    assert [a["name"] for a in km["args"]] == ["x", "mean_keepdim_count", "mean"]
    # slot 0: plain launches; slots 1..reps: back-to-back overlapped launches
    ms.launch(ks["grid"], ks["block"], 0, [xb.ptr, out.ptr])
    mm.launch(km["grid"], km["block"], 0, [xb.ptr, cb.ptr, out.ptr + 4])
    for r in range(1, reps + 1):
        ms.launch(ks["grid"], ks["block"], 0, [xb.ptr, out.ptr + 8 * r], overlap=True)
        mm.launch(km["grid"], km["block"], 0, [xb.ptr, cb.ptr, out.ptr + 8 * r + 4],
                  overlap=True)
    runtime.sync()
    got = np.zeros(2 * (reps + 1), np.float32)
    out.download(got)
    got = got.reshape(reps + 1, 2)
    assert ms.error_word() == 0 and mm.error_word() == 0
    want = x.astype(np.float64).sum()
    assert abs(float(got[0, 0]) - want) <= 1e-5 * max(abs(want), 1.0) + 1e-5 * n ** 0.5
    assert abs(float(got[0, 1]) - want / n) <= 1e-5 * max(abs(want / n), 1e-3)
    for r in range(1, reps + 1):
        assert got[r].tobytes() == got[0].tobytes(), (r, got[r], got[0])
    ms.close()
    mm.close()


def test_overlapped_pointwise_chain_stays_ordered():
    """A chain of overlapped pointwise launches where each kernel reads what the previous one
    wrote: y_(i+1) = y_i + b for 24 launches. The pointwise kernel waits for its predecessor
    (``griddepcontrol.wait``) before its first global access, so every step sees the finished
    previous result; a missing wait would read a stale or half-written y and break the
    bit-exact match with the same additions done in numpy float32."""
    from emmyptx import runtime, workloads
    from emmyptx.emit import compile_payload
    runtime.init(0)
    n = (1 << 22) + 12
    payload, meta = workloads.pointwise_add(n)
    ptx, template, _ = compile_payload(payload, meta)
    assert template == "pointwise" and "griddepcontrol.wait" in ptx
    k = meta["kernels"][0]
    assert [a["name"] for a in k["args"]] == ["x0", "x1", "add"]
    rng = np.random.default_rng(5)
    a = rng.standard_normal(n).astype(np.float32)
    b = rng.standard_normal(n).astype(np.float32)
    steps = 24
    ys = [runtime.DeviceBuffer.from_array(a)] + [runtime.DeviceBuffer(4 * n) for _ in range(2)]
    bb = runtime.DeviceBuffer.from_array(b)
    mod = runtime.Module(ptx, k["entry"])
    src = 0
    for i in range(steps):
        dst = 1 + (i % 2)
        mod.launch(k["grid"], k["block"], 0, [ys[src].ptr, bb.ptr, ys[dst].ptr], overlap=True)
        src = dst
    runtime.sync()
    got = ys[src].download(np.zeros(n, np.float32))
    want = a.copy()
    for _ in range(steps):
        want = want + b
    assert mod.error_word() == 0
    assert np.array_equal(got, want)
    mod.close()
    for buf in ys + [bb]:
        buf.free()


@pytest.mark.parametrize("op", ["softmax", "rmsnorm"])
def test_overlapped_row_chain_stays_ordered(op):
    """A chain of overlapped row-kernel launches, each reading the rows the previous one
    wrote (12 launches over 2048 x 4096). The row kernels wait for their predecessor
    (``griddepcontrol.wait``) before any global access, so the chain gives the bits of the
    same launches made one after another without overlap."""
    from emmyptx import runtime, workloads
    from emmyptx.emit import compile_payload
    from oracle.expressions import kernel_inputs
    runtime.init(0)
    payload, meta = workloads.row_op(op, rows=2048)
    ptx, template, _ = compile_payload(payload, meta)
    assert template == "rowreduce" and "griddepcontrol.wait" in ptx
    k = meta["kernels"][0]
    inputs = kernel_inputs(k)
    out = next(a for a in k["args"] if a.get("output"))
    x_name = next(a["name"] for a in k["args"]
                  if not a.get("output") and a["shape"] == out["shape"])
    others = [a["name"] for a in k["args"] if a["name"] not in (x_name, out["name"])]
    steps = 12

    def chain(overlap):
        bufs = {n: runtime.DeviceBuffer.from_array(inputs[n]) for n in others}
        ys = [runtime.DeviceBuffer.from_array(inputs[x_name])] + [
            runtime.DeviceBuffer(inputs[x_name].nbytes) for _ in range(2)]
        mod = runtime.Module(ptx, k["entry"])
        src = 0
        for i in range(steps):
            dst = 1 + (i % 2)
            where = {x_name: ys[src].ptr, out["name"]: ys[dst].ptr}
            where.update({n: b.ptr for n, b in bufs.items()})
            ptrs = [where[a["name"]] for a in k["args"]]
            mod.launch(k["grid"], k["block"], k.get("smem_bytes", 0), ptrs, overlap=overlap)
            src = dst
        runtime.sync()
        got = ys[src].download(np.zeros_like(inputs[x_name]))
        assert mod.error_word() == 0
        mod.close()
        for b in list(bufs.values()) + ys:
            b.free()
        return got

    plain, overlapped = chain(False), chain(True)
    assert np.all(np.isfinite(plain))
    assert np.array_equal(plain.view(np.uint32), overlapped.view(np.uint32))
