"""TMA-fed attention on B200: tiles copied by ``cp.async.bulk.tensor`` through tensor maps that
libemmyrt writes at launch time, against the register-staged loads of the same kernel.

The TMA path leaves each raw f32 tile in shared memory as the TF32 hi operand and writes only
the lo part, where the register path writes ``x & 0xFFFFE000`` and the lo part; the products
are the same, so the two paths must agree bit for bit. ``emmy_path`` shows which path the
CTAs took (bit 0 TMA, bit 1 registers)."""

import numpy as np
import pytest

import tolerance as tol

pytestmark = pytest.mark.gpu

TMA, REGS = 1, 2


class _Launch:
    """One compiled attention kernel with device buffers for its arguments."""

    def __init__(self, runtime, payload, meta, grid=None):
        from emmyptx.emit import compile_payload
        from oracle.expressions import kernel_inputs
        self.rt = runtime
        k = dict(meta["kernels"][0])
        if grid is not None:
            k["grid"] = [grid, 1, 1]
            meta = dict(meta, kernels=[k])
        ptx, used, _ = compile_payload(payload, meta)
        assert used == "attention"
        self.k = k
        self.inputs = kernel_inputs(k)
        self.mod = runtime.Module(ptx, k["entry"])
        self.bufs, self.out = {}, None
        for a in k["args"]:
            if a.get("output"):
                self.out = np.zeros(a["shape"], np.float32)
                self.bufs[a["name"]] = runtime.DeviceBuffer(self.out.nbytes)
                self.out_name = a["name"]
            else:
                self.bufs[a["name"]] = runtime.DeviceBuffer.from_array(self.inputs[a["name"]])

    def __call__(self, **override):
        bufs = dict(self.bufs, **override)
        bufs[self.out_name].zero()
        ptrs = [bufs[a["name"]].ptr for a in self.k["args"]]
        self.mod.path_word(clear=True)
        self.mod.launch(self.k["grid"], self.k["block"], self.k["smem_bytes"], ptrs)
        self.rt.sync()
        assert self.mod.error_word() == 0
        return bufs[self.out_name].download(np.empty_like(self.out)), self.mod.path_word()

    def close(self):
        for b in self.bufs.values():
            b.free()
        self.mod.close()


def _both_paths(runtime, payload, meta, grid=None):
    run = _Launch(runtime, payload, meta, grid)
    try:
        assert run.mod.tensor_maps()["maps"] == 2
        got_tma, path = run()
        assert path == TMA, f"emmy_path {path:#x}: the CTAs did not all take the TMA path"
        assert run.mod.tensor_maps()["uploads"] == 1
        run.mod.tensor_maps(enable=False)
        got_regs, path = run()
        assert path == REGS, f"emmy_path {path:#x} with the maps switched off"
        return run.inputs, got_tma, got_regs
    finally:
        run.close()


@pytest.mark.parametrize("name", ["attention_d64", "attention_d128"])
def test_tma_matches_register_path_full_size(name, gpu_runtime):
    """[8,16,2048,D]: the TMA path's output equals the register path's bit for bit."""
    from emmyptx import workloads
    payload, meta = workloads.WORKLOADS[name]()
    _, got_tma, got_regs = _both_paths(gpu_runtime, payload, meta)
    assert np.all(np.isfinite(got_tma))
    diff = np.count_nonzero(got_tma.view(np.uint32) != got_regs.view(np.uint32))
    assert diff == 0, f"{diff} of {got_tma.size} outputs differ between the paths"


@pytest.mark.parametrize("shape,grid", [((1, 2, 256, 128, None), None),
                                        ((2, 1, 384, 64, None), None),
                                        ((1, 1, 512, 128, 0.25), None),
                                        ((2, 2, 384, 128, None), 5),
                                        ((1, 3, 128, 64, None), 1),
                                        ((2, 2, 512, 32, None), None),
                                        ((1, 3, 384, 32, 0.25), 2),
                                        ((2, 2, 512, 96, None), None),
                                        ((1, 2, 384, 96, 0.25), 3)],
                         ids=["d128", "d64", "d128-peaked", "d128-grid5", "d64-grid1", "d32",
                              "d32-peaked-grid2", "d96", "d96-peaked-grid3"])
def test_tma_matches_register_path_small(shape, grid, gpu_runtime):
    """Small shapes (two to eight key blocks; several work items per CTA): bit-equal paths,
    and the TMA result within 1e-4 of fp64 (row-scaled, as the other attention checks)."""
    from emmyptx import workloads
    from oracle.expressions import _attention
    B, H, S, D, c = shape
    payload, meta = workloads.attention(B, H, S, D, scale=c, stages=2 if D == 96 else 3)
    inputs, got_tma, got_regs = _both_paths(gpu_runtime, payload, meta, grid)
    assert np.array_equal(got_tma.view(np.uint32), got_regs.view(np.uint32))
    cc = float(inputs["div_c1"][0])
    want = np.stack([_attention(inputs["q"][b, h], inputs["kt"][b, h], inputs["v"][b, h], cc)
                     for b in range(B) for h in range(H)]).reshape(got_tma.shape)
    ok, err = tol.rowscaled(got_tma, want, 1e-4, label="attention TMA path")
    assert ok, f"relative error {err:.3e}"


def test_maps_follow_the_pointers(gpu_runtime):
    """New kt / v buffers re-encode the maps before the launch; going back re-encodes them
    again and reproduces the first result."""
    from emmyptx import workloads
    payload, meta = workloads.attention(1, 2, 512, 64)
    run = _Launch(gpu_runtime, payload, meta)
    rng = np.random.default_rng(7)
    other = {n: gpu_runtime.DeviceBuffer.from_array(
                 rng.standard_normal(run.inputs[n].shape).astype(np.float32))
             for n in ("kt", "v")}
    try:
        first, p1 = run()
        second, p2 = run(**other)
        again, p3 = run()
        assert (p1, p2, p3) == (TMA, TMA, TMA)
        assert run.mod.tensor_maps()["uploads"] == 3
        assert np.array_equal(first.view(np.uint32), again.view(np.uint32))
        assert not np.array_equal(first, second)
        run.mod.tensor_maps(enable=False)
        regs, p4 = run(**other)
        assert p4 == REGS
        assert np.array_equal(second.view(np.uint32), regs.view(np.uint32))
    finally:
        for b in other.values():
            b.free()
        run.close()


def test_runner_path_takes_tma(gpu_runtime):
    """``emmy_rt_run`` (host buffers, the reference runner's semantics) writes the maps too."""
    from emmyptx import workloads
    from emmyptx.emit import compile_payload
    from oracle.expressions import kernel_inputs
    payload, meta = workloads.attention(1, 1, 256, 128)
    k = meta["kernels"][0]
    ptx, _, _ = compile_payload(payload, meta)
    mod = gpu_runtime.Module(ptx, k["entry"])
    try:
        inputs = kernel_inputs(k)
        host = []
        for a in k["args"]:
            if a.get("output"):
                out = np.zeros(a["shape"], np.float32)
                host.append((out, True, False))
            else:
                host.append((np.ascontiguousarray(inputs[a["name"]]), False, False))
        mod.run(k["grid"], k["block"], k["smem_bytes"], host, warmup=1, iters=2)
        assert mod.error_word() == 0
        assert mod.path_word() == TMA
        assert mod.tensor_maps()["uploads"] == 1
    finally:
        mod.close()


def test_runner_repeated_calls(gpu_runtime):
    """Many ``emmy_rt_run`` calls on one module, each with buffers and a stream of its own:
    every call writes the maps it needs (after the earlier calls' launches), takes the TMA path
    and gives the same bits."""
    from emmyptx import workloads
    from emmyptx.emit import compile_payload
    from oracle.expressions import kernel_inputs
    payload, meta = workloads.attention(1, 2, 256, 64)
    k = meta["kernels"][0]
    ptx, _, _ = compile_payload(payload, meta)
    mod = gpu_runtime.Module(ptx, k["entry"])
    inputs = kernel_inputs(k)
    results = []
    try:
        for _ in range(12):
            host = []
            for a in k["args"]:
                if a.get("output"):
                    out = np.zeros(a["shape"], np.float32)
                    host.append((out, True, False))
                else:
                    host.append((np.ascontiguousarray(inputs[a["name"]]), False, False))
            mod.path_word(clear=True)
            mod.run(k["grid"], k["block"], k["smem_bytes"], host, warmup=0, iters=1)
            assert mod.error_word() == 0 and mod.path_word() == TMA
            results.append(out.copy())
        assert mod.tensor_maps()["uploads"] >= 1
        for r in results[1:]:
            assert np.array_equal(r.view(np.uint32), results[0].view(np.uint32))
    finally:
        mod.close()
