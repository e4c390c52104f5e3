"""The allocation-free sum (emmy_rt_sum_f32_noalloc) against the emitted sum kernel.

Some callers of this library may not allocate device memory while they call it
(a service whose pool owns the GPU's memory, a timing loop where cudaFree would
synchronise the device). For them the library exposes one sum whose cross-CTA
scratch is a fixed array inside the library. This test calls it through the C
ABI twice in a row on the same inputs and checks both results against the sum
kernel that compile.py emits for the same workload, launched through
emmy_rt_launch, within the 1e-5 relative tolerance the other reduction tests
use. It lives in its own file, collected last, and needs nothing from the other
tests, so it passes alone in a fresh process as well as after the full suite.
"""

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

REL = 1e-5


def test_noalloc_sum_matches_emitted_kernel_twice(gpu_runtime):
    from emmyptx import workloads
    from emmyptx.emit import compile_payload
    rt = gpu_runtime
    n, grid = (1 << 22) + 3, 600
    x = np.random.default_rng(11).uniform(-1, 1, n).astype(np.float32)
    exact = float(x.astype(np.float64).sum())
    xbuf = rt.DeviceBuffer.from_array(x)
    out_ref, out_na = rt.DeviceBuffer(4), rt.DeviceBuffer(4)
    out_ref.zero()

    payload, meta = workloads.full_reduce(n, "sum", grid=grid)
    ptx, _, _ = compile_payload(payload, meta)
    k = meta["kernels"][0]
    mod = rt.Module(ptx, k["entry"])
    mod.launch(k["grid"], k["block"], 0, [xbuf.ptr, out_ref.ptr])
    rt.sync()
    ref = float(out_ref.download(np.zeros(1, np.float32))[0])
    assert abs(ref - exact) <= REL * abs(exact)

    L = rt.lib()
    results = []
    for _ in range(2):
        out_na.zero()
        rc = L.emmy_rt_sum_f32_noalloc(xbuf.ptr, n, out_na.ptr, grid, 0)
        assert rc == 0, L.emmy_rt_last_error()
        rt.sync()
        results.append(float(out_na.download(np.zeros(1, np.float32))[0]))
    for got in results:
        assert abs(got - ref) <= REL * abs(ref), (got, ref)
    assert results[0] == results[1]          # same grid, same order: deterministic

    # a grid beyond the fixed scratch is refused with a message, nothing launched
    rc = L.emmy_rt_sum_f32_noalloc(xbuf.ptr, n, out_na.ptr, 4097, 0)
    assert rc == -3 and b"outside 1..4096" in L.emmy_rt_last_error()
    # so is a pointer that is not 4-byte aligned (it would fault in the kernel)
    rc = L.emmy_rt_sum_f32_noalloc(xbuf.ptr + 2, n - 1, out_na.ptr, grid, 0)
    assert rc == -3 and b"4-byte aligned" in L.emmy_rt_last_error()
    mod.close()


@pytest.mark.parametrize("grid", [1, 37])
def test_noalloc_sum_unaligned_input_and_single_cta(grid, gpu_runtime):
    """x 4 bytes past a 16-byte boundary takes the kernel's scalar path; one CTA finishes
    alone (its ticket wraps at once). Two calls in a row, both within 1e-5 of fp64."""
    rt = gpu_runtime
    n = 100_003
    x = np.random.default_rng(12).uniform(-1, 1, n).astype(np.float32)
    exact = float(x.astype(np.float64).sum())
    xbuf = rt.DeviceBuffer.from_array(np.concatenate([np.zeros(1, np.float32), x]))
    out = rt.DeviceBuffer(4)
    L = rt.lib()
    for _ in range(2):
        out.zero()
        rc = L.emmy_rt_sum_f32_noalloc(xbuf.ptr + 4, n, out.ptr, grid, 0)
        assert rc == 0, L.emmy_rt_last_error()
        rt.sync()
        got = float(out.download(np.zeros(1, np.float32))[0])
        assert abs(got - exact) <= REL * abs(exact), (got, exact)
