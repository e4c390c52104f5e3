"""PyTorch-CPU evaluation of the benchmark expressions. TEST AND CPU-BASELINE INFRASTRUCTURE ONLY.

The reference has no CPU execution path of its own; its problems are defined
by PyTorch expressions (reference ``tools/expressions_open.py:33-105``, the
``code`` field of ``meta.json``) and the benchmark's CPU baseline is that
expression evaluated by PyTorch on the host cores, with every core in use.
"""

from __future__ import annotations

import os
import time

import torch


def threads() -> int:
    n = os.cpu_count() or 1
    torch.set_num_threads(n)
    return torch.get_num_threads()


def reduce_inputs(n: int, seed: int = 0):
    g = torch.Generator().manual_seed(seed)
    return torch.rand(n, generator=g, dtype=torch.float32) * 2 - 1


def reduce_step(x):
    """One step of the full-reduction workload: sum and mean of x (f32)."""
    return x.sum(), x.mean()


def reduce_rate(x, seconds: float):
    """Seconds per ``reduce_step(x)``, averaged over as many back-to-back steps as fit in
    ``seconds`` (at least 3), after one untimed step. Returns (seconds per step, steps)."""
    reduce_step(x)
    t_end = time.perf_counter() + seconds
    n, t = 0, 0.0
    while time.perf_counter() < t_end or n < 3:
        t0 = time.perf_counter()
        reduce_step(x)
        t += time.perf_counter() - t0
        n += 1
    return t / n, n


def time_steps(fn, steps: int, warmup: int = 1):
    for _ in range(warmup):
        fn()
    t0 = time.perf_counter()
    for _ in range(steps):
        fn()
    return (time.perf_counter() - t0) / steps


def expression_fns(n_rows=8192, n_cols=4096, eps_rms=1e-6, eps_l2=1e-12):
    """CPU versions of every benchmark expression (same f32 math as the IR)."""
    def rmsnorm(x, w):
        return x * torch.rsqrt((x * x).mean(-1, keepdim=True) + eps_rms) * w

    def softmax(x):
        return torch.softmax(x, -1)

    def l2norm(x):
        return x / torch.clamp(x.norm(dim=-1, keepdim=True), min=eps_l2)

    return {"rmsnorm": rmsnorm, "softmax": softmax, "l2norm": l2norm,
            "add": lambda a, b: a + b, "sum": lambda x: x.sum(), "mean": lambda x: x.mean()}


def workload_baseline(name: str, inputs: dict, *, algorithmic: float, unit: str,
                      reps: int = 3) -> dict:
    """PyTorch CPU (all host cores) on one benchmark workload, for the suite's per-workload
    ``cpu_baseline``: the same f32 expression as the kernel, median of ``reps`` timed runs
    after one warm-up. ``algorithmic`` is the workload's bytes (GB/s) or FLOP (TFLOP/s) per
    launch; attention is timed on one batch entry (16 heads, 1/8 of the work) and the rate
    reported for that sample."""
    import torch.nn.functional as F
    cores = threads()
    t = {k: torch.from_numpy(v) for k, v in inputs.items()}
    scale = 1.0
    sample = "full workload"
    if name == "add":
        fn = lambda: t["x0"] + t["x1"]                                    # noqa: E731
    elif name == "sum":
        fn = lambda: t["x"].sum()                                         # noqa: E731
    elif name == "mean":
        fn = lambda: t["x"].mean()                                        # noqa: E731
    elif name in ("rmsnorm", "softmax", "l2norm"):
        f = expression_fns()[name]
        fn = (lambda: f(t["x"], t["w"])) if name == "rmsnorm" else (lambda: f(t["x"]))
    elif name.startswith("matmul"):
        fn = lambda: t["x0"] @ t["x1"]                                    # noqa: E731
    elif name.startswith("attention"):
        c = float(t["div_c1"].reshape(-1)[0])
        q, k, v = t["q"][:1], t["kt"][:1].transpose(-1, -2), t["v"][:1]
        fn = lambda: F.scaled_dot_product_attention(q, k, v, scale=1.0 / c)   # noqa: E731
        scale = 1.0 / t["q"].shape[0]
        sample = f"batch entry 0 of {t['q'].shape[0]} (16 heads)"
    else:
        raise KeyError(name)
    fn()
    times = []
    for _ in range(reps):
        t0 = time.perf_counter()
        fn()
        times.append(time.perf_counter() - t0)
    sec = sorted(times)[len(times) // 2]
    work = algorithmic * scale
    value = work / sec / (1e9 if unit == "GB/s" else 1e12)
    return {"value": round(value, 3), "unit": unit, "cores": cores, "kind": "port",
            "sample": f"torch CPU f32, {sample}, median of {reps}"}
