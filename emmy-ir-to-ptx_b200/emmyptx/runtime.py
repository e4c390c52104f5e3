"""ctypes binding of ``libemmyrt.so`` (C ABI in ``include/emmy_rt.h``).

This is the in-process replacement of the reference harness's remote runner
(reference ``submit.py:99-137``, ``docs/API.md:14-56``): PTX is JIT-loaded
with ``cuModuleLoadDataEx`` and launched with ``cuLaunchKernel`` under the
grid/block/shared bytes of ``meta.json``. There is no CPU fallback: if the
library or the driver is missing, every call raises :class:`RuntimeError`.
"""

from __future__ import annotations

import ctypes
from pathlib import Path

import numpy as np

LIB_NAME = "libemmyrt.so"
_HERE = Path(__file__).resolve().parent

EMMY_RT_ENOTFOUND = -4


class RuntimeErrorEmmy(RuntimeError):
    def __init__(self, code, msg):
        super().__init__(f"emmy_rt error {code}: {msg}")
        self.code = code


class _Arg(ctypes.Structure):
    _fields_ = [("host", ctypes.c_void_p), ("bytes", ctypes.c_uint64),
                ("is_output", ctypes.c_int32), ("zero_each", ctypes.c_int32)]


class _Stats(ctypes.Structure):
    _fields_ = [("kernel_us_median", ctypes.c_float), ("e2e_us_median", ctypes.c_float),
                ("h2d_bytes", ctypes.c_uint64), ("d2h_bytes", ctypes.c_uint64),
                ("iters", ctypes.c_int32)]


_U32x3 = ctypes.c_uint32 * 3
LAUNCH_OVERLAP = 1        # EMMY_RT_LAUNCH_OVERLAP
_lib = None


def library_path() -> Path:
    return _HERE / LIB_NAME


def lib():
    """Load ``libemmyrt.so`` once; raises if it was not built."""
    global _lib
    if _lib is not None:
        return _lib
    path = library_path()
    if not path.is_file():
        raise RuntimeError(f"{path} is missing: build it first (python __graft_entry__.py build)")
    L = ctypes.CDLL(str(path))
    c = ctypes
    sig = {
        "emmy_rt_abi_version": ([], c.c_int),
        "emmy_rt_last_error": ([], c.c_char_p),
        "emmy_rt_init": ([c.c_int], c.c_int),
        "emmy_rt_device_info": ([c.c_int, c.POINTER(c.c_int), c.POINTER(c.c_int),
                                 c.POINTER(c.c_int), c.POINTER(c.c_int), c.POINTER(c.c_int),
                                 c.c_char_p, c.c_size_t], c.c_int),
        "emmy_rt_module_load": ([c.c_char_p, c.c_char_p, c.POINTER(c.c_void_p), c.c_char_p,
                                 c.c_size_t], c.c_int),
        "emmy_rt_module_unload": ([c.c_void_p], c.c_int),
        "emmy_rt_module_attrs": ([c.c_void_p, c.POINTER(c.c_int), c.POINTER(c.c_int),
                                  c.POINTER(c.c_int)], c.c_int),
        "emmy_rt_module_error_word": ([c.c_void_p, c.POINTER(c.c_uint32), c.c_int], c.c_int),
        "emmy_rt_module_global": ([c.c_void_p, c.c_char_p, c.POINTER(c.c_uint64),
                                   c.POINTER(c.c_uint64)], c.c_int),
        "emmy_rt_module_tensor_maps": ([c.c_void_p, c.c_int, c.POINTER(c.c_int),
                                        c.POINTER(c.c_uint64)], c.c_int),
        "emmy_rt_launch": ([c.c_void_p, _U32x3, _U32x3, c.c_uint32, c.POINTER(c.c_uint64),
                            c.c_int, c.c_uint64], c.c_int),
        "emmy_rt_launch_ex": ([c.c_void_p, _U32x3, _U32x3, c.c_uint32, c.POINTER(c.c_uint64),
                               c.c_int, c.c_uint64, c.c_uint32], c.c_int),
        "emmy_rt_sync": ([c.c_uint64, c.c_int], c.c_int),
        "emmy_rt_time": ([c.c_void_p, _U32x3, _U32x3, c.c_uint32, c.POINTER(c.c_uint64), c.c_int,
                          c.c_uint64, c.c_int, c.c_int, c.c_uint64, c.c_uint64,
                          c.POINTER(c.c_float)], c.c_int),
        "emmy_rt_run": ([c.c_void_p, _U32x3, _U32x3, c.c_uint32, c.POINTER(_Arg), c.c_int, c.c_int,
                         c.c_int, c.POINTER(_Stats)], c.c_int),
        "emmy_rt_mem_alloc": ([c.c_uint64, c.POINTER(c.c_uint64)], c.c_int),
        "emmy_rt_mem_free": ([c.c_uint64], c.c_int),
        "emmy_rt_memcpy_htod": ([c.c_uint64, c.c_void_p, c.c_uint64], c.c_int),
        "emmy_rt_memcpy_dtoh": ([c.c_void_p, c.c_uint64, c.c_uint64], c.c_int),
        "emmy_rt_memset_zero": ([c.c_uint64, c.c_uint64], c.c_int),
        "emmy_rt_host_alloc": ([c.c_uint64, c.POINTER(c.c_void_p)], c.c_int),
        "emmy_rt_host_free": ([c.c_void_p], c.c_int),
        "emmy_rt_sum_f32_noalloc": ([c.c_uint64, c.c_uint64, c.c_uint64, c.c_uint32, c.c_uint64],
                                    c.c_int),
        "emmy_rt_fold_f32": ([c.c_uint64, c.c_uint32, c.c_uint64, c.c_uint32, c.c_uint32,
                              c.c_uint32, c.c_uint64, c.c_uint64, c.c_uint64, c.c_uint32], c.c_int),
        "emmy_rt_ipc_handle": ([c.c_uint64, c.c_void_p], c.c_int),
        "emmy_rt_ipc_open": ([c.c_void_p, c.POINTER(c.c_uint64)], c.c_int),
        "emmy_rt_ipc_close": ([c.c_uint64], c.c_int),
    }
    for name, (argtypes, restype) in sig.items():
        fn = getattr(L, name)
        fn.argtypes = argtypes
        fn.restype = restype
    _lib = L
    return L


def exported_symbols():
    """Entry points the header declares (checked against the built library in tests)."""
    import re
    text = (_HERE.parents[1] / "include" / "emmy_rt.h").read_text()
    return sorted(set(re.findall(r"\b(emmy_rt_\w+)\s*\(", text)))


def check(rc):
    if rc != 0:
        msg = lib().emmy_rt_last_error().decode(errors="replace")
        raise RuntimeErrorEmmy(rc, msg)


_initialised = set()


def init(device: int | None = None):
    """Make ``device``'s primary context current (once per device). Without a device: keep
    the device this process already initialised (a rank bound to GPU k stays on GPU k), or
    initialise device 0."""
    if device is None:
        if _initialised:
            return
        device = 0
    if device not in _initialised:
        check(lib().emmy_rt_init(device))
        _initialised.add(device)
        _note_sm_count(device)


B200_SM_COUNT = 148


def _note_sm_count(device: int):
    """The emitted PTX sizes some work splits for B200's 148 SMs (the matmul's working CTA
    pairs, the benchmark's default reduction grid of 4 CTAs per SM). Every kernel stays
    correct on another SM count (all walk their work grid-stride), but the split is then not
    the tuned one: say so once per device instead of silently running it."""
    try:
        sm = device_info(device)["sm_count"]
    except RuntimeError:
        return
    if sm != B200_SM_COUNT:
        import warnings
        warnings.warn(f"device {device} has {sm} SMs; the emitted kernels' work splits are "
                      f"sized for B200's {B200_SM_COUNT} (results stay correct, the split is "
                      "not the tuned one)", RuntimeWarning, stacklevel=3)


def device_info(device: int = 0) -> dict:
    vals = [ctypes.c_int() for _ in range(5)]
    name = ctypes.create_string_buffer(256)
    check(lib().emmy_rt_device_info(device, *[ctypes.byref(v) for v in vals], name, 256))
    sm, ccM, ccm, l2, smem = (v.value for v in vals)
    return {"sm_count": sm, "cc": (ccM, ccm), "l2_bytes": l2, "max_smem_optin": smem,
            "name": name.value.decode()}


def _dims(v):
    v = list(v) + [1] * (3 - len(v))
    return _U32x3(*[int(x) for x in v[:3]])


class Module:
    """One JIT-loaded PTX module and its entry point."""

    def __init__(self, ptx: str, entry: str, device: int | None = None):
        init(device)
        self.entry = entry
        h = ctypes.c_void_p()
        log = ctypes.create_string_buffer(16384)
        rc = lib().emmy_rt_module_load(ptx.encode("ascii"), entry.encode(), ctypes.byref(h), log,
                                       16384)
        if rc != 0:
            msg = lib().emmy_rt_last_error().decode(errors="replace")
            raise RuntimeErrorEmmy(rc, f"{msg}\n{log.value.decode(errors='replace')}")
        self.handle = h

    def close(self):
        if self.handle:
            lib().emmy_rt_module_unload(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:  # noqa: BLE001 - interpreter shutdown
            pass

    def attrs(self) -> dict:
        r, s, t = ctypes.c_int(), ctypes.c_int(), ctypes.c_int()
        check(lib().emmy_rt_module_attrs(self.handle, ctypes.byref(r), ctypes.byref(s),
                                         ctypes.byref(t)))
        return {"registers": r.value, "static_smem": s.value, "max_threads": t.value}

    def error_word(self, clear=True) -> int:
        v = ctypes.c_uint32()
        check(lib().emmy_rt_module_error_word(self.handle, ctypes.byref(v), int(clear)))
        return v.value

    def global_symbol(self, name):
        p, n = ctypes.c_uint64(), ctypes.c_uint64()
        check(lib().emmy_rt_module_global(self.handle, name.encode(), ctypes.byref(p),
                                          ctypes.byref(n)))
        return p.value, n.value

    def tensor_maps(self, enable=None) -> dict:
        """Tensor maps the module declares and how often the runtime has written them;
        ``enable=False`` stops writing them and clears the keys (the kernel then stages its
        tiles through registers), ``enable=True`` resumes."""
        n, up = ctypes.c_int(), ctypes.c_uint64()
        mode = -1 if enable is None else int(bool(enable))
        check(lib().emmy_rt_module_tensor_maps(self.handle, mode, ctypes.byref(n),
                                               ctypes.byref(up)))
        return {"maps": n.value, "uploads": up.value}

    def path_word(self, clear=False) -> int:
        """``emmy_path`` of a module with tensor maps (bit 0: a CTA loaded tiles by TMA,
        bit 1: one staged them through registers); 0 for other modules."""
        try:
            p, _ = self.global_symbol("emmy_path")
        except RuntimeErrorEmmy:
            return 0
        v = np.zeros(1, np.uint32)
        check(lib().emmy_rt_memcpy_dtoh(v.ctypes.data, p, 4))
        if clear:
            check(lib().emmy_rt_memset_zero(p, 4))
        return int(v[0])

    def launch(self, grid, block, smem, ptrs, stream=0, overlap=False):
        """Launch on ``stream``. ``overlap=True`` lets the grid start while the previous
        kernel on the stream finishes (programmatic stream serialization; the full sum/mean
        trigger it once their threads have streamed 7/8 of the input); only for kernels that
        order their writes with ``griddepcontrol.wait`` (the full sum/mean) and whose inputs
        the previous kernel does not write."""
        arr = (ctypes.c_uint64 * len(ptrs))(*[int(p) for p in ptrs])
        if overlap:
            check(lib().emmy_rt_launch_ex(self.handle, _dims(grid), _dims(block), int(smem),
                                          arr, len(ptrs), int(stream), LAUNCH_OVERLAP))
        else:
            check(lib().emmy_rt_launch(self.handle, _dims(grid), _dims(block), int(smem), arr,
                                       len(ptrs), int(stream)))

    def time(self, grid, block, smem, ptrs, *, iters=20, warmup=3, stream=0, flush_ptr=0,
             flush_bytes=0):
        """Per-launch milliseconds (CUDA events), L2 flushed before each launch if asked."""
        arr = (ctypes.c_uint64 * len(ptrs))(*[int(p) for p in ptrs])
        out = (ctypes.c_float * iters)()
        check(lib().emmy_rt_time(self.handle, _dims(grid), _dims(block), int(smem), arr,
                                 len(ptrs), int(stream), int(warmup), int(iters), int(flush_ptr),
                                 int(flush_bytes), out))
        return list(out)

    def run(self, grid, block, smem, host_args, *, warmup=0, iters=1):
        """Runner semantics with host numpy buffers; returns the timing stats dict.

        ``host_args`` is a list of ``(array, is_output, zero_each)`` in arg_order; output
        arrays are filled in place.
        """
        n = len(host_args)
        args = (_Arg * n)()
        keep = []
        for i, (arr, is_out, zero_each) in enumerate(host_args):
            if not arr.flags["C_CONTIGUOUS"]:
                raise ValueError("host buffers must be C-contiguous")
            keep.append(arr)
            args[i].host = arr.ctypes.data
            args[i].bytes = arr.nbytes
            args[i].is_output = int(bool(is_out))
            args[i].zero_each = int(bool(zero_each))
        st = _Stats()
        check(lib().emmy_rt_run(self.handle, _dims(grid), _dims(block), int(smem), args, n,
                                int(warmup), int(iters), ctypes.byref(st)))
        return {"kernel_us": st.kernel_us_median, "e2e_us": st.e2e_us_median,
                "h2d_bytes": st.h2d_bytes, "d2h_bytes": st.d2h_bytes}


def sync(stream=0, timeout_ms=60000):
    check(lib().emmy_rt_sync(int(stream), int(timeout_ms)))


class DeviceBuffer:
    """Device allocation through the runtime (for hosts without their own allocator)."""

    def __init__(self, nbytes: int):
        init()
        p = ctypes.c_uint64()
        check(lib().emmy_rt_mem_alloc(int(nbytes), ctypes.byref(p)))
        self.ptr = p.value
        self.nbytes = int(nbytes)

    @classmethod
    def from_array(cls, arr: np.ndarray):
        b = cls(max(arr.nbytes, 4))
        b.upload(arr)
        return b

    def upload(self, arr: np.ndarray):
        arr = np.ascontiguousarray(arr)
        check(lib().emmy_rt_memcpy_htod(self.ptr, arr.ctypes.data, arr.nbytes))

    def download(self, arr: np.ndarray):
        check(lib().emmy_rt_memcpy_dtoh(arr.ctypes.data, self.ptr, arr.nbytes))
        return arr

    def zero(self):
        check(lib().emmy_rt_memset_zero(self.ptr, self.nbytes))

    def free(self):
        if self.ptr:
            lib().emmy_rt_mem_free(self.ptr)
            self.ptr = 0

    def __del__(self):
        try:
            self.free()
        except Exception:  # noqa: BLE001
            pass


def run_kernel(ptx: str, kmeta: dict, inputs: dict, *, iters=1, warmup=0, device=0):
    """Compile-free runner: launch ``ptx`` under ``kmeta`` with host inputs.

    ``inputs`` maps argument names to numpy arrays (every non-output arg).
    Returns ``(outputs: name -> array, stats)``. Mirrors ``POST /run``.
    """
    mod = Module(ptx, kmeta["entry"], device)
    zero = set(kmeta.get("zero_outputs", ()))
    host, outs = [], {}
    for a in kmeta["args"]:
        shape = tuple(a.get("shape") or (1,))
        if a.get("output"):
            arr = np.zeros(shape, dtype=np.float32)
            outs[a["name"]] = arr
            host.append((arr, True, a["name"] in zero))
        else:
            arr = np.ascontiguousarray(inputs[a["name"]], dtype=np.float32).reshape(shape)
            host.append((arr, False, False))
    stats = mod.run(kmeta["grid"], kmeta["block"], kmeta.get("smem_bytes", 0), host,
                    warmup=warmup, iters=iters)
    err = mod.error_word()
    mod.close()
    if err:
        raise RuntimeErrorEmmy(-6, f"kernel {kmeta['entry']} reported error word {err:#x}")
    return outs, stats
