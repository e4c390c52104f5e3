"""The C-ABI library loads here (no GPU) and exports every entry point its header declares."""

import ctypes
import subprocess

from emmyptx import runtime


def test_library_exports_header_symbols():
    path = runtime.library_path()
    assert path.is_file(), "build libemmyrt.so first (python __graft_entry__.py build)"
    declared = runtime.exported_symbols()
    assert "emmy_rt_launch" in declared and "emmy_rt_run" in declared
    out = subprocess.run(["nm", "-D", "--defined-only", str(path)], capture_output=True,
                         text=True).stdout
    exported = {line.split()[-1] for line in out.splitlines() if line.strip()}
    missing = [s for s in declared if s not in exported]
    assert not missing, missing
    lib = ctypes.CDLL(str(path))
    for s in declared:
        getattr(lib, s)


def test_abi_version_and_error_path():
    L = runtime.lib()
    assert L.emmy_rt_abi_version() == 1
    import torch
    if not torch.cuda.is_available():
        rc = L.emmy_rt_init(0)
        assert rc != 0
        assert L.emmy_rt_last_error()


class _FakeLib:
    def emmy_rt_init(self, device):
        return 0


def test_init_notes_a_device_that_is_not_a_b200(monkeypatch):
    """Initialising a device whose SM count differs from B200's warns once (the emitted work
    splits are sized for 148 SMs) and stays silent on a B200; no GPU needed (fake library)."""
    import warnings

    import pytest
    monkeypatch.setattr(runtime, "lib", lambda: _FakeLib())
    monkeypatch.setattr(runtime, "_initialised", set())
    monkeypatch.setattr(runtime, "device_info", lambda d: {"sm_count": 132})
    with pytest.warns(RuntimeWarning, match="132 SMs"):
        runtime.init(3)
    with warnings.catch_warnings():
        warnings.simplefilter("error")
        runtime.init(3)                                  # already initialised: no second note
        monkeypatch.setattr(runtime, "device_info", lambda d: {"sm_count": 148})
        runtime.init(4)
