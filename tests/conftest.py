import json
import os
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
PKG = ROOT / "emmy-ir-to-ptx_b200"
for p in (str(ROOT), str(PKG)):
    if p not in sys.path:
        sys.path.insert(0, p)

PROBLEMS = ROOT / "tests" / "golden" / "problems"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (runs the emitted PTX through libemmyrt)")


def pytest_addoption(parser):
    parser.addoption("--synth-seeds", type=int, default=None,
                     help="seeds per family for the synthesized-IR GPU checks "
                          "(tests/test_gpu_synth.py; default 24-40 per family)")


def problem_dirs():
    return sorted(p for p in PROBLEMS.iterdir() if (p / "meta.json").is_file())


def load_problem(pdir):
    meta = json.loads((pdir / "meta.json").read_text())
    return meta


@pytest.fixture(scope="session")
def gpu_runtime():
    from emmyptx import runtime
    runtime.init(0)
    return runtime


def pytest_terminal_summary(terminalreporter):
    """The largest errors each parity check saw against its bound (tests/tolerance.py); with
    EMMY_TOLERANCE_REPORT set, also written there as JSON."""
    import tolerance
    lines = tolerance.report_lines()
    if not lines:
        return
    terminalreporter.section("parity errors against fp64 (largest per check)")
    for line in lines:
        terminalreporter.write_line(line)
    out = os.environ.get("EMMY_TOLERANCE_REPORT")
    if out:
        Path(out).write_text(json.dumps(tolerance.RECORD, indent=1, sort_keys=True))
