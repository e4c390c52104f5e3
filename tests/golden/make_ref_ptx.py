"""Generate the reference-PTX goldens: the reference compiler's own PTX for every fixture and
for the benchmark configurations in the forms its lowerers accept.

Run where the reference checkout is present (the tests read the committed PTX, so a machine
that runs them needs no checkout):

    python tests/golden/make_ref_ptx.py <reference checkout>/compile.py

emmy-ml is not installable offline, so the reference runs against the stand-in package in
``emmy_stub``, whose ``Graph.from_dict`` has a decoder of its own (``ast`` over Emmy's repr
text; nothing from this project is on the reference's path). Outputs go to
``ref_ptx/<name>.ptx`` with ``ref_ptx/MANIFEST.json`` recording, per PTX, its source (a fixture
folder, or a workload constructor call and the SHA-256 of the IR + meta it produced), so a
test can tell when a workload generator drifted from the IR the PTX was made from.

The reference's gates (rank <= 2, grid 1 for the scalar sum, 128-thread row kernels, the
f02/f03 statement forms) decide the config variants below; each is the same computation as
the benchmark workload it stands beside.
"""

from __future__ import annotations

import hashlib
import json
import os
import subprocess
import sys
import tempfile
from pathlib import Path

HERE = Path(__file__).resolve().parent
REPO = HERE.parents[1]
PKG = REPO / "emmy-ir-to-ptx_b200"
OUT = HERE / "ref_ptx"

# name -> (workload constructor, positional args, keyword args, benchmark workload it mirrors)
CONFIG_VARIANTS = {
    "add": ("pointwise_add", [1 << 20], {}, "add"),
    "sum_grid1": ("full_reduce", [1 << 26, "sum"], {"grid": 1}, "sum"),
    "mean_grid1": ("full_reduce", [1 << 26, "mean"], {"grid": 1}, "mean"),
    "rmsnorm_b128": ("row_op", ["rmsnorm"], {"block": 128}, "rmsnorm"),
    "softmax_b128": ("row_op", ["softmax"], {"block": 128}, "softmax"),
    "l2norm_b128": ("row_op", ["l2norm"], {"block": 128, "clamp": False}, "l2norm"),
    "matmul_sq": ("matmul", [4096, 4096, 4096], {}, "matmul_sq"),
    "matmul_rect": ("matmul", [8192, 2048, 4096], {}, "matmul_rect"),
    "attention_rows_d128": ("attention_rows", [2048, 128], {}, "attention_d128"),
    "attention_rows_d64": ("attention_rows", [2048, 64], {}, "attention_d64"),
}


def ir_digest(payload, meta) -> str:
    blob = json.dumps([payload, meta], sort_keys=True, separators=(",", ":")).encode()
    return hashlib.sha256(blob).hexdigest()


def make_variant(name):
    sys.path.insert(0, str(PKG))
    from emmyptx import workloads
    fn, args, kwargs, _ = CONFIG_VARIANTS[name]
    return getattr(workloads, fn)(*args, **kwargs)


def _run_reference(compile_py, ir_path):
    env = dict(os.environ, PYTHONPATH=str(HERE / "emmy_stub"))
    r = subprocess.run([sys.executable, str(compile_py), str(ir_path)], capture_output=True,
                       text=True, env=env, cwd=tempfile.gettempdir(), timeout=600)
    if r.returncode != 0:
        raise RuntimeError(f"reference compiler failed on {ir_path}: {r.stderr.strip()[-300:]}")
    return r.stdout


def main(compile_py: str) -> int:
    compile_py = Path(compile_py)
    OUT.mkdir(exist_ok=True)
    manifest = {"reference_compile_sha256": hashlib.sha256(compile_py.read_bytes()).hexdigest(),
                "entries": {}}
    for pdir in sorted(p for p in (HERE / "problems").iterdir() if p.is_dir()):
        ir = sorted(pdir.glob("*.ir.json"))[0]
        ptx = _run_reference(compile_py, ir)
        (OUT / f"{pdir.name}.ptx").write_text(ptx)
        manifest["entries"][pdir.name] = {"source": "fixture", "ir": ir.name,
                                          "ptx_sha256": hashlib.sha256(ptx.encode()).hexdigest()}
    for name, (fn, args, kwargs, mirrors) in CONFIG_VARIANTS.items():
        payload, meta = make_variant(name)
        with tempfile.TemporaryDirectory() as d:
            entry = meta["kernels"][0]["entry"]
            ir = Path(d) / f"{entry}.ir.json"
            ir.write_text(json.dumps(payload))
            (Path(d) / "meta.json").write_text(json.dumps(meta))
            ptx = _run_reference(compile_py, ir)
        (OUT / f"{name}.ptx").write_text(ptx)
        manifest["entries"][name] = {
            "source": "workload", "call": [fn, args, kwargs], "mirrors": mirrors,
            "ir_sha256": ir_digest(payload, meta),
            "ptx_sha256": hashlib.sha256(ptx.encode()).hexdigest()}
    (OUT / "MANIFEST.json").write_text(json.dumps(manifest, indent=1, sort_keys=True) + "\n")
    print(f"wrote {len(manifest['entries'])} reference PTX files to {OUT}")
    return 0


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit(f"usage: python {sys.argv[0]} <reference checkout>/compile.py")
    sys.exit(main(sys.argv[1]))
