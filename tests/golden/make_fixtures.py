"""Copy the reference's fixture problems into ``tests/golden/problems``.

Run once in a container that has the reference checkout:

    python tests/golden/make_fixtures.py <reference checkout>/problems

For every problem folder it copies the Kernel IR (``*.ir.json``), the launch
record (``meta.json``) and the golden outputs (``expected.npz``). These are
data, not code: Emmy's CUDA renderings (``*.ref.cu``) are not copied. The
tests read these copies only, so a machine that runs them needs no
reference checkout.

It then checks that the oracle's fp64 expressions reproduce every
``expected.npz`` array byte for byte from the seeded inputs, which pins the
oracle to the reference's own goldens.
"""

from __future__ import annotations

import hashlib
import json
import shutil
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
DEST = HERE / "problems"


def main(src: str) -> int:
    src_dir = Path(src)
    problems = sorted(p for p in src_dir.iterdir() if (p / "meta.json").is_file())
    if not problems:
        print(f"no problems under {src_dir}", file=sys.stderr)
        return 1
    DEST.mkdir(parents=True, exist_ok=True)
    manifest = {}
    for p in problems:
        out = DEST / p.name
        out.mkdir(exist_ok=True)
        files = sorted(p.glob("*.ir.json")) + [p / "meta.json", p / "expected.npz"]
        entry = {}
        for f in files:
            shutil.copyfile(f, out / f.name)
            entry[f.name] = hashlib.sha256(f.read_bytes()).hexdigest()
        manifest[p.name] = entry
    (DEST / "MANIFEST.json").write_text(json.dumps(manifest, indent=1, sort_keys=True) + "\n")

    sys.path.insert(0, str(HERE.parents[1]))
    from oracle.expressions import check_goldens
    bad = check_goldens(DEST)
    for name, msg in bad:
        print(f"golden mismatch {name}: {msg}", file=sys.stderr)
    print(f"copied {len(problems)} problems; {len(bad)} golden mismatches")
    return 1 if bad else 0


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit(f"usage: python {sys.argv[0]} <reference checkout>/problems")
    sys.exit(main(sys.argv[1]))
