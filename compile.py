"""Emmy Kernel IR -> PTX for B200 (sm_100a).

    python compile.py path/to/<kernel>.ir.json > out.ptx

Reads one Kernel IR file and its sibling ``meta.json`` (grid, block, shared
bytes, ``arg_order``) and writes PTX to stdout. Exit codes follow the
reference contract (reference ``compile.py:5884-5923``): 2 for a usage
error, 1 for a missing file or any compile failure (traceback on stderr),
0 on success. Only the standard library is imported on this path.
"""

import os
import sys

_PKG = os.path.join(os.path.dirname(os.path.abspath(__file__)), "emmy-ir-to-ptx_b200")
if _PKG not in sys.path:
    sys.path.insert(0, _PKG)


# The reference's public classes, importable from this module as its tests do
# (``from compile import EmmyIRParser, EmmyKernelIR, PTXKernelGenerator``); resolved on
# first use so that the command line path imports nothing extra.
_API = ("EmmyKernelIR", "EmmyIRParser", "PTXKernelGenerator", "EmmyIRLowering", "PTXEmitter")


def __getattr__(name):
    if name in _API:
        import emmyptx
        return getattr(emmyptx, name)
    raise AttributeError(name)


def main(argv=None) -> int:
    argv = sys.argv if argv is None else argv
    if len(argv) != 2:
        print("Usage: python compile.py <kernel.ir.json>", file=sys.stderr)
        return 2
    path = argv[1]
    if not os.path.isfile(path):
        print(f"Input file not found: {path}", file=sys.stderr)
        return 1
    try:
        from emmyptx.emit import compile_file
        ptx = compile_file(path)
    except Exception:  # noqa: BLE001 - any failure is a compile failure (exit 1)
        import traceback
        traceback.print_exc()
        return 1
    sys.stdout.write(ptx)
    return 0


if __name__ == "__main__":
    sys.exit(main())
