"""The ``python compile.py <ir.json>`` contract (reference compile.py:5884-5923, TASK.md:1-35)."""

import json
import re
import shutil
import subprocess
import sys

import pytest

from conftest import PROBLEMS, ROOT, problem_dirs

COMPILE = ROOT / "compile.py"
PTXAS = shutil.which("ptxas")


def run_cli(*args):
    return subprocess.run([sys.executable, str(COMPILE), *map(str, args)], capture_output=True,
                          text=True)


def test_usage_exit_2():
    r = run_cli()
    assert r.returncode == 2 and "Usage" in r.stderr and r.stdout == ""
    assert run_cli("a", "b").returncode == 2


def test_missing_file_exit_1(tmp_path):
    r = run_cli(tmp_path / "nope.ir.json")
    assert r.returncode == 1 and r.stdout == ""


def test_missing_meta_exit_1(tmp_path):
    src = next((PROBLEMS / "p00_scalar_add").glob("*.ir.json"))
    dst = tmp_path / src.name
    dst.write_text(src.read_text())
    r = run_cli(dst)
    assert r.returncode == 1 and "meta" in r.stderr and r.stdout == ""


def test_unsupported_statement_fails_closed(tmp_path):
    src = next((PROBLEMS / "p00_scalar_add").glob("*.ir.json"))
    payload = json.loads(src.read_text())
    body = payload["nodes"]["add"]["op_fields"]["body"][0]
    payload["nodes"]["add"]["op_fields"]["body"][0] = body.replace(
        "ElementwiseImpl('add')", "ElementwiseImpl('frobnicate')")
    (tmp_path / src.name).write_text(json.dumps(payload))
    (tmp_path / "meta.json").write_text((PROBLEMS / "p00_scalar_add" / "meta.json").read_text())
    r = run_cli(tmp_path / src.name)
    assert r.returncode == 1 and r.stdout == ""
    assert "frobnicate" in r.stderr


def test_warp_shuffle_with_a_partial_warp_fails_closed():
    """r01's sum rescheduled for 48 threads per CTA (cells fill the CTA, but its second warp
    has 16 lanes): the walker refuses it rather than emit a full-warp shuffle."""
    from emmyptx.emit import compile_payload
    pdir = PROBLEMS / "r01_array_sum"
    payload = json.loads((pdir / "k_sum_1_reduce.ir.json").read_text())
    node = payload["nodes"]["sum_1"]["op_fields"]
    node["body"] = [b.replace("Dim(128)", "Dim(48)").replace("value=128", "value=48")
                    for b in node["body"]]
    meta = json.loads((pdir / "meta.json").read_text())
    meta["kernels"][0]["block"] = [48, 1, 1]
    with pytest.raises(NotImplementedError, match="WarpShuffle needs whole warps"):
        compile_payload(payload, meta, template="walker")
    with pytest.raises(NotImplementedError, match="whole"):
        compile_payload(payload, meta)


_SYNC = "Sync(barrier_id=0, count=None, warp=False)"
_ACCUM = ("Accum(name='acc0', value='in0', op=ElementwiseImpl('add'), dtype=DataType(name='f32', "
          "np=dtype('float32'), nbytes=4), axes=('a0',), base=None)")


@pytest.mark.parametrize("old,new,where", [
    (_SYNC, "Cond(cond=BinaryExpr(op='==', left=Var(name='lane'), right=Literal(value=0, "
            f"dtype='int')), body=({_SYNC},), else_body=())", "a Cond"),
    (_ACCUM, f"{_ACCUM}, {_SYNC}", "a StridedLoop with variable bounds"),
])
def test_barrier_off_the_convergent_path_fails_closed(old, new, where):
    """r01's sum with its CTA barrier moved under a lane test, or into the strided loop whose
    start is the thread's own index (trip counts differ between threads): refused, since a
    thread that never reaches the barrier would leave the others waiting."""
    from emmyptx.emit import compile_payload
    pdir = PROBLEMS / "r01_array_sum"
    payload = json.loads((pdir / "k_sum_1_reduce.ir.json").read_text())
    node = payload["nodes"]["sum_1"]["op_fields"]
    assert all(old in b for b in node["body"])
    node["body"] = [b.replace(old, new) for b in node["body"]]
    meta = json.loads((pdir / "meta.json").read_text())
    for template in ("walker", None):
        with pytest.raises(NotImplementedError, match=f"Sync inside {where}"):
            compile_payload(payload, meta, template=template)


@pytest.mark.parametrize("sync,refused", [
    ("Sync(barrier_id=1, count=128, warp=False)", None),
    ("Sync(barrier_id=16, count=None, warp=False)", "barrier id 16"),
    ("Sync(barrier_id=1, count=256, warp=False)", "barrier count 256"),
    ("Sync(barrier_id=1, count=48, warp=False)", "barrier count 48"),
])
def test_barrier_ids_and_counts(sync, refused):
    """A CTA has 16 barriers, and a counted barrier waits for that many threads, in whole
    warps: a count above the CTA's 128 threads would never be met."""
    from emmyptx.emit import compile_payload
    pdir = PROBLEMS / "r01_array_sum"
    payload = json.loads((pdir / "k_sum_1_reduce.ir.json").read_text())
    node = payload["nodes"]["sum_1"]["op_fields"]
    node["body"] = [b.replace(_SYNC, sync) for b in node["body"]]
    meta = json.loads((pdir / "meta.json").read_text())
    if refused is None:
        ptx, template, _ = compile_payload(payload, meta, template="walker")
        assert "bar.sync 1, 128;" in ptx
    else:
        with pytest.raises(NotImplementedError, match=refused):
            compile_payload(payload, meta, template="walker")


_F32_IR = "DataType(name='f32', np=dtype('float32'), nbytes=4)"
_F16_IR = "DataType(name='f16', np=dtype('float16'), nbytes=2)"


@pytest.mark.parametrize("where", ["ir", "meta"])
@pytest.mark.parametrize("pdir", problem_dirs(), ids=lambda p: p.name)
def test_other_dtypes_fail_closed(pdir, where):
    """Every template computes in f32: a fixture retyped to f16, in its IR statements or in
    meta.json's argument records, is refused (reference compile.py:2297-2306) instead of
    being compiled as if its buffers held f32."""
    from emmyptx.emit import compile_payload
    meta = json.loads((pdir / "meta.json").read_text())
    for k in meta["kernels"]:
        payload = json.loads((pdir / f"{k['entry']}.ir.json").read_text())
        if where == "ir":
            for node in payload["nodes"].values():
                if node["op"] == "KernelOp":
                    node["op_fields"]["body"] = [b.replace(_F32_IR, _F16_IR)
                                                 for b in node["op_fields"]["body"]]
        else:
            k["args"][0]["dtype"] = "f16"
        one = dict(meta, kernels=[k])
        with pytest.raises(NotImplementedError, match="f16"):
            compile_payload(payload, one)


@pytest.mark.parametrize("field,value", [("block", [0, 1, 1]), ("block", [2048, 1, 1]),
                                         ("block", ["128", 1, 1]), ("grid", [0, 1, 1]),
                                         ("grid", [-4, 1, 1]), ("grid", [1, 70000, 1]),
                                         ("block", [128, 1]), ("smem_bytes", -1)])
def test_impossible_launch_records_fail_closed(field, value):
    """A meta.json launch CUDA could not make is refused before any template sizes its work
    from it."""
    from emmyptx.emit import compile_payload
    for problem in ("p01_vector_add", "m01_matmul_512"):
        pdir = PROBLEMS / problem
        meta = json.loads((pdir / "meta.json").read_text())
        meta["kernels"][0][field] = value
        payload = json.loads(next(pdir.glob("*.ir.json")).read_text())
        with pytest.raises(ValueError, match=f"launch {field}"):
            compile_payload(payload, meta)


def test_deeply_nested_json_fails_closed(tmp_path):
    (tmp_path / "k.ir.json").write_text("[" * 200000 + "]" * 200000)
    (tmp_path / "meta.json").write_text((PROBLEMS / "p00_scalar_add" / "meta.json").read_text())
    r = run_cli(tmp_path / "k.ir.json")
    assert r.returncode == 1 and r.stdout == ""
    assert "nested too deeply" in r.stderr


LOWERED = problem_dirs()


@pytest.mark.parametrize("pdir", LOWERED, ids=lambda p: p.name)
def test_cli_emits_sm100a_ptx(pdir, tmp_path):
    meta = json.loads((pdir / "meta.json").read_text())
    for k in meta["kernels"]:
        r = run_cli(pdir / f"{k['entry']}.ir.json")
        assert r.returncode == 0, r.stderr
        ptx = r.stdout
        assert ptx.isascii()
        lines = [ln.strip() for ln in ptx.splitlines() if ln.strip()]
        assert lines[0] == ".version 8.8"
        assert lines[1] == ".target sm_100a"
        assert lines[2] == ".address_size 64"
        m = re.search(r"\.visible \.entry (\w+)\(([^)]*)\)", ptx)
        assert m and m.group(1) == k["entry"]
        params = re.findall(r"\.param \.u64 param_(\w+)", m.group(2))
        assert params == k["arg_order"]
        assert ptx.count("ret;") >= 1
        if PTXAS:
            f = tmp_path / "k.ptx"
            f.write_text(ptx)
            a = subprocess.run([PTXAS, "-arch=sm_100a", "-o", str(tmp_path / "k.cubin"), str(f)],
                               capture_output=True, text=True)
            assert a.returncode == 0, a.stderr


def test_pointwise_is_vectorised_and_uncontracted():
    from emmyptx.emit import compile_file
    ptx = compile_file(next((PROBLEMS / "p02_scale_shift").glob("*.ir.json")))
    assert "ld.global.nc.L1::no_allocate.v4.f32" in ptx
    assert "st.global.v4.f32" in ptx
    assert "mul.rn.f32" in ptx and "add.rn.f32" in ptx
    assert re.search(r"\b(add|mul)\.f32\b", ptx) is None
    assert "fma" not in ptx


def test_reduction_uses_cross_cta_finish():
    from emmyptx import workloads
    from emmyptx.emit import compile_payload
    ptx, template, _ = compile_payload(*workloads.full_reduce(1 << 20, "sum", grid=64))
    assert template == "rowreduce"
    assert "atom.acq_rel.gpu.global.inc.u32" in ptx
    assert ptx.count("shfl.sync.bfly.b32") >= 5
    assert ".global .align 16 .f64 emmy_partials64" in ptx


def test_sums_accumulate_in_f64():
    """Sums (full sum and mean, row sums) widen every element and add in f64, in the
    per-thread loop and in every fold; the fused row operations (their statistics have no
    cancellation) keep f32."""
    from emmyptx import workloads
    from emmyptx.emit import compile_payload
    for payload, meta in (workloads.full_reduce(1 << 20, "sum", grid=64),
                          workloads.full_reduce(1 << 20, "mean", grid=64),
                          workloads.row_op("rowsum", rows=4, cols=512)):
        ptx, _, _ = compile_payload(payload, meta)
        assert "cvt.f64.f32" in ptx and "add.rn.f64" in ptx and "cvt.rn.f32.f64" in ptx
        assert "shfl.sync.bfly.b32" in ptx and "ld.shared.f64" in ptx
    for kind in ("rmsnorm", "softmax", "l2norm"):
        ptx, _, _ = compile_payload(*workloads.row_op(kind, rows=4, cols=512))
        assert ".f64" not in ptx and "cvt.f64" not in ptx


def test_single_cta_reduction_skips_the_ticket():
    """r02's launch has one CTA (CTAs beyond the compiled grid return), so its partial is the
    result: no partials round trip, no ticket."""
    from emmyptx.emit import compile_file
    ptx = compile_file(next((PROBLEMS / "r02_big_sum").glob("*.ir.json")))
    assert "atom" not in ptx and "ld.relaxed" not in ptx
    assert ptx.count("shfl.sync.bfly.b32") >= 5


def test_rows_are_staged_with_bulk_copies():
    from emmyptx.emit import compile_file
    ptx = compile_file(next((PROBLEMS / "f01_rmsnorm").glob("*.ir.json")))
    assert "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes" in ptx
    assert "mbarrier.try_wait.parity" in ptx
    assert "red.global.or.b32 [emmy_error], 1;" in ptx     # bounded wait records a timeout


@pytest.mark.parametrize("pdir", problem_dirs(), ids=lambda p: p.name)
def test_general_walker_lowers_every_fixture(pdir, tmp_path):
    """Forcing the statement walker (no template) still yields assembling sm_100a PTX."""
    from emmyptx.emit import compile_file
    meta = json.loads((pdir / "meta.json").read_text())
    for k in meta["kernels"]:
        ptx = compile_file(pdir / f"{k['entry']}.ir.json", template="walker")
        assert f".visible .entry {k['entry']}(" in ptx
        if PTXAS:
            f = tmp_path / "w.ptx"
            f.write_text(ptx)
            a = subprocess.run([PTXAS, "-arch=sm_100a", "-o", str(tmp_path / "w.cubin"), str(f)],
                               capture_output=True, text=True)
            assert a.returncode == 0, a.stderr
