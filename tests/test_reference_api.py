"""The reference compiler's Python API, exercised the way its own unit tests use it.

The reference's tests bind ``from compile import EmmyIRParser, EmmyKernelIR,
PTXKernelGenerator`` (reference ``tests/test_ptx_kernel_generator.py`` and
``tests/test_emmy_ir_parser.py``). This file restates the portable part of those two files
against this repository's ``compile`` module, case by case, with the same expectations:
parameter order and names, register names, shared declarations, the single-instruction
rule, the ``ret`` handling, metadata authority, and the error messages the reference's tests
match on.

Not restated, by design:
* the parser tests that inject a fake ``emmy.compiler.graph`` module (reference
  ``tests/test_emmy_ir_parser.py:10-48``): this parser decodes the IR itself and never
  imports emmy, so the same checks are made here on real IR payloads built by ``_payload``;
* the register *declaration* lines (``.reg .u32 %r0;`` per register, reference
  ``tests/test_ptx_kernel_generator.py:80-106``): registers are declared in ranges
  (``.reg .b32 %r<2>;``), one line per register class. The register *names* the reference
  expects are kept and checked below;
* the lowering tests' checks of the reference templates' own instruction text (reference
  ``tests/test_emmy_ir_lowering.py``, ``test_emmy_reduction_lowering.py``,
  ``test_emmy_rmsnorm_ptx.py``, ``test_emmy_softmax_lowering.py``,
  ``test_emmy_l2norm_lowering.py``): counts of scalar ``ld.global.f32`` (these templates
  load 16-byte vectors), ``add.f32`` (every add carries ``.rn``), ``max.f32``/``min.f32``
  (``max.NaN``/``min.NaN``, which propagate NaN as numpy and PyTorch do), the reference's
  label, shared-array and register names, its barrier and shuffle counts, and
  ``.version 8.0`` (sm_100a needs a later PTX ISA). What those tests check about behaviour
  (entry and parameters, one ``ret``, a cooperative reduction with warp shuffles and CTA
  barriers, the op table's instruction per operation, fail-closed errors) is restated
  below.
"""

import json

import pytest

from types import SimpleNamespace

from compile import EmmyIRLowering, EmmyIRParser, EmmyKernelIR, PTXKernelGenerator
from conftest import PROBLEMS

_F32 = "DataType(name='f32', np=dtype('float32'), nbytes=4)"
_BODY = ("Tile(axes=(Axis(name='a0', extent=Dim(4), window=None),), body=(Load(names=('v',), "
         f"input='a', index=(Var(name='a0'),), dtype={_F32}), Write(output='out', "
         f"index=(Var(name='a0'),), values=('v',), value_dtype={_F32}, atomic=False, "
         "swizzle='NONE')), block_threads=None, aux_threads=0, raster_axes=None, "
         "raster_group=None, raster_orient='m')")


def _payload(kernels=1, body=None):
    """A graph with two inputs and ``kernels`` KernelOps named ``sample_kernel``."""
    nodes = {n: {"op": "InputOp", "op_fields": {}, "inputs": [],
                 "outputs": [{"name": n, "shape": [4], "dtype": "f32"}]} for n in ("a", "b")}
    for i in range(kernels):
        nodes[f"node{i}"] = {"op": "KernelOp",
                             "op_fields": {"name": "sample_kernel",
                                           "body": [_BODY] if body is None else body},
                             "inputs": ["a", "b"],
                             "outputs": [{"name": "out", "shape": [4], "dtype": "f32"}]}
    return {"inputs": ["a", "b"], "outputs": ["out"], "nodes": nodes}


def _write(tmp_path, data):
    path = tmp_path / "sample.ir.json"
    path.write_text(json.dumps(data), encoding="utf-8")
    return path


def _meta(*, arg_order=("a", "out"), include_arg_order=True, **extra):
    rec = {"node": "node0", "entry": "sample_kernel", "grid": [1, 1, 1], "block": [128, 1, 1],
           "smem_bytes": 0}
    if include_arg_order:
        rec["arg_order"] = arg_order if not isinstance(arg_order, tuple) else list(arg_order)
    return {"id": "test_problem", "kernels": [rec], **extra}


# ---------------------------------------------------------------------------
# EmmyIRParser (reference tests/test_emmy_ir_parser.py)
# ---------------------------------------------------------------------------

def test_parse_gives_kernel_view(tmp_path):
    parsed = EmmyIRParser(_write(tmp_path, _payload())).parse()
    assert isinstance(parsed, EmmyKernelIR)
    assert parsed.name == "sample_kernel"
    assert parsed.inputs == ("a", "b")
    assert parsed.outputs == ("out",)
    assert len(parsed.body) == 1 and type(parsed.body[0]).__name__ == "Tile"
    assert parsed.arg_order is None                  # no meta.json beside it


def test_required_metadata_missing(tmp_path):
    with pytest.raises(ValueError, match="Missing required metadata"):
        EmmyIRParser(_write(tmp_path, _payload()), require_meta=True).parse()


@pytest.mark.parametrize("count", [0, 2])
def test_exactly_one_kernel(tmp_path, count):
    with pytest.raises(ValueError, match="exactly one KernelOp"):
        EmmyIRParser(_write(tmp_path, _payload(kernels=count))).parse()


def test_undecodable_graph(tmp_path):
    with pytest.raises(ValueError, match="could not deserialize"):
        EmmyIRParser(_write(tmp_path, _payload(body=["NotAStatement(1)"]))).parse()


def test_malformed_json(tmp_path):
    path = tmp_path / "broken.ir.json"
    path.write_text("{bad json", encoding="utf-8")
    with pytest.raises(ValueError, match="Invalid JSON"):
        EmmyIRParser(path).parse()


def test_missing_ir_file(tmp_path):
    with pytest.raises(ValueError, match="Cannot read"):
        EmmyIRParser(tmp_path / "missing.ir.json").parse()


def test_metadata_arg_order_wins(tmp_path):
    path = _write(tmp_path, _payload())
    (tmp_path / "meta.json").write_text(json.dumps(_meta(arg_order=("out", "b", "a"),
                                                         rtol=1e-5)), encoding="utf-8")
    parsed = EmmyIRParser(path, require_meta=True).parse()
    assert parsed.arg_order == ("out", "b", "a")
    assert parsed.launch["block"] == [128, 1, 1]
    assert parsed.launch["smem_bytes"] == 0
    assert parsed.metadata["rtol"] == 1e-5
    assert parsed.metadata["selected_kernel"]["entry"] == "sample_kernel"


def test_metadata_from_explicit_path(tmp_path):
    path = _write(tmp_path, _payload())
    other = tmp_path / "other.json"
    other.write_text(json.dumps(_meta(arg_order=("a", "out"))), encoding="utf-8")
    parsed = EmmyIRParser(path, meta_path=other, require_meta=True).parse()
    assert parsed.arg_order == ("a", "out")


def test_arg_order_required(tmp_path):
    path = _write(tmp_path, _payload())
    (tmp_path / "meta.json").write_text(json.dumps(_meta(include_arg_order=False)),
                                        encoding="utf-8")
    with pytest.raises(ValueError, match="arg_order"):
        EmmyIRParser(path, require_meta=True).parse()


@pytest.mark.parametrize("order", [["a", "a"], ["a", 3], "a"])
def test_arg_order_must_be_distinct_names(tmp_path, order):
    path = _write(tmp_path, _payload())
    (tmp_path / "meta.json").write_text(json.dumps(_meta(arg_order=order)), encoding="utf-8")
    with pytest.raises(ValueError, match="arg_order"):
        EmmyIRParser(path, require_meta=True).parse()


def test_json_must_be_an_object(tmp_path):
    with pytest.raises(ValueError, match="Expected a JSON object"):
        EmmyIRParser(_write(tmp_path, [])).parse()


# ---------------------------------------------------------------------------
# PTXKernelGenerator (reference tests/test_ptx_kernel_generator.py)
# ---------------------------------------------------------------------------

@pytest.fixture
def kernel():
    """The launch record of the r01_array_sum fixture, as a kernel view."""
    selected = {"node": "sum_1", "entry": "k_sum_1_reduce", "arg_order": ["x", "sum_1"],
                "grid": [1, 1, 1], "block": [128, 1, 1], "smem_bytes": 0,
                "args": [{"name": "x", "dtype": "f32", "shape": [1024], "seed": 0},
                         {"name": "sum_1", "dtype": "f32", "shape": [1], "output": True}]}
    return EmmyKernelIR(name="k_sum_1_reduce", body=(), graph=object(), node_key="sum_1",
                        inputs=("x",), outputs=("sum_1",), arg_order=("x", "sum_1"),
                        launch={"grid": [1, 1, 1], "block": [128, 1, 1], "smem_bytes": 0},
                        metadata={"selected_kernel": selected})


def test_entry_signature(kernel):
    ptx = PTXKernelGenerator(kernel).render_entry()
    assert ".visible .entry k_sum_1_reduce(" in ptx
    assert ".param .u64 param_x" in ptx and ".param .u64 param_sum_1" in ptx
    assert ptx.endswith("    ret;\n}\n")
    assert ptx.index("param_x") < ptx.index("param_sum_1")
    assert ".version" not in ptx and ".target" not in ptx     # the header is the emitter's


def test_parameter_names(kernel):
    gen = PTXKernelGenerator(kernel)
    assert gen.parameter("x") == "param_x"
    assert gen.parameter("sum_1") == "param_sum_1"
    with pytest.raises(KeyError):
        gen.parameter("unknown")


def test_register_names(kernel):
    gen = PTXKernelGenerator(kernel)
    assert [gen.register(".u32"), gen.register(".u32"), gen.register(".f32"),
            gen.register(".pred"), gen.register(".u64")] == ["%r0", "%r1", "%f0", "%p0", "%rd0"]
    ptx = gen.render_entry()
    for decl in (".reg .b32 %r<2>;", ".reg .f32 %f<1>;", ".reg .pred %p<1>;",
                 ".reg .b64 %rd<1>;"):
        assert decl in ptx


def test_shared_declaration(kernel):
    gen = PTXKernelGenerator(kernel)
    gen.shared("scratch", ".f32", length=32, align=16)
    assert ".shared .align 16 .f32 scratch[32];" in gen.render_entry()


@pytest.mark.parametrize("length", [0, -1, 1.5, True])
def test_shared_length_must_be_positive_int(kernel, length):
    with pytest.raises(ValueError):
        PTXKernelGenerator(kernel).shared("scratch", ".f32", length=length)


def test_thread_index_1d_sequence(kernel):
    gen = PTXKernelGenerator(kernel)
    assert gen.thread_index_1d() == "%r4"
    ptx = gen.render_entry()
    for line in ("mov.u32 %r0, %tid.x;", "mov.u32 %r1, %ctaid.x;", "mov.u32 %r2, %ntid.x;",
                 "mul.lo.u32 %r3, %r1, %r2;", "add.u32 %r4, %r3, %r0;"):
        assert line in ptx


def test_emit_one_instruction(kernel):
    gen = PTXKernelGenerator(kernel)
    a, b, c = (gen.register(".f32") for _ in range(3))
    gen.emit(f"add.f32 {c}, {a}, {b};")
    assert "add.f32 %f2, %f0, %f1;" in gen.render_entry()


@pytest.mark.parametrize("instruction", ["", "add.f32 %f0, %f1, %f2", "ret;\ntrap;",
                                         "mov.u32 %r0, 1; ret;", "ret;\n"])
def test_emit_refuses_anything_but_one_instruction(kernel, instruction):
    with pytest.raises(ValueError):
        PTXKernelGenerator(kernel).emit(instruction)


def test_single_ret(kernel):
    gen = PTXKernelGenerator(kernel)
    gen.emit("ret;")
    assert gen.render_entry().count("ret;") == 1


def test_selected_kernel_required(kernel):
    kernel.metadata.clear()
    with pytest.raises(ValueError, match="selected_kernel"):
        PTXKernelGenerator(kernel)


def test_args_must_match_arg_order(kernel):
    kernel.metadata["selected_kernel"]["args"] = [{"name": "x", "dtype": "f32", "shape": [1024]}]
    with pytest.raises(ValueError, match="do not match"):
        PTXKernelGenerator(kernel)


# ---------------------------------------------------------------------------
# EmmyIRLowering (reference tests/test_emmy_ir_lowering.py and the row-operation lowering
# tests): the behaviour they check, on the reference's own fixtures
# ---------------------------------------------------------------------------

def _fixture(problem, entry):
    return EmmyIRParser(PROBLEMS / problem / f"{entry}.ir.json", require_meta=True).parse()


@pytest.fixture
def pointwise():
    return _fixture("p00_scalar_add", "k_add_pointwise")


def test_pointwise_kernel_view(pointwise):
    assert pointwise.name == "k_add_pointwise"
    assert pointwise.arg_order == ("x0", "x1", "add")


def test_pointwise_entry_parameters_and_single_ret(pointwise):
    ptx = EmmyIRLowering(pointwise).lower()
    assert ".visible .entry k_add_pointwise(" in ptx
    for arg in ("x0", "x1", "add"):
        assert f".param .u64 param_{arg}" in ptx
        assert f"[param_{arg}]" in ptx
    assert "ld.param.u64" in ptx
    assert ptx.count("ret;") == 1
    assert ptx.rstrip().endswith("}")


@pytest.mark.parametrize("problem,entry", [("r01_array_sum", "k_sum_1_reduce"),
                                           ("r03_mean", None),
                                           ("f01_rmsnorm", None), ("f02_row_softmax", None),
                                           ("f03_l2norm", None)])
def test_cooperative_reductions_lower(problem, entry):
    """Every reduction and row-normalisation fixture lowers to a kernel that reduces across
    the CTA: warp shuffles and CTA barriers."""
    if entry is None:
        entry = next((PROBLEMS / problem).glob("*.ir.json")).name[:-len(".ir.json")]
    kernel = _fixture(problem, entry)
    ptx = EmmyIRLowering(kernel).lower()
    assert f".visible .entry {kernel.name}(" in ptx
    assert "shfl.sync.bfly.b32" in ptx
    assert "bar.sync 0;" in ptx


def test_unknown_statement_fails_naming_it(pointwise):
    import dataclasses

    class WarpMagic:
        pass

    broken = dataclasses.replace(pointwise, body=(WarpMagic(),))
    with pytest.raises(NotImplementedError, match="WarpMagic"):
        EmmyIRLowering(broken).lower()


def _assign(lowering, op, args):
    for a in args:
        lowering.values[a] = lowering.gen.register(".f32")
    stmt = SimpleNamespace(name="result", op=SimpleNamespace(name=op), args=args,
                           dtype=SimpleNamespace(name="f32"))
    lowering._assign(stmt)
    assert "result" in lowering.values
    return lowering.gen.render_entry()


@pytest.mark.parametrize("op,args,instruction", [
    ("negative", ("a",), "neg.f32"), ("absolute", ("a",), "abs.f32"),
    ("identity", ("a",), "mov.f32"), ("sqrt", ("a",), "sqrt.rn.f32"),
    ("rsqrt", ("a",), "rsqrt.approx.f32"), ("divide", ("a", "b"), "div.rn.f32"),
    ("reciprocal", ("a",), "rcp.rn.f32"), ("exp", ("a",), "ex2.approx.f32"),
    ("relu", ("a",), "max.NaN.f32"), ("maximum", ("a", "b"), "max.NaN.f32"),
    ("minimum", ("a", "b"), "min.NaN.f32"), ("add", ("a", "b"), "add.rn.f32"),
])
def test_op_table_instruction(pointwise, op, args, instruction):
    assert instruction in _assign(EmmyIRLowering(pointwise), op, args)


def test_unknown_unary_operation_fails(pointwise):
    with pytest.raises(NotImplementedError, match="Unsupported unary"):
        _assign(EmmyIRLowering(pointwise), "unsupported_op", ("a",))
