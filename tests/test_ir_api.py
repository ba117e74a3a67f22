"""IR, DSL and frontend behave like the reference's (host only)."""

import json
from pathlib import Path

import pytest
import torch

import devproc
from devproc.ir.verifier import IRVerifier
from devproc_b200 import workloads
from devproc_b200.ir.function import Function
from devproc_b200.ir.ops import OpBuilder
from devproc_b200.ir.types import ScalarType, TensorType

GOLD = json.loads((Path(__file__).parent / "golden" / "ir_ops.json").read_text())


def test_types_validate_like_reference():
    with pytest.raises(TypeError):
        TensorType([224, 224], "float32")
    with pytest.raises(ValueError):
        TensorType((0, 3), "float32")
    with pytest.raises(ValueError):
        TensorType((3,), "complex64")
    with pytest.raises(ValueError):
        ScalarType("uint8")
    assert TensorType((2, 3), "bfloat16").nbytes == 12
    assert repr(TensorType((224, 224, 3), "uint8")) == "uint8[224,224,3]"


def test_argmax_keeps_reference_scalar_type_by_default():
    v = OpBuilder.input("x", TensorType((1, 10), "float32")).outputs[0]
    op = OpBuilder.argmax(v, dim=1)
    assert isinstance(op.outputs[0].type, ScalarType) and op.outputs[0].type.dtype == "int64"
    op2 = OpBuilder.argmax(v, dim=1, dtype="int32")
    assert op2.outputs[0].type == TensorType((1,), "int32")


def test_verifier_reports_ssa_and_def_use_errors():
    f = Function("bad")
    x = OpBuilder.input("x", TensorType((4, 4), "float32")).outputs[0]
    f.add_input(x)
    f.add_input(x)
    ghost = OpBuilder.input("ghost", TensorType((4, 4), "float32")).outputs[0]
    f.add_op(OpBuilder.relu(ghost))
    v = IRVerifier(f)
    assert not v.verify()
    errs = " ".join(v.get_errors())
    assert "SSA violation" in errs and "Def-use error" in errs


def test_matmul_shape_mismatch_rejected():
    a = OpBuilder.input("a", TensorType((4, 8), "float32")).outputs[0]
    b = OpBuilder.input("b", TensorType((7, 2), "float32")).outputs[0]
    with pytest.raises(ValueError):
        OpBuilder.matmul(a, b)


def test_dsl_programs_match_reference_op_lists():
    @devproc.kernel
    def vision_preproc(img):
        img = devproc.resize(img, (224, 224))
        img = devproc.to(img, devproc.Float32)
        return img

    ir = devproc.parse_ir(vision_preproc, torch.randn(256, 256, 3))
    ref = GOLD["dsl_vision_preproc"]
    assert [o.name for o in ir.block.ops] == ref["ops"]
    assert [v.name for v in ir.inputs] == ref["inputs"]
    assert list(ir.output.type.shape) == ref["out_shape"]

    @devproc.kernel
    def mlp(x, w1, b1, w2, b2):
        h = devproc.relu(devproc.linear(x, w1, b1))
        return devproc.argmax(devproc.linear(h, w2, b2))

    ir = devproc.parse_ir(mlp, torch.randn(1, 128), torch.randn(256, 128), torch.randn(256),
                          torch.randn(10, 256), torch.randn(10))
    assert [o.name for o in ir.block.ops] == GOLD["dsl_mlp"]["ops"]
    assert [v.name for v in ir.inputs] == GOLD["dsl_mlp"]["inputs"]
    assert IRVerifier(ir).verify()


def test_fx_programs_match_reference_op_lists():
    class MLP(torch.nn.Module):
        def __init__(s):
            super().__init__()
            s.fc1 = torch.nn.Linear(128, 256)
            s.fc2 = torch.nn.Linear(256, 10)

        def forward(s, x):
            return s.fc2(torch.relu(s.fc1(x)))

    ir = devproc.from_torch(MLP(), torch.randn(1, 128), backend="ir")
    assert [o.name for o in ir.block.ops] == GOLD["fx_mlp"]["ops"]
    ir = devproc.from_torch(torch.nn.Sequential(torch.nn.Linear(128, 256), torch.nn.ReLU()),
                            torch.randn(1, 128), backend="ir")
    assert [o.name for o in ir.block.ops] == GOLD["fx_sequential"]["ops"]
    ir = devproc.from_torch(lambda x: torch.sigmoid(x), torch.randn(4, 8), backend="ir")
    assert [o.name for o in ir.block.ops] == GOLD["fx_sigmoid"]["ops"]


def test_fx_token_pipeline_shapes_and_constants():
    m = workloads.TokenPipeline()
    ir = devproc.from_torch(m, workloads.token_ids(), backend="ir")
    names = [o.name for o in ir.block.ops]
    assert names == ["embedding", "linear", "gelu", "linear", "layer_norm", "linear", "argmax", "to"]
    runtime_inputs = [v.name for v in ir.inputs if v.name not in ir.constants]
    assert runtime_inputs == ["l_ids_"]
    assert len(ir.constants) == 9
    assert ir.output.type == TensorType((8, 128), "int32")
    assert IRVerifier(ir).verify()


def test_fx_rejects_unknown_ops_loudly():
    with pytest.raises(ValueError, match="Unsupported FX function"):
        devproc.from_torch(lambda x: torch.cumsum(x, 0), torch.randn(4, 8), backend="ir")


def test_conv_patchify_lowered_to_linear():
    conv = torch.nn.Conv2d(3, 32, kernel_size=14, stride=14)
    ir = devproc.from_torch(conv, torch.randn(2, 3, 56, 56), backend="ir")
    names = [o.name for o in ir.block.ops]
    assert "linear" in names and names[-1] == "transpose"
    assert ir.output.type.shape == (2, 32, 4, 4)


def test_rows_touched_model():
    assert workloads.rows_touched(480, 224) == 448
    assert workloads.rows_touched(640, 224) == 448
