"""The oracle against the reference's own kernels (golden vectors) and against
an independent restatement of the bilinear arithmetic."""

import numpy as np
import torch
import torch.nn.functional as F

from devproc_b200.ir.function import Function
from devproc_b200.ir.ops import OpBuilder
from devproc_b200.ir.types import TensorType
from oracle import interp, preproc_np


def _run1(build, *tensors):
    """Build a one-op IR function over ``tensors`` and run the oracle on it."""
    fn = Function("t")
    vals = []
    for i, t in enumerate(tensors):
        v = OpBuilder.input(f"x{i}", TensorType(tuple(t.shape), str(t.dtype).replace("torch.", ""))).outputs[0]
        fn.add_input(v)
        vals.append(v)
    op = build(*vals)
    fn.add_op(op)
    fn.output = op.outputs[0]
    return interp.run_function(fn, {f"x{i}": t for i, t in enumerate(tensors)})[0]


def g(golden, case, key):
    return torch.from_numpy(golden[f"{case}/{key}"].copy())


def test_normalize_matches_reference_template(golden):
    for case in ("normalize_f32", "normalize_u8"):
        out = _run1(OpBuilder.normalize, g(golden, case, "x"))
        assert torch.equal(out, g(golden, case, "y"))


def test_relu_add_match_reference_exactly(golden):
    assert torch.equal(_run1(OpBuilder.relu, g(golden, "relu", "x")), g(golden, "relu", "y"))
    out = _run1(OpBuilder.add, g(golden, "add", "x"), g(golden, "add", "x2"))
    assert torch.equal(out, g(golden, "add", "y"))


def test_sigmoid_softmax_match_reference(golden):
    # tolerances: the reference's own test uses atol 1e-3 (test_triton.py:87, 179); the
    # interpreter's exp and torch's differ by a few ulp.
    out = _run1(OpBuilder.sigmoid, g(golden, "sigmoid", "x"))
    assert torch.allclose(out, g(golden, "sigmoid", "y"), rtol=1e-6, atol=1e-7)
    out = _run1(OpBuilder.softmax, g(golden, "softmax", "x"))
    assert torch.allclose(out, g(golden, "softmax", "y"), rtol=1e-5, atol=1e-8)


def test_cast_to_int_truncates_like_reference(golden):
    out = _run1(lambda v: OpBuilder.to(v, "int32"), g(golden, "to_i32", "x"))
    assert torch.equal(out, g(golden, "to_i32", "y"))


def test_argmax_bit_exact_with_reference(golden):
    for case in ("argmax_small", "argmax_wide", "argmax_ties"):
        out = _run1(lambda v: OpBuilder.argmax(v, -1, dtype="int64"), g(golden, case, "x"))
        assert torch.equal(out, g(golden, case, "y")), case


def test_sum_matches_reference(golden):
    x = g(golden, "sum", "x")
    out = _run1(lambda v: OpBuilder.reduce("sum", v, -1), x)
    tol = 1e-6 * x.abs().sum(-1)
    assert ((out - g(golden, "sum", "y")).abs() <= tol).all()


def test_matmul_linear_match_reference(golden):
    out = _run1(OpBuilder.matmul, g(golden, "matmul", "x"), g(golden, "matmul", "x2"))
    assert torch.allclose(out, g(golden, "matmul", "y"), rtol=1e-5, atol=1e-5)
    out = _run1(OpBuilder.linear, g(golden, "linear", "x"), g(golden, "linear", "x2"), g(golden, "linear", "b"))
    assert torch.allclose(out, g(golden, "linear", "y"), rtol=1e-5, atol=1e-5)


def test_argmax_nan_and_ties_semantics():
    x = torch.tensor([[1.0, 3.0, 3.0, 2.0], [1.0, float("nan"), 5.0, float("nan")], [-1.0, -1.0, -1.0, -1.0]])
    out = _run1(lambda v: OpBuilder.argmax(v, -1, dtype="int64"), x)
    assert out.tolist() == [1, 1, 0]


def test_bilinear_restatement_within_four_ulp_of_torch():
    """torch's CPU result depends on its thread chunking (vectorised FMA body vs
    scalar tail, whose rounding differs by up to 3 ulp); the restatement
    follows the vectorised arithmetic and stays within 4 ulp (3e-5 absolute
    at pixel values up to 255) of torch at every thread count."""
    gen = torch.Generator().manual_seed(0)
    sizes = [(480, 640, 224, 224), (37, 53, 224, 99), (224, 224, 224, 224), (96, 128, 56, 64), (5, 7, 3, 2),
             (1, 9, 4, 4), (17, 300, 5, 77)]
    old = torch.get_num_threads()
    try:
        for threads in (1, old):
            torch.set_num_threads(threads)
            for (H, W, OH, OW) in sizes:
                x = torch.randint(0, 256, (2, H, W, 3), generator=gen, dtype=torch.uint8)
                ref = F.interpolate(x.permute(0, 3, 1, 2).float(), (OH, OW), mode="bilinear",
                                    align_corners=False).numpy()
                mine = preproc_np.resize_nhwc(x.numpy(), OH, OW).transpose(0, 3, 1, 2)
                ulp = np.spacing(np.abs(ref).astype(np.float32))
                assert (np.abs(mine - ref) <= 4 * ulp).all(), (threads, H, W, OH, OW)
    finally:
        torch.set_num_threads(old)


def test_bilinear_restatement_equal_sizes_copy_exactly():
    x = torch.randint(0, 256, (1, 31, 17, 3), dtype=torch.uint8)
    assert np.array_equal(preproc_np.resize_nhwc(x.numpy(), 31, 17), x.numpy().astype(np.float32))


def test_preprocess_oracle_agrees_with_restatement():
    gen = torch.Generator().manual_seed(1)
    x = torch.randint(0, 256, (2, 96, 128, 3), generator=gen, dtype=torch.uint8)
    mean = [0.485 * 255, 0.456 * 255, 0.406 * 255]
    std = [0.229 * 255, 0.224 * 255, 0.225 * 255]
    fn = Function("pre")
    v = OpBuilder.input("img", TensorType(tuple(x.shape), "uint8")).outputs[0]
    fn.add_input(v)
    ops = [OpBuilder.resize(v, (56, 64))]
    ops.append(OpBuilder.normalize(ops[-1].outputs[0], mean, std))
    ops.append(OpBuilder.transpose(ops[-1].outputs[0], (0, 3, 1, 2)))
    for o in ops:
        fn.add_op(o)
    fn.output = ops[-1].outputs[0]
    out = interp.run_function(fn, {"img": x})[0]
    mine = preproc_np.preprocess_nhwc(x.numpy(), 56, 64, mean, std)
    assert np.array_equal(out.numpy(), mine)
