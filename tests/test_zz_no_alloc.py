"""The allocation-free plan runner, called through the C ABI.

Some callers cannot allocate device memory at run time (a host application
that owns all device memory, a loop that must not enter the driver's
allocator).  ``dp_program_run_noalloc`` runs a compiled plan with its
intermediates in a fixed static array inside the library instead of an
arena from cudaMalloc.  These tests run small plans through it twice in a row
and check both results against the regular entry point (``dp_program_run``
behind ``CompiledProgram.run``; the same kernels on the same inputs, so the
results must be identical) and against the CPU oracle interpreter.  One plan
reads a slice of its input through a sub-range slot, which the caller binds
at the input's pointer plus the slice's byte offset.

Named so that pytest collects it last.
"""

import ctypes

import pytest
import torch

import devproc
from devproc_b200 import _native as N
from devproc_b200 import workloads
from oracle import interp

pytestmark = pytest.mark.gpu


def _bound_buffers(prog, inputs, outputs):
    """Caller buffers of every bound slot in slot order: inputs, constants,
    outputs, and each sub-range slot at its root's pointer plus the offset."""
    by_slot = {}
    for io, t in zip(prog.spec.inputs, inputs):
        by_slot[io.slot] = (t.data_ptr(), t.numel() * t.element_size())
    for c in prog.spec.consts:
        t = prog._dev_consts[c.name]
        by_slot[c.slot] = (t.data_ptr(), t.numel() * t.element_size())
    for o, t in zip(prog.spec.outputs, outputs):
        by_slot[o.slot] = (t.data_ptr(), t.numel() * t.element_size())
    for slot, root, off in prog.spec.aliases:
        ptr, nbytes = by_slot[root]
        by_slot[slot] = (ptr + off, nbytes - off)
    order = sorted(by_slot)
    ptrs = (ctypes.c_void_p * len(order))(*[by_slot[s][0] for s in order])
    sizes = (ctypes.c_uint64 * len(order))(*[by_slot[s][1] for s in order])
    return ptrs, sizes, len(order)


def _run_noalloc(prog, inputs, fill):
    dev = inputs[0].device
    outs = [torch.full(tuple(o.shape), fill, dtype=getattr(torch, o.dtype), device=dev) for o in prog.spec.outputs]
    ptrs, sizes, n = _bound_buffers(prog, inputs, outs)
    plan = prog.spec.plan
    st = N.lib().dp_program_run_noalloc(plan, len(plan), ptrs, sizes, n, torch.cuda.current_stream(dev).cuda_stream)
    N.check(st, "dp_program_run_noalloc")
    torch.cuda.synchronize()
    assert N.device_error_pending(0) == N.DP_DEVERR_NONE
    return outs


def _runtime_input(ir):
    return [v.name for v in ir.inputs if v.name not in ir.constants][0]


def _gpu():
    if not torch.cuda.is_available():
        pytest.fail("GPU test run without a visible CUDA device")
    N.device_init(0)
    return torch.device("cuda", 0)


def test_noalloc_plan_runner_matches_regular_runner_and_oracle():
    dev = _gpu()
    m = workloads.TokenPipeline().eval()
    ids = workloads.token_ids(2, 16)
    prog = devproc.compile(m, ids)
    assert 0 < prog.spec.arena_bytes <= N.DP_NOALLOC_ARENA_BYTES
    ids_dev = ids.to(dev)
    ref = prog.run(ids_dev, to_cpu=False)[0].clone()  # regular entry point (arena from cudaMalloc)
    prog.synchronize()
    ir = devproc.from_torch(m, ids, backend="ir")
    oracle = interp.run_function(ir, {_runtime_input(ir): ids})[0]
    # fp32 logits: rows whose top-2 gap is above the float tolerance must match the oracle exactly
    with torch.no_grad():
        logits = m.head(m.ln(m.fc2(torch.nn.functional.gelu(m.fc1(m.emb(ids.long()))))))
    top2 = logits.topk(2, dim=-1).values
    decided = (top2[..., 0] - top2[..., 1]) > 1e-4 * logits.abs().max()
    assert decided.float().mean() > 0.9
    for call in range(2):
        out = _run_noalloc(prog, [ids_dev], -1)[0]
        assert torch.equal(out, ref), f"call {call}: no-alloc result differs from the regular runner"
        assert torch.equal(out.cpu()[decided], oracle[decided]), f"call {call}: differs from the oracle"


class _SliceLinearSoftmax(torch.nn.Module):
    def __init__(self):
        super().__init__()
        self.lin = torch.nn.Linear(64, 48)

    def forward(self, x):
        return torch.softmax(self.lin(x[8:]), dim=-1)


def test_noalloc_binds_sub_range_slots():
    dev = _gpu()
    torch.manual_seed(3)
    m = _SliceLinearSoftmax().eval()
    x = torch.randn(24, 64)
    prog = devproc.compile(m, x)
    assert prog.spec.aliases, "the slice x[8:] should be a sub-range slot of the input"
    ref = prog.run(x)[0]
    ir = devproc.from_torch(m, x, backend="ir")
    oracle = interp.run_function(ir, {_runtime_input(ir): x})[0]
    torch.testing.assert_close(ref, oracle, rtol=1e-4, atol=1e-6)
    xd = x.to(dev)
    for call in range(2):
        out = _run_noalloc(prog, [xd], float("nan"))[0]
        assert torch.equal(out.cpu(), ref), f"call {call}: no-alloc result differs from the regular runner"
        torch.testing.assert_close(out.cpu(), oracle, rtol=1e-4, atol=1e-6)


class _ScaledSoftmax(torch.nn.Module):
    def forward(self, x):
        return torch.softmax(x * 2.0, dim=-1)


def test_noalloc_rejects_plans_over_the_limit():
    _gpu()
    prog = devproc.compile(_ScaledSoftmax(), torch.zeros(8192, 4096))  # the scaled input is a 128 MiB intermediate
    assert prog.spec.arena_bytes > N.DP_NOALLOC_ARENA_BYTES
    plan = prog.spec.plan
    st = N.lib().dp_program_run_noalloc(plan, len(plan), None, None, 0, None)
    assert st == N.DP_ERR_UNSUPPORTED
    assert "static arena holds" in N.last_error()


def test_noalloc_checks_buffers_before_enqueuing():
    _gpu()
    m = _SliceLinearSoftmax().eval()
    prog = devproc.compile(m, torch.randn(24, 64))
    plan = prog.spec.plan
    n_bound = sum(1 for _ in prog.spec.inputs) + len(prog.spec.consts) + len(prog.spec.outputs) + \
        len(prog.spec.aliases)
    ptrs = (ctypes.c_void_p * (n_bound - 1))(*([16] * (n_bound - 1)))  # one buffer short: never dereferenced
    st = N.lib().dp_program_run_noalloc(plan, len(plan), ptrs, None, n_bound - 1, None)
    assert st == N.DP_ERR_ARG and "fewer buffers" in N.last_error()
