"""The allocation-free plan runner, called through the C ABI.

Some callers cannot allocate device memory at run time (a host application
that owns all device memory, a loop that must not enter the driver's
allocator).  ``dp_program_run_noalloc`` runs a compiled plan with its
intermediates in a fixed static array inside the library instead of an
arena from cudaMalloc.  This test runs a small fp32 token pipeline through it
twice in a row and checks both results against the regular entry point
(``dp_program_run`` behind ``CompiledProgram.run``): the same kernels run on
the same inputs, so the int32 argmax output must match exactly.

Named so that pytest collects it last.
"""

import ctypes

import pytest
import torch

import devproc
from devproc_b200 import _native as N
from devproc_b200 import workloads

pytestmark = pytest.mark.gpu


def _bound_buffers(prog, ids_dev, out_dev):
    """Caller buffers of every bound slot, in slot order."""
    by_slot = {}
    for io in prog.spec.inputs:
        by_slot[io.slot] = ids_dev
    for c in prog.spec.consts:
        by_slot[c.slot] = prog._dev_consts[c.name]
    for o in prog.spec.outputs:
        by_slot[o.slot] = out_dev
    order = sorted(by_slot)
    ptrs = (ctypes.c_void_p * len(order))(*[by_slot[s].data_ptr() for s in order])
    sizes = (ctypes.c_uint64 * len(order))(*[by_slot[s].numel() * by_slot[s].element_size() for s in order])
    return ptrs, sizes, len(order)


def test_noalloc_plan_runner_matches_regular_runner():
    if not torch.cuda.is_available():
        pytest.fail("GPU test run without a visible CUDA device")
    N.device_init(0)
    dev = torch.device("cuda", 0)
    m = workloads.TokenPipeline().eval()
    ids = workloads.token_ids(2, 16)
    prog = devproc.compile(m, ids)
    assert 0 < prog.spec.arena_bytes <= N.DP_NOALLOC_ARENA_BYTES
    ids_dev = ids.to(dev)
    ref = prog.run(ids_dev, to_cpu=False)[0].clone()  # regular entry point (arena from cudaMalloc)
    torch.cuda.synchronize()

    plan = prog.spec.plan
    stream = torch.cuda.current_stream(dev).cuda_stream
    for call in range(2):
        out = torch.full(tuple(prog.spec.outputs[0].shape), -1, dtype=torch.int32, device=dev)
        ptrs, sizes, n = _bound_buffers(prog, ids_dev, out)
        st = N.lib().dp_program_run_noalloc(plan, len(plan), ptrs, sizes, n, stream)
        N.check(st, "dp_program_run_noalloc")
        torch.cuda.synchronize()
        assert torch.equal(out, ref), f"call {call}: no-alloc result differs from the regular runner"


def test_noalloc_rejects_plans_over_the_limit():
    if not torch.cuda.is_available():
        pytest.fail("GPU test run without a visible CUDA device")
    N.device_init(0)
    m = workloads.TokenPipeline().eval()
    prog = devproc.compile(m, workloads.token_ids())  # 8 x 128 tokens: logits alone are 131 MB
    assert prog.spec.arena_bytes > N.DP_NOALLOC_ARENA_BYTES
    plan = prog.spec.plan
    st = N.lib().dp_program_run_noalloc(plan, len(plan), None, None, 0, None)
    assert st == N.DP_ERR_UNSUPPORTED
    assert "static arena holds" in N.last_error()
