"""A kernel whose bounded wait runs out reports it, and the program stays usable.

The staged fp32 softmax kernel waits on one mbarrier per row copy.  The
library's failure-detection switch (``dp_test_withhold_copies``) makes it arm
those barriers without issuing the copies, so every wait can end only by its
limit, set here to 1 ms with ``dp_set_wait_limit``.  ``run`` must then raise
DevProcError naming the timeout and the wait site (700), instead of handing
back a partial result as the reference's silent skip did
(src/devproc/backend/triton/compiler.py:302-304, 343-346).  With the switch
cleared and the default limit restored, the same program (same arena, same
CUDA graph) must give the oracle's result again.

Nothing here faults or hangs a GPU: every wait is bounded, the switch issues
no copy at all, and the kernel's exit-time drain wait has its own 100 ms limit.
"""

import pytest
import torch

import devproc
from devproc_b200 import _native as N
from oracle import interp

pytestmark = pytest.mark.gpu

SITE_STAGED_ROW_WAIT = 700


class _Softmax(torch.nn.Module):
    def forward(self, x):
        return torch.softmax(x, dim=-1)


def _program(rows=1024, cols=1024):
    """fp32 softmax over enough rows (>= 4 per SM) to take the staged kernel."""
    x = torch.randn(rows, cols, generator=torch.Generator().manual_seed(11))
    m = _Softmax()
    prog = devproc.compile(m, x)
    assert [r["kernel"] for r in prog.spec.records] == ["rowreduce"]
    ir = devproc.from_torch(m, x, backend="ir")
    ref = interp.run_function(ir, {ir.inputs[0].name: x})[0]
    return prog, x, ref


def test_timed_out_wait_raises_and_program_recovers(cuda):
    prog, x, ref = _program()
    # a healthy run first: the CUDA graph of the program is captured on later runs
    for _ in range(3):
        got = prog.run(x)[0]
    torch.testing.assert_close(got, ref, rtol=1e-5, atol=1e-7)
    try:
        N.set_wait_limit(0, 1_000_000)  # 1 ms
        N.test_withhold_copies(0, True)
        with pytest.raises(N.DevProcError) as e:
            prog.run(x)
        assert e.value.status == N.DP_ERR_DEVICE
        assert "bounded wait" in str(e.value) and f"site {SITE_STAGED_ROW_WAIT}" in str(e.value)
        # the error word was read and cleared by run()
        assert N.device_error_pending(0) == N.DP_DEVERR_NONE
    finally:
        N.test_withhold_copies(0, False)
        N.set_wait_limit(0, 0)
    for _ in range(2):
        got = prog.run(x)[0]
        torch.testing.assert_close(got, ref, rtol=1e-5, atol=1e-7)
    assert N.device_error_pending(0) == N.DP_DEVERR_NONE


def test_async_runs_report_through_synchronize(cuda):
    prog, x, ref = _program()
    d = x.to(cuda)
    prog.run(d, to_cpu=False)
    prog.synchronize()
    try:
        N.set_wait_limit(0, 1_000_000)
        N.test_withhold_copies(0, True)
        prog.run(d, to_cpu=False)  # enqueued only: nothing raised yet
        with pytest.raises(N.DevProcError, match="bounded wait"):
            prog.synchronize()
    finally:
        N.test_withhold_copies(0, False)
        N.set_wait_limit(0, 0)
    out = prog.run(d, to_cpu=False)[0]
    prog.synchronize()
    torch.testing.assert_close(out.cpu(), ref, rtol=1e-5, atol=1e-7)
