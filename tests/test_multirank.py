"""Batch sharding and the final gather of ``ShardedRuntime`` on 2 gloo ranks (CPU).

Each rank builds ``devproc.ShardedRuntime`` for its shard of a global batch of
images, exactly as a GPU job does, and runs several steps through ``run``:
the product's shard selection, double-buffered program alternation and
gather-to-rank-0 code.  On the CPU the compiled plan cannot execute, so the
runtime wraps a stand-in program that evaluates the same IR with the CPU
oracle; everything else is the product's code.  Rank 0's gathered result of
every step must equal the single-process oracle result of the global batch;
a rank that fails must surface as an error instead of a hang.
"""

import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from devproc_b200 import workloads


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


class _OracleProgram:
    """CPU stand-in for a compiled program: same spec, the oracle computes."""

    def __init__(self, prog, ir):
        self.spec, self.ir, self.device_id = prog.spec, ir, None
        self.runs = 0

    def run(self, *args, to_cpu=True, **kwargs):
        from oracle import interp
        self.runs += 1
        return interp.run_function(self.ir, kwargs)

    def clone(self):
        return _OracleProgram(self, self.ir)

    def synchronize(self):
        pass

    def close(self):
        pass


def _global_batch(step):
    return workloads.preprocess_images(8, 48, 64, seed=100 + step)


def _worker(rank, world, port, fail_rank, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    import datetime
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=30))
    try:
        import devproc
        mine0 = devproc.shard_batch(_global_batch(0), rank, world)
        assert mine0.shape[0] == 8 // world
        prog = devproc.compile(workloads.vision_preprocess, mine0)  # host-only: the plan this rank would run
        assert [r["kernel"] for r in prog.spec.records] == ["preproc"]
        ir = devproc.parse_ir(workloads.vision_preprocess, mine0)
        rt = devproc.ShardedRuntime(program=_OracleProgram(prog, ir), gather=True)
        assert (rt.rank, rt.world_size) == (rank, world) and rt.global_batch() == 8
        if rank == fail_rank:
            raise RuntimeError("injected failure on rank %d" % rank)
        results = []
        for step in range(3):
            out = rt.run(images=rt.shard_batch(_global_batch(step)))
            if rank == 0:
                results.append(out[0].float().numpy().copy())
        rt.synchronize()
        assert [p.runs for p in rt._progs] == [2, 1]  # the two program copies alternate
        if rank == 0:
            q.put(("ok", results))
    except Exception as e:  # report, then let the process group time out on the others
        q.put(("err", f"rank {rank}: {e}"))
    finally:
        try:
            dist.destroy_process_group()
        except Exception:
            pass


def _run(world, fail_rank=-1):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, fail_rank, q)) for r in range(world)]
    for p in procs:
        p.start()
    out = []
    import queue as _queue
    for _ in range(world):
        try:
            out.append(q.get(timeout=120))
        except _queue.Empty:
            break
        if out[-1][0] == "ok":
            break
    for p in procs:
        p.join(timeout=60)
    for p in procs:
        if p.is_alive():
            p.kill()
    return out


def test_sharded_runtime_gathers_every_step_to_rank0():
    results = _run(2)
    oks = [r for r in results if r[0] == "ok"]
    assert len(oks) == 1, results
    import devproc
    from oracle import interp
    for step, got in enumerate(oks[0][1]):
        imgs = _global_batch(step)
        ir = devproc.parse_ir(workloads.vision_preprocess, imgs)
        full = interp.run_function(ir, {"images": imgs})[0].float()
        assert torch.equal(torch.from_numpy(got), full), f"step {step}"


def test_failing_rank_is_reported_not_hung():
    results = _run(2, fail_rank=1)
    errs = [r for r in results if r[0] == "err"]
    assert any("injected failure on rank 1" in e[1] for e in errs), results


def test_shard_ranges():
    import devproc
    assert [devproc.shard_range(256, r, 8) for r in (0, 7)] == [(0, 32), (224, 256)]
    with pytest.raises(ValueError):
        devproc.shard_range(10, 0, 4)
    with pytest.raises(ValueError):
        devproc.shard_range(8, 2, 2)
