"""Batch sharding across ranks (host side, 2 gloo ranks on the CPU).

Each rank of the weak-scaled pipeline compiles the same program and runs its
own shard of images; results are combined only for checking.  Here the ranks
run the compile step and the CPU oracle on their shard and gather through
gloo: the union of the shards must equal the single-process result, a rank
that fails must surface as an error on the others, and no data-path
collective is needed for correctness.
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


def _shard(total, rank, world):
    per = total // world
    return rank * per, (rank + 1) * per


def _worker(rank, world, port, fail_rank, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    import datetime
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=30))
    try:
        import devproc
        from oracle import interp
        imgs = workloads.preprocess_images(8, 48, 64, seed=0)
        lo, hi = _shard(8, rank, world)
        mine = imgs[lo:hi]
        ir = devproc.parse_ir(workloads.vision_preprocess, mine)
        prog = devproc.compile(workloads.vision_preprocess, mine)
        assert [r["kernel"] for r in prog.spec.records] == ["preproc"]
        if rank == fail_rank:
            raise RuntimeError("injected failure on rank %d" % rank)
        out = interp.run_function(ir, {"images": mine})[0].float()
        gathered = [torch.empty_like(out) for _ in range(world)]
        dist.all_gather(gathered, out)
        if rank == 0:
            q.put(("ok", torch.cat(gathered).numpy().copy()))
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


def test_two_rank_shards_equal_single_process():
    results = _run(2)
    oks = [r for r in results if r[0] == "ok"]
    assert len(oks) == 1, results
    import devproc
    from oracle import interp
    imgs = workloads.preprocess_images(8, 48, 64, seed=0)
    ir = devproc.parse_ir(workloads.vision_preprocess, imgs)
    full = interp.run_function(ir, {"images": imgs})[0].float()
    assert torch.equal(torch.from_numpy(oks[0][1]), full)


def test_failing_rank_is_reported_not_hung():
    results = _run(2, fail_rank=1)
    errs = [r for r in results if r[0] == "err"]
    assert any("injected failure on rank 1" in e[1] for e in errs), results
