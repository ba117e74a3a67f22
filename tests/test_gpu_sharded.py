"""``ShardedRuntime`` on two GPUs (NCCL): the gathered result equals one GPU's.

Two processes, one per GPU, each run their shard of a global batch of images
through the preprocessing pipeline and gather to rank 0 with ``run`` (three
steps, so both program copies and both gather buffers are used).  Rank 0's
gathered bits of every step must equal a single-GPU run of the whole batch.
Skipped when fewer than two GPUs are visible.
"""

import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

from devproc_b200 import workloads

pytestmark = pytest.mark.gpu

STEPS = 3


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _global_batch(step):
    return workloads.preprocess_images(16, seed=300 + step)


def _worker(rank, world, port, q):
    import datetime
    import torch.distributed as dist
    os.environ.update({"MASTER_ADDR": "127.0.0.1", "MASTER_PORT": str(port), "RANK": str(rank),
                       "WORLD_SIZE": str(world), "LOCAL_RANK": str(rank)})
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", device_id=dev, timeout=datetime.timedelta(seconds=60))
    try:
        import devproc
        mine = devproc.shard_batch(_global_batch(0), rank, world)
        rt = devproc.ShardedRuntime(workloads.vision_preprocess, mine)
        got = []
        for step in range(STEPS):
            out = rt.run(images=rt.shard_batch(_global_batch(step)).to(dev))
            rt.synchronize()
            if rank == 0:
                got.append(out[0].cpu().view(torch.int16).numpy().copy())
        rt.close()
        if rank == 0:
            q.put(("ok", got))
    except Exception as e:
        q.put(("err", f"rank {rank}: {type(e).__name__}: {e}"))
    finally:
        dist.destroy_process_group()


def test_two_gpu_gather_equals_one_gpu(cuda):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    import devproc
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    import queue as _queue
    try:
        res = q.get(timeout=300)
    except _queue.Empty:
        res = ("err", "no result within 300 s")
    for p in procs:
        p.join(timeout=120)
        if p.is_alive():
            p.kill()
    assert res[0] == "ok", res[1]
    whole = devproc.compile(workloads.vision_preprocess, _global_batch(0))
    for step in range(STEPS):
        ref = whole.run(images=_global_batch(step))[0].view(torch.int16).numpy()
        assert (res[1][step] == ref).all(), f"step {step}"
