"""Batch-sharded execution of one compiled pipeline over the GPUs of a node.

The reference runs every program on one device (``device_id``,
src/devproc/backend/triton/compiler.py:452-461); samples of the benchmark
pipelines are independent, so a job of G processes (one per GPU, launched by
torchrun) splits the global batch into G equal shards along dim 0:

* every rank compiles the same pipeline for its shard's shape and runs it on
  its own GPU, with no collective on the data path (``run_local``);
* ``run`` also brings every rank's outputs to rank 0 — the one collective the
  path has — over the process group (NCCL over NVLink on GPUs, gloo on the
  CPU in tests).  The gather of step i runs on a side stream while step i+1
  computes: two copies of the program alternate, so an output buffer is
  rewritten only after the gather that reads it has finished, and rank 0 keeps
  two gather buffers, so step i's result stays valid until step i+2.

The process group must already be initialised (``torch.distributed``) when
``world_size > 1``.  Every rank must call ``run`` / ``run_local`` the same
number of times in the same order.
"""

from typing import Dict, List, Optional, Sequence

import torch


def shard_range(total: int, rank: int, world_size: int):
    """[lo, hi) of rank's shard of ``total`` samples (equal shards; the global
    batch must divide evenly, as every rank runs the same static-shape plan)."""
    if world_size < 1 or not 0 <= rank < world_size:
        raise ValueError(f"rank {rank} outside a world of {world_size}")
    if total % world_size:
        raise ValueError(f"global batch {total} does not split into {world_size} equal shards")
    per = total // world_size
    return rank * per, (rank + 1) * per


def shard_batch(x: torch.Tensor, rank: int, world_size: int) -> torch.Tensor:
    """Rank's shard of a global batch along dim 0 (a view)."""
    lo, hi = shard_range(x.shape[0], rank, world_size)
    return x[lo:hi]


def gather_to_root(outputs: Sequence[torch.Tensor], buffers: Optional[Sequence[torch.Tensor]], world_size: int,
                   rank: int, group=None) -> None:
    """Gather each of this rank's ``outputs`` into ``buffers`` (rank 0 only:
    [world_size · b, ...] per output, rank r's rows at [r·b, (r+1)·b)).
    One point-to-point gather per output on the process group's backend."""
    import torch.distributed as dist
    for i, out in enumerate(outputs):
        if rank == 0:
            parts = list(buffers[i].chunk(world_size, dim=0))
            dist.gather(out.contiguous(), gather_list=parts, dst=0, group=group)
        else:
            dist.gather(out.contiguous(), gather_list=None, dst=0, group=group)


def _dist_rank_world():
    import os
    try:
        import torch.distributed as dist
        if dist.is_available() and dist.is_initialized():
            return dist.get_rank(), dist.get_world_size()
    except Exception:
        pass
    return int(os.environ.get("RANK", 0)), int(os.environ.get("WORLD_SIZE", 1))


class ShardedRuntime:
    """One pipeline, batch-sharded over ``world_size`` ranks (one GPU each).

    ``ShardedRuntime(target, *shard_examples, ...)`` compiles ``target`` with
    ``devproc.compile`` for this rank's shard (the examples have the shard's
    shape), or wraps an already compiled ``program=``.  ``shard_batch`` cuts a
    global batch into this rank's shard.
    """

    def __init__(self, target=None, *shard_examples, program=None, rank: Optional[int] = None,
                 world_size: Optional[int] = None, device_id: Optional[int] = None, gather: bool = True,
                 group=None, **compile_kwargs):
        r, w = _dist_rank_world()
        self.rank = r if rank is None else rank
        self.world_size = w if world_size is None else world_size
        if device_id is None:
            import os
            device_id = int(os.environ.get("LOCAL_RANK", 0))
        self.device_id = device_id
        self.group = group
        if program is None:
            from . import compile as _compile
            program = _compile(target, *shard_examples, device_id=device_id, **compile_kwargs)
        self.program = program
        self.gather_enabled = gather and self.world_size > 1
        self.gather_kind = ("torch.distributed gather to rank 0 (NCCL point-to-point over NVLink on GPUs), on a side "
                            "stream overlapped with the next step") if self.gather_enabled else None
        self._progs = [program] + ([program.clone()] if self.gather_enabled else [])
        self._step = 0
        self._cuda = False  # set by the first run: whether the program's outputs live on a GPU
        self._comm = None
        self._done: List = []
        self._freed: List = []
        self._gbuf: List[List[torch.Tensor]] = []

    # ------------------------------------------------------------ data
    def shard_batch(self, x: torch.Tensor) -> torch.Tensor:
        return shard_batch(x, self.rank, self.world_size)

    def global_batch(self) -> int:
        return self.program.spec.inputs[0].shape[0] * self.world_size

    # ------------------------------------------------------------- run
    def run_local(self, *args, **kwargs) -> List[torch.Tensor]:
        """This rank's shard only; device outputs, enqueued (no collective)."""
        return self.program.run(*args, to_cpu=False, **kwargs)

    def _ensure_gather_state(self, outs):
        if self._gbuf:
            return
        if self._cuda:
            dev = torch.device("cuda", self.device_id)
            self._comm = torch.cuda.Stream(dev)
            self._done = [torch.cuda.Event() for _ in range(2)]
            self._freed = [torch.cuda.Event() for _ in range(2)]
        if self.rank == 0:
            self._gbuf = [[torch.empty((self.world_size * o.shape[0],) + tuple(o.shape[1:]), dtype=o.dtype,
                                       device=o.device) for o in outs] for _ in range(2)]
        else:
            self._gbuf = [[], []]

    def run(self, *args, **kwargs) -> List[torch.Tensor]:
        """Run this rank's shard and gather every output to rank 0.  Returns,
        on rank 0, the gathered device tensors [global batch, ...] of this
        step (complete after ``synchronize()``; valid until two steps later);
        on the other ranks, their local outputs."""
        if not self.gather_enabled:
            return self.run_local(*args, **kwargs)
        j = self._step % 2
        prog = self._progs[j]
        cur = None
        if self._cuda:
            cur = torch.cuda.current_stream(torch.device("cuda", self.device_id))
            if self._step >= 2:
                cur.wait_event(self._freed[j])  # the gather that read these outputs is done
        outs = prog.run(*args, to_cpu=False, **kwargs)
        if self._step == 0:
            self._cuda = outs[0].is_cuda
            cur = torch.cuda.current_stream(torch.device("cuda", self.device_id)) if self._cuda else None
        self._ensure_gather_state(outs)
        bufs = self._gbuf[j] if self.rank == 0 else None
        if self._cuda:
            self._done[j].record(cur)
            self._comm.wait_event(self._done[j])
            with torch.cuda.stream(self._comm):
                gather_to_root(outs, bufs, self.world_size, self.rank, self.group)
            self._freed[j].record(self._comm)
        else:
            gather_to_root(outs, bufs, self.world_size, self.rank, self.group)
        self._step += 1
        return list(bufs) if self.rank == 0 else outs

    def synchronize(self) -> None:
        """Wait for every enqueued step and gather; raise on a kernel error."""
        if self._cuda and self._comm is not None:
            torch.cuda.current_stream(torch.device("cuda", self.device_id)).wait_stream(self._comm)
        for p in self._progs:
            p.synchronize()

    def close(self) -> None:
        for p in self._progs[1:]:
            p.close()
        self._progs = self._progs[:1]
        self._gbuf = []
