"""Benchmark of the compiled-pipeline hot path on B200.

Default workload: the vision preprocessing pipeline — uint8 NHWC images
[256, 480, 640, 3] → bilinear 224×224 → fp32 → (x - mean) / std → CHW → bf16
[256, 3, 224, 224] — compiled with ``devproc.compile`` and run through the
program.  One step = one pass over one 256-image batch per GPU.  With
``--gpus N`` (launched under torchrun, one process per GPU) every rank runs
its own 256-image shard: weak scaling, no collective on the data path.

Prints ONE JSON line (rank 0):
  value          images/s of the whole job, inputs resident in HBM, device
                 time (CUDA events) of K steps, max over ranks;
  e2e            the same metric through ``Runtime.run`` with pinned host
                 buffers: host→device copy of the images and device→host
                 read of the result inside every timed step;
  roofline       achieved HBM GB/s of the preprocessing kernel (algorithmic
                 bytes per launch ÷ CUDA-event time per launch) against the
                 measured copy bandwidth;
  cpu_baseline   the same pipeline with torch on the host cores, on a
                 bounded sample of the batch.
``--impl reference`` times only that CPU path (rank 0; other ranks exit).
"""

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import threading
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

import torch  # noqa: E402

FALLBACK_HBM_GBS = 6650.0


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10000)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["b200", "reference"], default="b200")
    ap.add_argument("--batch", type=int, default=256)
    ap.add_argument("--cpu-sample", type=int, default=64, help="images in the CPU-baseline sample")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    return ap.parse_args()


def dist_env():
    return int(os.environ.get("RANK", 0)), int(os.environ.get("LOCAL_RANK", 0)), int(os.environ.get("WORLD_SIZE", 1))


def peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return float(d["hbm_gbs"]), "measured"
    return FALLBACK_HBM_GBS, "fallback"


def ncu_traffic():
    """Per-launch DRAM bytes of the preprocessing kernel from the committed ncu summary."""
    p = ROOT / "profiles" / "preproc_c2_ncu.md"
    if not p.exists():
        return None
    for line in p.read_text().splitlines():
        if line.startswith("traffic_bytes_per_launch_full_batch:"):
            return int(float(line.split(":")[1].strip()))
    return None


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled every 200 ms during the timed region."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.path = None

    def __enter__(self):
        fd, self.path = tempfile.mkstemp(suffix=".csv")
        os.close(fd)
        try:
            self.proc = subprocess.Popen(["nvidia-smi", "-i", str(self.gpu), f"--query-gpu={self.Q}",
                                          "--format=csv,noheader,nounits", "-lms", "200"],
                                         stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except OSError:
            self.proc = None
            return self
        # Start timing only once the sampler is producing lines.
        t0 = time.time()
        while time.time() - t0 < 5 and os.path.getsize(self.path) == 0:
            time.sleep(0.05)
        with open(self.path) as f:
            self.skip = len(f.readlines())
        return self

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self):
        if self.proc is None or not self.path or not os.path.exists(self.path):
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in open(self.path).readlines()[getattr(self, "skip", 0):]:
            f = [x.strip() for x in line.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx = float(f[2])
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        os.unlink(self.path)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm)}


def cpu_baseline_run(images, n_steps, sample):
    from oracle import cpu_pipeline
    from devproc_b200 import workloads
    cores = cpu_pipeline.use_all_threads()
    x = images[:sample].contiguous()
    cpu_pipeline.preprocess(x[:4], mean=workloads.IMAGENET_MEAN, std=workloads.IMAGENET_STD)  # warm
    times = []
    for _ in range(n_steps):
        t0 = time.perf_counter()
        cpu_pipeline.preprocess(x, mean=workloads.IMAGENET_MEAN, std=workloads.IMAGENET_STD)
        times.append(time.perf_counter() - t0)
    return sample / statistics.median(times), cores


def reference_arm(args):
    rank, _, world = dist_env()
    if rank != 0:
        return
    from devproc_b200 import workloads
    images = workloads.preprocess_images(args.cpu_sample)
    for _ in range(max(args.warmup, 1)):
        cpu_baseline_run(images, 1, args.cpu_sample)
    value, cores = cpu_baseline_run(images, max(args.steps, 1), args.cpu_sample)
    sample = f"{args.cpu_sample} of the {args.batch} images (480x640x3 u8) per step, torch CPU ops"
    line = {
        "impl": "reference", "metric": "pipeline samples/sec (vision preprocessing)", "value": value,
        "unit": "images/s", "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "u8->f32->bf16",
        "data": "synthetic (seeded uniform uint8 images)",
        "config": {"workload": "vision_preprocess 480x640x3 u8 -> 3x224x224 bf16", "global_batch": args.batch,
                   "parallelism": "host cores"},
        "cpu_baseline": {"value": value, "unit": "images/s", "cores": cores, "kind": "port", "sample": sample},
        "e2e": {"value": value, "unit": "images/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def main():
    args = parse()
    if args.impl == "reference":
        return reference_arm(args)
    rank, local_rank, world = dist_env()
    if world != args.gpus:
        if world == 1 and args.gpus > 1:
            raise SystemExit("--gpus N > 1 must be launched with torchrun (one process per GPU)")
    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    if world > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl", device_id=dev, timeout=datetime.timedelta(seconds=120))

    import devproc
    from devproc_b200 import workloads

    B = args.batch
    images_host = workloads.preprocess_images(B, seed=rank)
    prog = devproc.compile(workloads.vision_preprocess, images_host, device_id=local_rank)
    n_launch_per_step = len(prog.spec.records)
    # Two device-resident input batches used alternately: 2 × 236 MB > 126 MB L2.
    dev_in = [images_host.to(dev), workloads.preprocess_images(B, seed=1000 + rank).to(dev)]
    stream = torch.cuda.current_stream(dev)

    def barrier():
        if world > 1:
            import torch.distributed as dist
            dist.barrier()

    def max_over_ranks(x):
        if world == 1:
            return x
        import torch.distributed as dist
        t = torch.tensor([x], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return t.item()

    for i in range(max(args.warmup, 3)):
        prog.run(images=dev_in[i % 2], to_cpu=False)
    torch.cuda.synchronize()

    # ---- device-resident timed region
    K = args.steps
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(K + 1)]
    barrier()
    torch.cuda.synchronize()
    with ClockSampler(local_rank) as clk:
        ev[0].record(stream)
        for i in range(K):
            prog.run(images=dev_in[i % 2], to_cpu=False)
            ev[i + 1].record(stream)
        torch.cuda.synchronize()
    barrier()
    per_step = [ev[i].elapsed_time(ev[i + 1]) for i in range(K)]
    total_ms = max_over_ranks(ev[0].elapsed_time(ev[K]))
    clocks = clk.summary()
    value = B * world * K / (total_ms / 1e3)

    # ---- end to end: pinned host images in, host result out, through Runtime.run
    rt = devproc.Runtime(prog, device_id=local_rank)
    host_in = [images_host.pin_memory(), workloads.preprocess_images(B, seed=2000 + rank).pin_memory()]
    for i in range(2):
        rt.run(images=host_in[i % 2], reuse_host_buffers=True)
    barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for i in range(K):
        outs = rt.run(images=host_in[i % 2], reuse_host_buffers=True)
    e1.record(stream)
    torch.cuda.synchronize()
    barrier()
    e2e_ms = max_over_ranks(e0.elapsed_time(e1))
    e2e_value = B * world * K / (e2e_ms / 1e3)
    h2d = images_host.numel() * images_host.element_size()
    d2h = sum(o.numel() * o.element_size() for o in outs)

    # ---- roofline of the preprocessing kernel (one launch per step)
    bytes_per_launch = B * workloads.PREPROC_BYTES_PER_IMAGE
    launch_ms = statistics.mean(per_step) / n_launch_per_step
    achieved = bytes_per_launch / (launch_ms / 1e3) / 1e9
    peak, peak_kind = peaks()

    line = None
    if rank == 0:
        cpu = None
        if not args.no_cpu_baseline and world == 1:
            v, cores = cpu_baseline_run(images_host, 3, args.cpu_sample)
            cpu = {"value": v, "unit": "images/s", "cores": cores, "kind": "port",
                   "sample": f"{args.cpu_sample} of the {B} images per step, median of 3, torch CPU ops "
                             "(F.interpolate bilinear, normalise, bf16)"}
        line = {
            "metric": "pipeline samples/sec (vision preprocessing)", "value": value, "unit": "images/s",
            "n_gpus": world, "steps": K, "warmup": max(args.warmup, 3), "ms_per_step": total_ms / K,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "u8->f32->bf16",
            "data": "synthetic (seeded uniform uint8 images)",
            "config": {"workload": "vision_preprocess 256x480x640x3 u8 -> 256x3x224x224 bf16 (normalise, CHW)",
                       "global_batch": B * world, "per_gpu_batch": B,
                       "parallelism": f"dp{world} batch-sharded, no collective",
                       "l2": "inputs larger than L2: two 236 MB input batches alternate"},
            "e2e": {"value": e2e_value, "unit": "images/s", "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                    "path": "Runtime.run(images=pinned host uint8) -> pinned host bf16"},
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                         "frac": achieved / peak, "traffic": ncu_traffic(), "peak_kind": peak_kind,
                         "kernel": "preproc_bulk_kernel<u8,bf16,NHWC->NCHW>",
                         "algorithmic_bytes_per_launch": bytes_per_launch},
            "cpu_baseline": cpu,
            "clocks": clocks,
            "gpu_launches": K * n_launch_per_step,
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        import torch.distributed as dist
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
