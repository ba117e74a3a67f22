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
    ap.add_argument("--rows", type=int, default=65536, help="rows of the reduce workload (4096 fp32 columns)")
    ap.add_argument("--cpu-sample", type=int, default=64, help="images in the CPU-baseline sample")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--workload", choices=["preprocess", "gemm", "reduce", "token", "vit", "vla"],
                    default="preprocess",
                    help="preprocess = the headline pipeline; gemm / reduce / token = template microbenches "
                         "and the fp32 token pipeline")
    return ap.parse_args()


def dist_env():
    return int(os.environ.get("RANK", 0)), int(os.environ.get("LOCAL_RANK", 0)), int(os.environ.get("WORLD_SIZE", 1))


FALLBACK_BF16_TFLOPS = 1590.0


def peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return float(d["hbm_gbs"]), "measured"
    return FALLBACK_HBM_GBS, "fallback"


def tensor_peak():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return float(d["bf16_tflops"]), "measured (burst)"
    return FALLBACK_BF16_TFLOPS, "fallback"


def time_region(fn, steps, warmup, stream):
    """Average ms per call of ``fn`` over ``steps`` calls, CUDA events on ``stream``."""
    for _ in range(max(warmup, 3)):
        fn()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(steps):
        fn()
    e1.record(stream)
    torch.cuda.synchronize()
    return e0.elapsed_time(e1) / steps


def micro_gemm(args, dev):
    """bf16 × bf16 → bf16 GEMM, fp32 accumulate, B as [N, K] (tcgen05 kernel)."""
    from devproc_b200 import _native as N
    peak, kind = tensor_peak()
    out = {}
    stream = torch.cuda.current_stream(dev)
    for (M, Nn, K) in [(4096, 4096, 4096), (8192, 2048, 16384)]:
        g = torch.Generator(device=dev).manual_seed(0)
        a = torch.randn(M, K, device=dev, generator=g).bfloat16()
        b = torch.randn(Nn, K, device=dev, generator=g).bfloat16()
        c = torch.empty(M, Nn, device=dev, dtype=torch.bfloat16)
        p = N.GemmParams()
        p.M, p.N, p.K, p.lda, p.ldb, p.ldc, p.batch = M, Nn, K, K, K, Nn, 1
        p.a_dtype = p.b_dtype = p.c_dtype = N.DP_BF16
        p.b_layout = N.DP_B_NK
        sp = stream.cuda_stream
        ms = time_region(lambda: N.gemm(p, a, b, c, stream=sp), min(args.steps, 200), args.warmup, stream)
        tf = 2.0 * M * Nn * K / (ms / 1e3) / 1e12
        out[f"{M}x{Nn}x{K}"] = {"ms": ms, "tflops": tf, "frac": tf / peak}
    best = max(out.values(), key=lambda v: v["tflops"])
    return {"metric": "bf16 GEMM TFLOP/s (fp32 accumulate)", "value": out["4096x4096x4096"]["tflops"],
            "unit": "TFLOP/s", "higher_is_better": True, "dtype": "bf16", "shapes": out,
            "roofline": {"bound": "tensor", "achieved": best["tflops"], "peak": peak, "unit": "TFLOP/s",
                         "frac": best["tflops"] / peak, "peak_kind": kind, "kernel": "tc_gemm_kernel"},
            "config": {"workload": "GEMM 4096^3 and 8192x2048x16384, inputs N(0,1)"}}


def micro_reduce(args, dev):
    """Row reductions over fp32 [rows, 4096] (65536 rows by default)."""
    from devproc_b200 import _native as N
    peak, kind = peaks()
    rows, cols = args.rows, 4096
    g = torch.Generator(device=dev).manual_seed(0)
    x = torch.randn(rows, cols, device=dev, generator=g)
    ones = torch.ones(cols, device=dev)
    stream = torch.cuda.current_stream(dev)
    sp = stream.cuda_stream
    res = {}
    for name, kind_c, odt, nbytes in [("sum", N.DP_RED_SUM, torch.float32, rows * cols * 4 + rows * 4),
                                      ("max", N.DP_RED_MAX, torch.float32, rows * cols * 4 + rows * 4),
                                      ("argmax", N.DP_RED_ARGMAX, torch.int64, rows * cols * 4 + rows * 8),
                                      ("softmax", N.DP_RED_SOFTMAX, torch.float32, 2 * rows * cols * 4),
                                      ("rmsnorm", N.DP_RED_RMSNORM, torch.float32, 2 * rows * cols * 4)]:
        full = kind_c in (N.DP_RED_SOFTMAX, N.DP_RED_RMSNORM)
        out = torch.empty((rows, cols) if full else (rows,), device=dev, dtype=odt)
        p = N.RowReduceParams(kind_c, N.DP_F32, N.DTYPE_CODE[str(odt).replace("torch.", "")],
                              1 if kind_c == N.DP_RED_RMSNORM else 0, 0, 0, rows, cols, cols, cols if full else 1,
                              1e-6, 0.0)
        w = ones if kind_c == N.DP_RED_RMSNORM else None
        ms = time_region(lambda: N.rowreduce(p, x, out, weight=w, stream=sp), min(args.steps, 200), args.warmup,
                         stream)
        gbs = nbytes / (ms / 1e3) / 1e9
        res[name] = {"ms": ms, "gbs": gbs, "frac": gbs / peak}
    worst = min(v["frac"] for v in res.values())
    return {"metric": f"row reduction HBM GB/s, fp32 [{rows}, {cols}]", "value": res["sum"]["gbs"], "unit": "GB/s",
            "higher_is_better": True, "dtype": "f32", "kinds": res,
            "roofline": {"bound": "hbm", "achieved": res["softmax"]["gbs"], "peak": peak, "unit": "GB/s",
                         "frac": res["softmax"]["gbs"] / peak, "peak_kind": kind, "worst_frac": worst},
            "config": {"workload": f"rowreduce fp32 {rows}x{cols} (inputs {rows * cols * 4 / 2**30:.2f} GiB > L2)"}}


def micro_vit(args, dev):
    """Preprocessing (uint8 480x640 images, batch 128) chained into the SigLIP-shaped ViT classifier, bf16."""
    import devproc
    from devproc_b200 import workloads
    B = 128
    imgs = workloads.preprocess_images(B)
    pre = devproc.compile(workloads.vision_preprocess, imgs)
    m = workloads.VitClassifier().eval()
    pix = torch.zeros(B, 3, 224, 224, dtype=torch.bfloat16)
    t0 = time.time()
    vit = devproc.compile(m, pix)
    compile_s = time.time() - t0
    d_imgs = imgs.to(dev)
    stream = torch.cuda.current_stream(dev)

    def step():
        x = pre.run(images=d_imgs, to_cpu=False)[0]
        return vit.run(x, to_cpu=False)[0]

    steps = min(args.steps, 20)
    ms = time_region(step, steps, args.warmup, stream)
    flops = workloads.vit_flops_per_image() * B
    peak, kind = tensor_peak()
    tf = flops / (ms / 1e3) / 1e12
    return {"metric": "pipeline samples/sec (ViT classifier)", "value": B / (ms / 1e3), "unit": "images/s",
            "higher_is_better": True, "dtype": "bf16", "ms_per_step": ms, "tflops": tf,
            "roofline": {"bound": "tensor", "achieved": tf, "peak": peak, "unit": "TFLOP/s", "frac": tf / peak,
                         "peak_kind": kind},
            "launches_per_step": len(pre.spec.records) + len(vit.spec.records), "compile_s": compile_s,
            "arena_mib": vit.spec.arena_bytes / 2 ** 20,
            "config": {"workload": "preprocess 128x480x640x3 u8 -> SigLIP-So400m/14-shaped ViT (27 layers, width "
                                   "1152, 16 heads, MLP 4304) -> mean-pool -> Linear 1152->1000 -> argmax, bf16, "
                                   "random-init weights N(0, 0.02)"}}


def micro_vla(args, dev):
    """pi0.5-shaped policy at batch 64: 192 camera images (uint8 480x640) preprocessed, the SigLIP-shaped
    encoder, a Gemma-2B-shaped prefill over 816 tokens and 10 action-expert denoise steps, bf16."""
    import devproc
    from devproc_b200 import workloads
    B = 64
    t0 = time.time()
    m = workloads.Pi05Policy(device=dev).eval()
    build_s = time.time() - t0
    imgs, ids, noise = workloads.pi05_inputs(B)
    pre = devproc.compile(workloads.vision_preprocess, imgs)
    t0 = time.time()
    pol = devproc.compile(m, torch.zeros(B * 3, 3, 224, 224, dtype=torch.bfloat16, device=dev),
                          ids.to(dev), noise.to(dev))
    compile_s = time.time() - t0
    d_imgs, d_ids, d_noise = imgs.to(dev), ids.to(dev), noise.to(dev)
    names = {v.name: v for v in pol.ir_function.inputs}
    order = [i.name for i in pol.spec.inputs]
    feed = {n: (d_ids if "ids" in n else d_noise if "noise" in n else None) for n in order}
    pix_name = [n for n in order if "pixels" in n][0]
    stream = torch.cuda.current_stream(dev)

    def step():
        x = pre.run(images=d_imgs, to_cpu=False)[0]
        feed[pix_name] = x
        return pol.run(**feed, to_cpu=False)[0]

    ms = time_region(step, min(args.steps, 3), args.warmup, stream)
    flops = workloads.pi05_flops_per_sample() * B
    peak, kind = tensor_peak()
    tf = flops / (ms / 1e3) / 1e12
    return {"metric": "policy samples/sec (pi0.5-shaped VLA)", "value": B / (ms / 1e3), "unit": "samples/s",
            "higher_is_better": True, "dtype": "bf16", "ms_per_step": ms, "tflops": tf,
            "roofline": {"bound": "tensor", "achieved": tf, "peak": peak, "unit": "TFLOP/s", "frac": tf / peak,
                         "peak_kind": kind},
            "launches_per_step": len(pre.spec.records) + len(pol.spec.records), "build_s": build_s,
            "compile_s": compile_s, "arena_gib": pol.spec.arena_bytes / 2 ** 30,
            "config": {"workload": "pi0.5-shaped policy, batch 64: 3 cameras 480x640 u8 -> SigLIP-So400m/14-shaped "
                                   "encoder (768 tokens) -> proj 1152->2048; 48 text ids; Gemma-2B-shaped prefill "
                                   "(18 layers, width 2048, 8q/1kv heads of 256, GeGLU 16384, RMSNorm, RoPE) over "
                                   "816 tokens; action expert (18 layers, width 1024, MLP 4096) x 10 flow-matching "
                                   "steps on 50x32 noise; bf16, random-init weights N(0, 0.02)"}}


def micro_token(args, dev):
    """The fp32 token pipeline, compiled from the torch module through the FX frontend."""
    import devproc
    from devproc_b200 import workloads
    m = workloads.TokenPipeline().eval()
    ids = workloads.token_ids()
    prog = devproc.compile(m, ids)
    d_ids = ids.to(dev)
    stream = torch.cuda.current_stream(dev)
    ms = time_region(lambda: prog.run(d_ids, to_cpu=False), min(args.steps, 500), args.warmup, stream)
    flops = 2 * 8 * 128 * (512 * 2048 * 2 + 512 * 32000)
    return {"metric": "pipeline samples/sec (fp32 token pipeline)", "value": 8 / (ms / 1e3), "unit": "samples/s",
            "higher_is_better": True, "dtype": "f32", "ms_per_step": ms, "tflops": flops / (ms / 1e3) / 1e12,
            "launches_per_step": len(prog.spec.records), "kernels": [r["label"] for r in prog.spec.records],
            "config": {"workload": "token pipeline B=8 L=128 fp32 (Embedding 32000x512 .. argmax int32)"}}


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

    if args.workload != "preprocess":
        fn = {"gemm": micro_gemm, "reduce": micro_reduce, "token": micro_token, "vit": micro_vit,
              "vla": micro_vla}[args.workload]
        line = fn(args, dev)
        line.update({"n_gpus": world, "data": "synthetic"})
        if rank == 0:
            print(json.dumps(line), flush=True)
        if world > 1:
            import torch.distributed as dist
            dist.destroy_process_group()
        return

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

    # ---- with the optional final gather: every step's bf16 output is all-gathered over NCCL on a side
    # stream, overlapped with the next step's preprocessing (two programs, so two output buffers alternate)
    gather = None
    if world > 1:
        import torch.distributed as dist
        progs = [prog, devproc.compile(workloads.vision_preprocess, images_host, device_id=local_rank)]
        outs_g = [pg.run(images=dev_in[j], to_cpu=False)[0] for j, pg in enumerate(progs)]
        gbuf = torch.empty((world,) + tuple(outs_g[0].shape), dtype=outs_g[0].dtype, device=dev)
        comm = torch.cuda.Stream(dev)
        done = [torch.cuda.Event() for _ in range(2)]
        freed = [torch.cuda.Event() for _ in range(2)]
        dist.all_gather_into_tensor(gbuf, outs_g[0])
        torch.cuda.synchronize()
        barrier()
        g0, g1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        g0.record(stream)
        for i in range(K):
            j = i % 2
            if i >= 2:
                stream.wait_event(freed[j])  # the gather that read this output buffer is done
            progs[j].run(images=dev_in[j], to_cpu=False)
            done[j].record(stream)
            comm.wait_event(done[j])
            with torch.cuda.stream(comm):
                dist.all_gather_into_tensor(gbuf, outs_g[j])
            freed[j].record(comm)
        stream.wait_stream(comm)
        g1.record(stream)
        torch.cuda.synchronize()
        barrier()
        g_ms = max_over_ranks(g0.elapsed_time(g1))
        ingress = (world - 1) * outs_g[0].numel() * outs_g[0].element_size()
        link = 770.0  # measured peer copy GB/s per direction per GPU on this machine type
        gather = {"value": B * world * K / (g_ms / 1e3), "unit": "images/s", "ms_per_step": g_ms / K,
                  "collective": "all_gather_into_tensor of each rank's bf16 output (NCCL), overlapped with the "
                                "next step on a side stream",
                  "nvlink_ingress_bytes_per_step_per_gpu": ingress,
                  "nvlink_bound_ms_per_step": ingress / (link * 1e9) * 1e3,
                  "nvlink_frac": (ingress / (link * 1e9) * 1e3) / (g_ms / K)}

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
                         "kernel": "preproc_u8c3_kernel<bf16> (NHWC u8 -> NCHW bf16)",
                         "algorithmic_bytes_per_launch": bytes_per_launch},
            "cpu_baseline": cpu,
            "with_gather": gather,
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
