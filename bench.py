"""Benchmark of the compiled-pipeline hot path on B200.

Headline workload: the vision preprocessing pipeline — uint8 NHWC images
[256, 480, 640, 3] → bilinear 224×224 → fp32 → (x - mean) / std → CHW → bf16
[256, 3, 224, 224] — compiled with ``devproc.compile`` and run through the
program.  One step = one pass over one 256-image batch per GPU.  With
``--gpus N`` (launched under torchrun, one process per GPU) every rank runs
its own 256-image shard through ``devproc.ShardedRuntime``: weak scaling, no
collective on the data path.

Prints ONE JSON line (rank 0):
  value          images/s of the whole job, inputs resident in HBM: the
                 median over repeated timed regions of exactly K steps each
                 (CUDA events on the launching stream, max over ranks);
  e2e            the same metric through ``Runtime.run`` with pinned host
                 buffers: host→device copy of the images and device→host
                 read of the result inside every timed step;
  roofline       achieved HBM GB/s of the preprocessing kernel (algorithmic
                 bytes per launch ÷ CUDA-event time per launch) against the
                 measured copy bandwidth;
  cpu_baseline   the same pipeline with torch on the host cores, on a
                 bounded sample of the batch;
  clocks         SM clock and throttle reasons sampled (NVML, every 20 ms)
                 while the timed regions ran;
  configs        (one GPU) the other benchmark configurations, each with its
                 own CUDA-event timing, roofline, clocks and CPU baseline: the
                 bf16 GEMM template at 4096³ and 8192×2048×16384, the row
                 reductions over fp32 [65536, 4096], the fused attention kernel
                 alone at the ViT / prefill / expert shapes, the fp32 token
                 pipeline, the ViT classifier and the pi0.5-shaped policy.
``--impl reference`` times only the preprocessing CPU path (rank 0).

Timed regions: before each region a ~2 ms device sleep (outside the region)
lets the host queue all K steps, so a region measures device time only; the
host issues a preprocessing step in ~17 µs against ~54 µs of device time, so
the steady state is device-bound either way.  Regions repeat until about one
second has passed, so the clock sampler sees the work.
"""

import argparse
import datetime
import json
import math
import os
import statistics
import sys
import threading
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

import torch  # noqa: E402

FALLBACK_HBM_GBS = 6650.0
FALLBACK_BF16_TFLOPS = 1590.0
FALLBACK_BF16_TFLOPS_SUSTAINED = 1400.0
CONFIG_NAMES = ("gemm", "reduce", "attention", "token", "vit", "vla")


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["b200", "reference"], default="b200")
    ap.add_argument("--batch", type=int, default=256)
    ap.add_argument("--rows", type=int, default=65536, help="rows of the reduce workload (4096 fp32 columns)")
    ap.add_argument("--cpu-sample", type=int, default=64, help="images in the CPU-baseline sample")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--min-region-s", type=float, default=1.0, help="repeat timed regions for about this long")
    ap.add_argument("--configs", default=None,
                    help="comma list of extra configurations in the headline line (gemm,reduce,attention,token,vit,vla); "
                         "default: all on one GPU, none on several")
    ap.add_argument("--workload", choices=["preprocess", "gemm", "reduce", "attention", "token", "vit", "vla"],
                    default="preprocess",
                    help="preprocess = the headline line; the others print one configuration's line alone")
    return ap.parse_args()


def dist_env():
    return int(os.environ.get("RANK", 0)), int(os.environ.get("LOCAL_RANK", 0)), int(os.environ.get("WORLD_SIZE", 1))


def _peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    return json.loads(p.read_text()) if p.exists() else None


def hbm_peak():
    d = _peaks()
    return (float(d["hbm_gbs"]), "measured") if d else (FALLBACK_HBM_GBS, "fallback")


def tensor_peak(sustained=False):
    d = _peaks()
    if d:
        if sustained and "bf16_tflops_sustained" in d:
            return float(d["bf16_tflops_sustained"]), "measured (sustained)"
        return float(d["bf16_tflops"]), "measured (burst)"
    return (FALLBACK_BF16_TFLOPS_SUSTAINED, "fallback (sustained)") if sustained else \
        (FALLBACK_BF16_TFLOPS, "fallback (burst)")


# ------------------------------------------------------------------ clocks
REASON_BITS = {"sw_power_cap": 0x4, "hw_slowdown": 0x8, "sw_thermal_slowdown": 0x20, "hw_thermal_slowdown": 0x40,
               "hw_power_brake_slowdown": 0x80}


class ClockSampler:
    """SM clock, power and clock-event reasons of one GPU, read through NVML
    (read-only queries) every 20 ms on a background thread."""

    def __init__(self, torch_device_index: int):
        self.samples = []
        self.max_mhz = None
        self.err = None
        self._stop = threading.Event()
        self._thread = None
        self.h = None
        try:
            import pynvml as nv
            nv.nvmlInit()
            uuid = str(torch.cuda.get_device_properties(torch_device_index).uuid)
            self.h = nv.nvmlDeviceGetHandleByUUID(uuid if uuid.startswith("GPU-") else "GPU-" + uuid)
            self.max_mhz = float(nv.nvmlDeviceGetMaxClockInfo(self.h, nv.NVML_CLOCK_SM))
            self.nv = nv
            self._reasons = getattr(nv, "nvmlDeviceGetCurrentClocksEventReasons", None) or \
                nv.nvmlDeviceGetCurrentClocksThrottleReasons
        except Exception as e:  # no NVML: report it instead of clocks
            self.err = f"NVML unavailable: {type(e).__name__}: {e}"

    def _run(self):
        nv = self.nv
        while not self._stop.is_set():
            try:
                self.samples.append((float(nv.nvmlDeviceGetClockInfo(self.h, nv.NVML_CLOCK_SM)),
                                     int(self._reasons(self.h)), nv.nvmlDeviceGetPowerUsage(self.h) / 1000.0))
            except Exception as e:
                self.err = str(e)
                return
            self._stop.wait(0.02)

    def __enter__(self):
        if self.h is not None:
            self._thread = threading.Thread(target=self._run, daemon=True)
            self._thread.start()
        return self

    def __exit__(self, *exc):
        self._stop.set()
        if self._thread is not None:
            self._thread.join(timeout=2)

    def summary(self):
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": [], "samples": 0,
                    "note": self.err or "no samples"}
        sm = [s[0] for s in self.samples]
        active = set()
        for _, bits, _ in self.samples:
            for name, b in REASON_BITS.items():
                if bits & b:
                    active.add(name)
        return {"sm_mhz": statistics.median(sm), "sm_min_mhz": min(sm), "sm_max_mhz": self.max_mhz,
                "power_w_max": max(s[2] for s in self.samples), "reasons": sorted(active),
                "samples": len(sm), "source": "NVML every 20 ms during the timed regions"}


# ------------------------------------------------------------------ timing
class Timer:
    """Repeated timed regions of exactly K steps; device time by CUDA events."""

    GATE_MS = 2.0

    def __init__(self, dev, world, min_region_s):
        self.dev, self.world, self.min_s = dev, world, min_region_s
        self.stream = torch.cuda.current_stream(dev)
        self.sm_hz = None

    def barrier(self):
        if self.world > 1:
            import torch.distributed as dist
            dist.barrier()

    def max_over_ranks(self, x):
        if self.world == 1:
            return x
        import torch.distributed as dist
        t = torch.tensor([float(x)], dtype=torch.float64, device=self.dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return t.item()

    def _gate(self):
        # device sleep so the host queues the whole region before it starts (outside the region)
        if self.sm_hz is None:
            self.sm_hz = torch.cuda.get_device_properties(self.dev).clock_rate * 1e3 or 2.0e9
        torch.cuda._sleep(int(self.GATE_MS * 1e-3 * self.sm_hz))

    def _region(self, step, K):
        self.barrier()
        torch.cuda.synchronize()
        self._gate()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(self.stream)
        for i in range(K):
            step(i)
        e1.record(self.stream)
        torch.cuda.synchronize()
        self.barrier()
        return e0.elapsed_time(e1)

    def run(self, step, K, warmup, max_regions=1000):
        """Median ms of R regions of K steps (R the same on every rank)."""
        for i in range(max(warmup, 3)):
            step(i)
        torch.cuda.synchronize()
        first = self._region(step, K)
        region_ms = self.max_over_ranks(first)
        R = int(self.max_over_ranks(min(max_regions, max(3, math.ceil(self.min_s * 1e3 / max(region_ms, 1e-3))))))
        times = []
        with ClockSampler(self.dev.index) as clk:
            for _ in range(R):
                times.append(self._region(step, K))
        med = self.max_over_ranks(statistics.median(times))
        return {"ms_region": med, "ms_per_step": med / K, "steps": K, "regions": R,
                "ms_region_min": min(times), "ms_region_max": max(times), "clocks": clk.summary()}


# --------------------------------------------------------- configurations
def cfg_gemm(args, dev, timer, cpu):
    """bf16 × bf16 GEMM, fp32 accumulate, bf16 out, B as [N, K] (the tcgen05 kernel), both shapes."""
    from devproc_b200 import _native as N
    peak, kind = tensor_peak()
    shapes = {}
    K_steps = min(args.steps, 20)
    for (M, Nn, K) in [(4096, 4096, 4096), (8192, 2048, 16384)]:
        g = torch.Generator(device=dev).manual_seed(0)
        a = torch.randn(M, K, device=dev, generator=g).bfloat16()
        b = torch.randn(Nn, K, device=dev, generator=g).bfloat16()
        c = torch.empty(M, Nn, device=dev, dtype=torch.bfloat16)
        p = N.GemmParams()
        p.M, p.N, p.K, p.lda, p.ldb, p.ldc, p.batch = M, Nn, K, K, K, Nn, 1
        p.a_dtype = p.b_dtype = p.c_dtype = N.DP_BF16
        p.b_layout = N.DP_B_NK
        sp = timer.stream.cuda_stream
        t = timer.run(lambda i: N.gemm(p, a, b, c, stream=sp), K_steps, args.warmup)
        N.raise_device_error(dev.index, "gemm")
        tf = 2.0 * M * Nn * K / (t["ms_per_step"] / 1e3) / 1e12
        shapes[f"{M}x{Nn}x{K}"] = {"ms": t["ms_per_step"], "tflops": tf, "frac": tf / peak, "launches": K_steps,
                                   "regions": t["regions"], "clocks": t["clocks"],
                                   "cpu_baseline": cpu and cpu.gemm(M, Nn, K, rows=512 if K <= 4096 else 128)}
        del a, b, c
    worst = min(shapes.values(), key=lambda v: v["tflops"])
    return {"metric": "bf16 GEMM TFLOP/s (fp32 accumulate, bf16 out)", "value": shapes["4096x4096x4096"]["tflops"],
            "unit": "TFLOP/s", "higher_is_better": True, "dtype": "bf16", "shapes": shapes,
            "roofline": {"bound": "tensor", "achieved": worst["tflops"], "peak": peak, "unit": "TFLOP/s",
                         "frac": worst["tflops"] / peak, "peak_kind": kind, "kernel": "tc_gemm_kernel (CTA pairs)",
                         "note": "the slower of the two shapes; per shape in shapes"},
            "gpu_launches": K_steps * 2, "clocks": shapes["4096x4096x4096"]["clocks"],
            "config": {"workload": "GEMM 4096^3 and 8192x2048x16384, bf16 inputs N(0,1), fp32 accumulate",
                       "l2": "operands 64-320 MB; repeated launches over the same operands"}}


def cfg_attention(args, dev, timer, cpu):
    """The fused tcgen05 attention kernel alone at the three shapes the ViT and policy steps run:
    SigLIP-shaped self-attention (128 images x 16 heads, 256 x 256, head dim 72), the Gemma-2B-shaped
    prefill (64 samples, 8 query heads on 1 key/value head, 816 x 816, head dim 256) and the action
    expert over the prefix cache (64 samples, 8 / 1 heads, 50 queries x 866 keys, head dim 256)."""
    from devproc_b200 import _native as N
    peak, kind = tensor_peak()
    shapes = {}
    K_steps = min(args.steps, 20)
    for name, (B, Hk, g, L, S, D) in {"vit_128x16x256x256_d72": (128, 16, 1, 256, 256, 72),
                                      "prefill_64x8q1kv_816x816_d256": (64, 1, 8, 816, 816, 256),
                                      "expert_64x8q1kv_50x866_d256": (64, 1, 8, 50, 866, 256)}.items():
        gen = torch.Generator(device=dev).manual_seed(0)
        Hq = Hk * g
        q = torch.randn(B, Hq, L, D, device=dev, generator=gen).bfloat16()
        k = torch.randn(B, Hk, S, D, device=dev, generator=gen).bfloat16()
        v = torch.randn(B, Hk, S, D, device=dev, generator=gen).bfloat16()
        o = torch.empty(B, Hq, L, D, dtype=torch.bfloat16, device=dev)
        p = N.AttentionParams()
        p.batch, p.heads_kv, p.group, p.L, p.S, p.D, p.Dv = B, Hk, g, L, S, D, D
        p.q_sb, p.q_sh, p.q_sl = Hq * L * D, L * D, D
        p.k_sb, p.k_sh, p.k_ss = Hk * S * D, S * D, D
        p.v_sb, p.v_sh, p.v_ss = Hk * S * D, S * D, D
        p.o_sb, p.o_sh, p.o_sl = Hq * L * D, L * D, D
        p.scale, p.dtype = D ** -0.5, N.DP_BF16
        sp = timer.stream.cuda_stream
        t = timer.run(lambda i: N.attention(p, q, k, v, o, stream=sp), K_steps, args.warmup)
        N.raise_device_error(dev.index, "attention")
        flops = 4.0 * B * Hq * L * S * D
        tf = flops / (t["ms_per_step"] / 1e3) / 1e12
        shapes[name] = {"us": t["ms_per_step"] * 1e3, "tflops": tf, "frac": tf / peak, "launches": K_steps,
                        "regions": t["regions"], "clocks": t["clocks"],
                        "operand_mb": (q.numel() + k.numel() + v.numel() + o.numel()) * 2 / 1e6}
        del q, k, v, o
    worst = min(shapes.values(), key=lambda v: v["tflops"])
    return {"metric": "fused attention TFLOP/s (bf16, 4*rows*keys*head_dim per launch)",
            "value": shapes["prefill_64x8q1kv_816x816_d256"]["tflops"], "unit": "TFLOP/s",
            "higher_is_better": True, "dtype": "bf16", "shapes": shapes,
            "roofline": {"bound": "tensor", "achieved": worst["tflops"], "peak": peak, "unit": "TFLOP/s",
                         "frac": worst["tflops"] / peak, "peak_kind": kind, "kernel": "attn_kernel",
                         "note": "the slowest shape; per shape in shapes"},
            "gpu_launches": K_steps * len(shapes), "clocks": shapes["vit_128x16x256x256_d72"]["clocks"],
            "cpu_baseline": None,
            "config": {"workload": "fused attention at the ViT, prefill and action-expert shapes, q / k / v N(0,1)",
                       "l2": "q, k, v and o take 302 / 481 / 83 MB (operand_mb per shape): the ViT and prefill "
                             "operands exceed L2, the expert's fit in it",
                       "cpu_baseline": "none: a sub-operation of the ViT and policy configurations, whose CPU "
                                       "baselines cover it"}}


def cfg_reduce(args, dev, timer, cpu):
    """Row reductions over fp32 [rows, 4096] (65536 rows by default)."""
    from devproc_b200 import _native as N
    peak, kind = hbm_peak()
    rows, cols = args.rows, 4096
    g = torch.Generator(device=dev).manual_seed(0)
    x = torch.randn(rows, cols, device=dev, generator=g)
    ones = torch.ones(cols, device=dev)
    sp = timer.stream.cuda_stream
    res = {}
    K_steps = min(args.steps, 20)
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
        t = timer.run(lambda i: N.rowreduce(p, x, out, weight=w, stream=sp), K_steps, args.warmup)
        N.raise_device_error(dev.index, "rowreduce")
        gbs = nbytes / (t["ms_per_step"] / 1e3) / 1e9
        res[name] = {"ms": t["ms_per_step"], "gbs": gbs, "frac": gbs / peak, "algorithmic_bytes": nbytes,
                     "regions": t["regions"], "clocks": t["clocks"],
                     "cpu_baseline": cpu and cpu.reduce(name, rows, cols)}
        del out
    worst = min(res.values(), key=lambda v: v["frac"])
    return {"metric": f"row reduction HBM GB/s, fp32 [{rows}, {cols}]", "value": res["sum"]["gbs"], "unit": "GB/s",
            "higher_is_better": True, "dtype": "f32", "kinds": res,
            "roofline": {"bound": "hbm", "achieved": worst["gbs"], "peak": peak, "unit": "GB/s",
                         "frac": worst["frac"], "peak_kind": kind,
                         "note": "the kind furthest from the peak; per kind in kinds"},
            "gpu_launches": K_steps * 5, "clocks": res["softmax"]["clocks"],
            "config": {"workload": f"rowreduce fp32 {rows}x{cols} N(0,1): sum, max, argmax, softmax, RMSNorm",
                       "l2": f"inputs {rows * cols * 4 / 2**30:.2f} GiB > L2"}}


def cfg_token(args, dev, timer, cpu):
    """The fp32 token pipeline, compiled from the torch module through the FX frontend."""
    import devproc
    from devproc_b200 import workloads
    m = workloads.TokenPipeline().eval()
    ids = workloads.token_ids()
    prog = devproc.compile(m, ids, device_id=dev.index)
    d_ids = ids.to(dev)
    K_steps = min(args.steps, 20)
    t = timer.run(lambda i: prog.run(d_ids, to_cpu=False), K_steps, args.warmup)
    prog.synchronize()
    flops = 2 * 8 * 128 * (512 * 2048 * 2 + 512 * 32000)
    tf = flops / (t["ms_per_step"] / 1e3) / 1e12
    bf16, _ = tensor_peak()
    ceiling = bf16 / 6.0  # three TF32 products per fp32 product, TF32 at half the bf16 rate
    host_ids = ids.pin_memory()
    e2e = _e2e(timer, lambda i: prog.run(host_ids, reuse_host_buffers=True), K_steps)
    return {"metric": "pipeline samples/sec (fp32 token pipeline)", "value": 8 / (t["ms_per_step"] / 1e3),
            "unit": "samples/s", "higher_is_better": True, "dtype": "f32 (3xTF32 linears)",
            "ms_per_step": t["ms_per_step"], "steps": K_steps, "regions": t["regions"], "tflops": tf,
            "roofline": {"bound": "tensor", "achieved": tf, "peak": ceiling, "unit": "TFLOP/s", "frac": tf / ceiling,
                         "peak_kind": "measured bf16 burst / 6 (3xTF32: three TF32 products at half the bf16 rate)"},
            "e2e": {"value": 8 / (e2e / 1e3), "unit": "samples/s", "h2d_bytes_per_step": ids.numel() * 4,
                    "d2h_bytes_per_step": 8 * 128 * 4, "path": "program.run(pinned host int32 ids) -> host int32"},
            "gpu_launches": K_steps * len(prog.spec.records), "launches_per_step": len(prog.spec.records),
            "kernels": [r["label"] for r in prog.spec.records], "clocks": t["clocks"],
            "cpu_baseline": cpu and cpu.token_pipeline(m, ids.long()),
            "config": {"workload": "token pipeline B=8 L=128 fp32 (Embedding 32000x512 .. argmax int32)",
                       "l2": "weights 139 MB > L2"}}


def _e2e(timer, step, K):
    """ms per step of ``step`` (host in, host out) over K steps, CUDA events, max over ranks."""
    for i in range(2):
        step(i)
    timer.barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(timer.stream)
    for i in range(K):
        step(i)
    e1.record(timer.stream)
    torch.cuda.synchronize()
    timer.barrier()
    return timer.max_over_ranks(e0.elapsed_time(e1)) / K


def cfg_vit(args, dev, timer, cpu):
    """Preprocessing (uint8 480x640 images, batch 128) chained into the SigLIP-shaped ViT classifier, bf16."""
    import devproc
    from devproc_b200 import workloads
    B = 128
    imgs = workloads.preprocess_images(B)
    pre = devproc.compile(workloads.vision_preprocess, imgs, device_id=dev.index)
    t0 = time.time()
    m = workloads.VitClassifier(device=dev).eval()
    pix = torch.zeros(B, 3, 224, 224, dtype=torch.bfloat16)
    vit = devproc.compile(m, pix, device_id=dev.index)
    compile_s = time.time() - t0
    d_imgs = imgs.to(dev)

    def step(i):
        x = pre.run(images=d_imgs, to_cpu=False)[0]
        return vit.run(x, to_cpu=False)[0]

    K_steps = min(args.steps, 10)
    t = timer.run(step, K_steps, args.warmup)
    vit.synchronize()
    flops = workloads.vit_flops_per_image() * B
    peak, kind = tensor_peak(sustained=True)
    tf = flops / (t["ms_per_step"] / 1e3) / 1e12
    h_imgs = imgs.pin_memory()

    def e2e_step(i):
        x = pre.run(images=h_imgs, to_cpu=False)[0]
        return vit.run(x, reuse_host_buffers=True)[0]

    e2e = _e2e(timer, e2e_step, min(K_steps, 5))
    return {"metric": "pipeline samples/sec (ViT classifier)", "value": B / (t["ms_per_step"] / 1e3),
            "unit": "images/s", "higher_is_better": True, "dtype": "bf16", "ms_per_step": t["ms_per_step"],
            "steps": K_steps, "regions": t["regions"], "tflops": tf,
            "roofline": {"bound": "tensor", "achieved": tf, "peak": peak, "unit": "TFLOP/s", "frac": tf / peak,
                         "peak_kind": kind, "flops_per_step": flops},
            "e2e": {"value": B / (e2e / 1e3), "unit": "images/s", "h2d_bytes_per_step": imgs.numel(),
                    "d2h_bytes_per_step": B * 8, "path": "program.run(pinned host uint8 images) -> host argmax"},
            "gpu_launches": K_steps * (len(pre.spec.records) + len(vit.spec.records)),
            "launches_per_step": len(pre.spec.records) + len(vit.spec.records), "compile_s": compile_s,
            "clocks": t["clocks"], "cpu_baseline": cpu and cpu.vit(m),
            "config": {"workload": "preprocess 128x480x640x3 u8 -> SigLIP-So400m/14-shaped ViT (27 layers, width "
                                   "1152, 16 heads, MLP 4304) -> mean-pool -> Linear 1152->1000 -> argmax, bf16, "
                                   "random-init weights N(0, 0.02)"}}


def cfg_vla(args, dev, timer, cpu):
    """pi0.5-shaped policy at batch 64: 192 camera images (uint8 480x640) preprocessed, the SigLIP-shaped
    encoder, a Gemma-2B-shaped prefill over 816 tokens and 10 action-expert denoise steps, bf16."""
    import devproc
    from devproc_b200 import workloads
    B = 64
    t0 = time.time()
    m = workloads.Pi05Policy(device=dev).eval()
    build_s = time.time() - t0
    imgs, ids, noise = workloads.pi05_inputs(B)
    pre = devproc.compile(workloads.vision_preprocess, imgs, device_id=dev.index)
    t0 = time.time()
    pol = devproc.compile(m, torch.zeros(B * 3, 3, 224, 224, dtype=torch.bfloat16, device=dev),
                          ids.to(dev), noise.to(dev), device_id=dev.index)
    compile_s = time.time() - t0
    d_imgs, d_ids, d_noise = imgs.to(dev), ids.to(dev), noise.to(dev)
    order = [i.name for i in pol.spec.inputs]
    pix_name = [n for n in order if "pixels" in n][0]
    feed = {n: (d_ids if "ids" in n else d_noise) for n in order if n != pix_name}

    def step(i):
        x = pre.run(images=d_imgs, to_cpu=False)[0]
        return pol.run(**{pix_name: x}, **feed, to_cpu=False)[0]

    K_steps = min(args.steps, 3)
    t = timer.run(step, K_steps, min(args.warmup, 3), max_regions=5)
    pol.synchronize()
    flops = workloads.pi05_flops_per_sample() * B
    peak, kind = tensor_peak(sustained=True)
    tf = flops / (t["ms_per_step"] / 1e3) / 1e12
    h_imgs, h_feed = imgs.pin_memory(), {n: (ids if "ids" in n else noise).pin_memory() for n in feed}

    def e2e_step(i):
        x = pre.run(images=h_imgs, to_cpu=False)[0]
        return pol.run(**{pix_name: x}, **h_feed, reuse_host_buffers=True)[0]

    e2e = _e2e(timer, e2e_step, 2)
    return {"metric": "policy samples/sec (pi0.5-shaped VLA)", "value": B / (t["ms_per_step"] / 1e3),
            "unit": "samples/s", "higher_is_better": True, "dtype": "bf16", "ms_per_step": t["ms_per_step"],
            "steps": K_steps, "regions": t["regions"], "tflops": tf,
            "roofline": {"bound": "tensor", "achieved": tf, "peak": peak, "unit": "TFLOP/s", "frac": tf / peak,
                         "peak_kind": kind, "flops_per_step": flops},
            "e2e": {"value": B / (e2e / 1e3), "unit": "samples/s",
                    "h2d_bytes_per_step": imgs.numel() + ids.numel() * 4 + noise.numel() * 4,
                    "d2h_bytes_per_step": noise.numel() * 4,
                    "path": "program.run(pinned host images, ids, noise) -> host fp32 actions"},
            "gpu_launches": K_steps * (len(pre.spec.records) + len(pol.spec.records)),
            "launches_per_step": len(pre.spec.records) + len(pol.spec.records), "build_s": build_s,
            "compile_s": compile_s, "arena_gib": pol.spec.arena_bytes / 2 ** 30, "clocks": t["clocks"],
            "cpu_baseline": cpu and cpu.pi05(),
            "config": {"workload": "pi0.5-shaped policy, batch 64: 3 cameras 480x640 u8 -> SigLIP-So400m/14-shaped "
                                   "encoder (768 tokens) -> proj 1152->2048; 48 text ids; Gemma-2B-shaped prefill "
                                   "(18 layers, width 2048, 8q/1kv heads of 256, GeGLU 16384, RMSNorm, RoPE) over "
                                   "816 tokens; action expert (18 layers, width 1024, MLP 4096) x 10 flow-matching "
                                   "steps on 50x32 noise; bf16, random-init weights N(0, 0.02)"}}


CONFIG_FNS = {"gemm": cfg_gemm, "reduce": cfg_reduce, "attention": cfg_attention, "token": cfg_token, "vit": cfg_vit,
              "vla": cfg_vla}


# ----------------------------------------------------------- headline (C2)
def ncu_traffic():
    """Per-launch DRAM bytes of the preprocessing kernel from the committed ncu summary."""
    p = ROOT / "profiles" / "preproc_c2_ncu.md"
    if not p.exists():
        return None
    for line in p.read_text().splitlines():
        if line.startswith("traffic_bytes_per_launch_full_batch:"):
            return int(float(line.split(":")[1].strip()))
    return None


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


def measure_h2d_gbs(timer, host, dev):
    """Pinned host -> device copy bandwidth of this rank with every rank copying
    at once (best of 5 copies of ``host``), and the sum over ranks."""
    dst = torch.empty_like(host, device=dev)
    dst.copy_(host, non_blocking=True)
    torch.cuda.synchronize()
    best = None
    for _ in range(5):
        timer.barrier()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(timer.stream)
        dst.copy_(host, non_blocking=True)
        e1.record(timer.stream)
        torch.cuda.synchronize()
        ms = e0.elapsed_time(e1)
        best = ms if best is None else min(best, ms)
    per_rank = host.numel() * host.element_size() / (best / 1e3) / 1e9
    total = per_rank
    if timer.world > 1:
        import torch.distributed as dist
        t = torch.tensor([per_rank], dtype=torch.float64, device=dev)
        dist.all_reduce(t)
        total = t.item()
    del dst
    return per_rank, total


def measure_peer_copy_gbs(dev, world, rank):
    """Peer copy bandwidth rank 1 -> rank 0 over NVLink measured in this run
    (copy engine, 256 MiB, best of 5), broadcast to every rank; None on one GPU."""
    if world == 1:
        return None
    import torch.distributed as dist
    nbytes = 256 << 20
    buf = torch.empty(nbytes, dtype=torch.uint8, device=dev)
    gbs = torch.zeros(1, dtype=torch.float64, device=dev)
    # rank 0 receives one buffer from rank 1 through NCCL point-to-point (a peer copy over NVLink)
    for _ in range(2):
        if rank == 0:
            dist.recv(buf, src=1)
        elif rank == 1:
            dist.send(buf, dst=0)
    torch.cuda.synchronize()
    best = None
    for _ in range(5):
        dist.barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        if rank == 0:
            dist.recv(buf, src=1)
        elif rank == 1:
            dist.send(buf, dst=0)
        e1.record()
        torch.cuda.synchronize()
        ms = e0.elapsed_time(e1)
        best = ms if best is None else min(best, ms)
    if rank == 0:
        gbs.fill_(nbytes / (best / 1e3) / 1e9)
    dist.broadcast(gbs, src=0)
    return gbs.item()


def main():
    args = parse()
    if args.impl == "reference":
        return reference_arm(args)
    rank, local_rank, world = dist_env()
    if world != args.gpus and world == 1 and args.gpus > 1:
        raise SystemExit("--gpus N > 1 must be launched with torchrun (one process per GPU)")
    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    if world > 1:
        import torch.distributed as dist
        dist.init_process_group("nccl", device_id=dev, timeout=datetime.timedelta(seconds=120))

    import devproc
    from devproc_b200 import workloads
    timer = Timer(dev, world, args.min_region_s)
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        from oracle import cpu_baselines as cpu

    if args.workload != "preprocess":
        line = CONFIG_FNS[args.workload](args, dev, timer, cpu)
        line.update({"n_gpus": world, "data": "synthetic", "warmup": max(args.warmup, 3)})
        if rank == 0:
            print(json.dumps(line), flush=True)
        if world > 1:
            import torch.distributed as dist
            dist.destroy_process_group()
        return

    B = args.batch
    images_host = workloads.preprocess_images(B, seed=rank)
    # one 256-image shard per rank, through the product's sharded runner
    shard = devproc.ShardedRuntime(workloads.vision_preprocess, images_host, rank=rank, world_size=world,
                                   device_id=local_rank, gather=world > 1)
    prog = shard.program
    n_launch_per_step = len(prog.spec.records)
    # Two device-resident input batches used alternately: 2 × 236 MB > 126 MB L2.
    dev_in = [images_host.to(dev), workloads.preprocess_images(B, seed=1000 + rank).to(dev)]

    t = timer.run(lambda i: shard.run_local(images=dev_in[i % 2]), args.steps, args.warmup)
    shard.synchronize()
    K = args.steps
    value = B * world / (t["ms_per_step"] / 1e3)

    # ---- end to end: pinned host images in, host result out, through Runtime.run
    rt = devproc.Runtime(prog, device_id=local_rank)
    host_in = [images_host.pin_memory(), workloads.preprocess_images(B, seed=2000 + rank).pin_memory()]
    outs = []
    e2e_ms = _e2e(timer, lambda i: outs.append(rt.run(images=host_in[i % 2], reuse_host_buffers=True)) or None, K)
    e2e_value = B * world / (e2e_ms / 1e3)
    h2d = images_host.numel() * images_host.element_size()
    d2h = sum(o.numel() * o.element_size() for o in outs[-1])
    # the host link: H2D of every rank at once (the step's device->host copy runs the other way, overlapped)
    h2d_rank, h2d_total = measure_h2d_gbs(timer, host_in[0], dev)
    link_bound = h2d_total * 1e9 / (h2d / B)  # images/s if the input copies ran at that rate back to back

    # ---- with the final gather: every step's bf16 output goes to rank 0 (ShardedRuntime.run), overlapped
    gather = None
    if world > 1:
        link = measure_peer_copy_gbs(dev, world, rank)
        tg = timer.run(lambda i: shard.run(images=dev_in[i % 2]), K, args.warmup)
        shard.synchronize()
        ingress = (world - 1) * B * 3 * 224 * 224 * 2
        bound_ms = ingress / (link * 1e9) * 1e3
        gather = {"value": B * world / (tg["ms_per_step"] / 1e3), "unit": "images/s",
                  "ms_per_step": tg["ms_per_step"], "collective": shard.gather_kind,
                  "nvlink_ingress_bytes_per_step_rank0": ingress, "peer_copy_gbs_measured": link,
                  "nvlink_bound_ms_per_step": bound_ms, "nvlink_frac": bound_ms / tg["ms_per_step"]}

    # ---- roofline of the preprocessing kernel (one launch per step)
    bytes_per_launch = B * workloads.PREPROC_BYTES_PER_IMAGE
    launch_ms = t["ms_per_step"] / n_launch_per_step
    achieved = bytes_per_launch / (launch_ms / 1e3) / 1e9
    peak, peak_kind = hbm_peak()

    configs = None
    names = args.configs.split(",") if args.configs else (list(CONFIG_NAMES) if world == 1 else [])
    names = [n for n in names if n and n != "none"]
    if names:
        configs = {}
        for n in names:
            t0 = time.time()
            try:
                configs[n] = CONFIG_FNS[n](args, dev, timer, cpu)
            except Exception as e:  # one configuration failing must not hide the others
                configs[n] = {"error": f"{type(e).__name__}: {e}"}
            configs[n]["wall_s"] = time.time() - t0
            torch.cuda.empty_cache()

    if rank == 0:
        cpu_line = None
        if cpu is not None:
            v, cores = cpu_baseline_run(images_host, 3, args.cpu_sample)
            cpu_line = {"value": v, "unit": "images/s", "cores": cores, "kind": "port",
                        "sample": f"{args.cpu_sample} of the {B} images per step, median of 3, torch CPU ops "
                                  "(F.interpolate bilinear, normalise, bf16)"}
        line = {
            "metric": "pipeline samples/sec (vision preprocessing)", "value": value, "unit": "images/s",
            "n_gpus": world, "steps": K, "warmup": max(args.warmup, 3), "ms_per_step": t["ms_per_step"],
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "u8->f32->bf16",
            "data": "synthetic (seeded uniform uint8 images)",
            "config": {"workload": "vision_preprocess 256x480x640x3 u8 -> 256x3x224x224 bf16 (normalise, CHW)",
                       "global_batch": B * world, "per_gpu_batch": B,
                       "parallelism": f"dp{world} batch-sharded (ShardedRuntime), no collective",
                       "l2": "inputs larger than L2: two 236 MB input batches alternate",
                       "timing": f"median of {t['regions']} regions of {K} steps, each after a 2 ms device "
                                 "sleep outside the region (device time of queued steps)"},
            "regions": t["regions"], "ms_region_min": t["ms_region_min"], "ms_region_max": t["ms_region_max"],
            "e2e": {"value": e2e_value, "unit": "images/s", "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                    "path": "Runtime.run(images=pinned host uint8) -> pinned host bf16",
                    "host_link": {"h2d_gbs_rank0": h2d_rank, "h2d_gbs_all_ranks": h2d_total,
                                  "bound_images_per_s": link_bound, "frac": e2e_value / link_bound,
                                  "note": "pinned H2D copies of every rank at once, best of 5; the bound is the "
                                          "input bytes at that aggregate rate"}},
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                         "frac": achieved / peak, "traffic": ncu_traffic(), "peak_kind": peak_kind,
                         "kernel": "preproc_u8c3_kernel<bf16> (NHWC u8 -> NCHW bf16)",
                         "algorithmic_bytes_per_launch": bytes_per_launch},
            "cpu_baseline": cpu_line,
            "with_gather": gather,
            "clocks": t["clocks"],
            "gpu_launches": K * n_launch_per_step,
            "configs": configs,
        }
        print(json.dumps(line), flush=True)
    shard.close()
    if world > 1:
        import torch.distributed as dist
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
