"""CPU baselines of the template microbenchmarks and model pipelines — test infrastructure.

``bench.py``'s ``cpu_baseline`` leg times these on the host cores next to the
GPU figures; the product never imports them.  Each is torch on the CPU with
every host thread, on a bounded sample of its configuration (stated in the
``sample`` string it returns), and reports the configuration's own unit:

* GEMM: ``torch.matmul`` in fp32 on a block of A's rows (CPU bf16 matmul has
  no fast path), TFLOP/s;
* row reductions: the oracle's definition of each kind (torch.sum / amax /
  argmax / softmax, RMSNorm as x·rsqrt(mean(x²)+eps)·w) on a block of rows,
  GB/s of algorithmic bytes;
* the fp32 token pipeline: the torch module itself, samples/s;
* the ViT classifier: the torch module in fp32 on one image, images/s;
* the pi0.5-shaped policy: one sample through a 2-layer copy of each stack
  (encoder, prefill, expert) at full widths and 10 denoise steps, in fp32,
  its time scaled by FLOPs to the full depth, samples/s.
"""

import copy
import statistics
import time

import torch

from .cpu_pipeline import use_all_threads


def _median_time(fn, reps):
    fn()  # warm
    ts = []
    for _ in range(reps):
        t0 = time.perf_counter()
        fn()
        ts.append(time.perf_counter() - t0)
    return statistics.median(ts)


def gemm(M, N, K, rows=512, reps=3):
    cores = use_all_threads()
    g = torch.Generator().manual_seed(0)
    a = torch.randn(rows, K, generator=g).bfloat16().float()
    b = torch.randn(N, K, generator=g).bfloat16().float()
    t = _median_time(lambda: a @ b.T, reps)
    return {"value": 2.0 * rows * N * K / t / 1e12, "unit": "TFLOP/s", "cores": cores, "kind": "port",
            "sample": f"{rows} of the {M} rows of A, fp32 torch.matmul, median of {reps}"}


def reduce(kind, rows_total, cols, rows=4096, reps=3):
    cores = use_all_threads()
    x = torch.randn(rows, cols, generator=torch.Generator().manual_seed(0))
    w = torch.ones(cols)
    fns = {"sum": lambda: x.sum(-1), "max": lambda: x.amax(-1), "argmax": lambda: x.argmax(-1),
           "softmax": lambda: torch.softmax(x, -1),
           "rmsnorm": lambda: x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + 1e-6) * w}
    t = _median_time(fns[kind], reps)
    out_bytes = {"sum": 4, "max": 4, "argmax": 8}.get(kind, cols * 4)
    nbytes = rows * (cols * 4 + out_bytes)
    return {"value": nbytes / t / 1e9, "unit": "GB/s", "cores": cores, "kind": "port",
            "sample": f"{rows} of the {rows_total} rows, torch CPU ops, median of {reps}"}


def token_pipeline(model, ids, reps=3):
    cores = use_all_threads()
    with torch.no_grad():
        t = _median_time(lambda: model(ids), reps)
    return {"value": ids.shape[0] / t, "unit": "samples/s", "cores": cores, "kind": "port",
            "sample": f"the whole {ids.shape[0]}x{ids.shape[1]} batch through the fp32 torch module, median of {reps}"}


def vit(model, reps=2):
    """One image through an fp32 copy of ``model`` (the bf16 benchmark module)."""
    cores = use_all_threads()
    m = copy.deepcopy(model).float().eval()
    x = torch.randn(1, 3, 224, 224, generator=torch.Generator().manual_seed(0))
    with torch.no_grad():
        t = _median_time(lambda: m(x), reps)
    return {"value": 1.0 / t, "unit": "images/s", "cores": cores, "kind": "port",
            "sample": f"1 image through an fp32 copy of the module (bf16 matmul has no fast CPU path), "
                      f"median of {reps}"}


def pi05(reps=1):
    """One sample through a 2-layer-per-stack fp32 copy, scaled by FLOPs to the full policy."""
    from devproc_b200 import workloads
    cores = use_all_threads()
    small = dict(layers=2, expert_layers=2, vit=dict(layers=2))
    m = workloads.Pi05Policy(dtype=torch.float32, **small).eval()
    imgs, ids, noise = workloads.pi05_inputs(1)
    pix = torch.randn(3, 3, 224, 224, generator=torch.Generator().manual_seed(0))
    with torch.no_grad():
        t = _median_time(lambda: m(pix, ids, noise), reps)
    f_small = workloads.pi05_flops_per_sample(layers=2, expert_layers=2, vit_layers=2)
    f_full = workloads.pi05_flops_per_sample()
    return {"value": 1.0 / (t * f_full / f_small), "unit": "samples/s", "cores": cores, "kind": "port",
            "sample": f"1 sample through an fp32 copy with 2 layers per stack (encoder, prefill, expert; full "
                      f"widths, 10 denoise steps), {t:.2f} s scaled by FLOPs ({f_small / 1e9:.0f} -> "
                      f"{f_full / 1e9:.0f} GFLOP)"}
