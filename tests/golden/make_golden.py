"""Generate golden vectors from the reference's own kernels (run here, on the CPU).

The reference (DevProc, read from its ``src`` folder) implements every
tensor op as a Triton template.  Triton's interpreter (TRITON_INTERPRET=1)
executes those templates with numpy on the CPU, so their outputs can be
recorded without a GPU.  Each case runs in its own subprocess because the
reference's elementwise templates index past the end of tensors whose size
is not a multiple of their block (templates/elementwise.py:20-22) — all
shapes here are multiples of 128 for that reason.

Recorded per case: the seeded inputs and the reference template's output,
in ``templates.npz``; plus ``ir_ops.json`` with the op lists the reference's
DSL and FX frontend build for the test programs of its own test-suite.

Usage (in a container that has the reference tree):
    python tests/golden/make_golden.py --ref-src <DevProc checkout>/src
or with DEVPROC_REF_SRC set to that folder.
"""

import argparse
import json
import os
import subprocess
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
REF_SRC = os.environ.get("DEVPROC_REF_SRC")

CASES = ["normalize_f32", "normalize_u8", "relu", "sigmoid", "add", "to_i32", "softmax", "argmax_small",
         "argmax_wide", "argmax_ties", "sum", "matmul", "linear"]

CHILD = r'''
import os, sys, json
os.environ["TRITON_INTERPRET"] = "1"
sys.path.insert(0, REF_SRC)
import numpy as np, torch
from devproc.backend.triton.templates import elementwise as ew, reduce as rd, matmul as mm
case = sys.argv[1]
g = torch.Generator().manual_seed(1234 + sum(map(ord, case)))
def rn(*s): return torch.randn(*s, generator=g)
out = {}
if case == "normalize_f32":
    x = rn(16, 32); y = torch.empty(16, 32); ew.launch_normalize(x, y)
elif case == "normalize_u8":
    x = torch.randint(0, 256, (4, 128), generator=g, dtype=torch.uint8); y = torch.empty(4, 128)
    ew.launch_normalize(x, y)
elif case == "relu":
    x = rn(16, 32); y = torch.empty(16, 32); ew.launch_relu(x, y)
elif case == "sigmoid":
    x = rn(16, 32) * 4; y = torch.empty(16, 32); ew.launch_sigmoid(x, y)
elif case == "add":
    x = rn(16, 32); x2 = rn(16, 32); y = torch.empty(16, 32); ew.launch_add(x, x2, y); out["x2"] = x2
elif case == "to_i32":
    x = rn(8, 128) * 100; y = torch.empty(8, 128, dtype=torch.int32); ew.launch_to_dtype(x, y, "int32")
elif case == "softmax":
    x = rn(4, 128); y = torch.empty(4, 128); rd.launch_softmax(x, y)
elif case == "argmax_small":
    x = rn(4, 128); y = torch.empty(4, dtype=torch.int64); rd.launch_argmax(x, y)
elif case == "argmax_wide":
    x = rn(16, 2048); y = torch.empty(16, dtype=torch.int64); rd.launch_argmax(x, y)
elif case == "argmax_ties":
    x = torch.round(rn(8, 512) * 2); y = torch.empty(8, dtype=torch.int64); rd.launch_argmax(x, y)
elif case == "sum":
    x = rn(16, 2048); y = torch.empty(16); rd.launch_reduce_sum(x, y)
elif case == "matmul":
    # K equals one BLOCK_K: the template's K loop is only right for a single K block.
    x = rn(16, 32); w = rn(32, 16); y = torch.empty(16, 16)
    mm.matmul_kernel.fn[(1,)](x, w, y, 16, 16, 32, x.stride(0), x.stride(1), w.stride(0), w.stride(1),
                              y.stride(0), y.stride(1), BLOCK_M=16, BLOCK_N=16, BLOCK_K=32)
    out["x2"] = w
elif case == "linear":
    # One tile, K equal to one BLOCK_K (see matmul above).
    x = rn(16, 32); w = rn(16, 32); b = rn(16); y = torch.empty(16, 16)
    mm.linear_kernel.fn[(1,)](x, w, b, y, 16, 16, 32, x.stride(0), x.stride(1), w.stride(0), w.stride(1),
                              y.stride(0), y.stride(1), BLOCK_M=16, BLOCK_N=16, BLOCK_K=32, HAS_BIAS=True)
    out["x2"] = w; out["b"] = b
out["x"] = x; out["y"] = y
np.savez(sys.argv[2], **{k: v.numpy() for k, v in out.items()})
'''


def main() -> None:
    global REF_SRC
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref-src", default=REF_SRC, help="the reference's src folder (default: $DEVPROC_REF_SRC)")
    REF_SRC = ap.parse_args().ref_src
    if not REF_SRC or not (Path(REF_SRC) / "devproc").is_dir():
        raise SystemExit("give the reference's src folder with --ref-src or DEVPROC_REF_SRC")
    arrays = {}
    skipped = {}
    for case in CASES:
        tmp = HERE / f"_tmp_{case}.npz"
        code = CHILD.replace("REF_SRC", repr(REF_SRC))
        r = subprocess.run([sys.executable, "-c", code, case, str(tmp)], capture_output=True, text=True,
                           timeout=600)
        if r.returncode != 0 or not tmp.exists():
            skipped[case] = (r.stdout + r.stderr).strip().splitlines()[-1:] or ["failed"]
            continue
        with np.load(tmp) as z:
            for k in z.files:
                arrays[f"{case}/{k}"] = z[k]
        tmp.unlink()
    np.savez_compressed(HERE / "templates.npz", **arrays)
    (HERE / "templates_skipped.json").write_text(json.dumps(skipped, indent=1) + "\n")
    (HERE / "ir_ops.json").write_text(json.dumps(reference_ir_ops(), indent=1) + "\n")
    print("cases:", sorted({k.split('/')[0] for k in arrays}), "skipped:", skipped)


def reference_ir_ops():
    """Op-name lists the reference builds for its own test programs (DSL and FX)."""
    code = r'''
import sys, json
sys.path.insert(0, REF_SRC)
import torch, devproc
from devproc.ir.from_torch import from_torch
res = {}
@devproc.kernel
def vision_preproc(img):
    img = devproc.resize(img, (224, 224))
    img = devproc.to(img, devproc.Float32)
    return img
ir = devproc.parse_ir(vision_preproc, torch.randn(256, 256, 3))
res["dsl_vision_preproc"] = {"ops": [o.name for o in ir.block.ops], "inputs": [v.name for v in ir.inputs],
                             "out_shape": list(ir.output.type.shape)}
@devproc.kernel
def mlp(x, w1, b1, w2, b2):
    h = devproc.relu(devproc.linear(x, w1, b1))
    return devproc.argmax(devproc.linear(h, w2, b2))
ir = devproc.parse_ir(mlp, torch.randn(1, 128), torch.randn(256, 128), torch.randn(256), torch.randn(10, 256),
                      torch.randn(10))
res["dsl_mlp"] = {"ops": [o.name for o in ir.block.ops], "inputs": [v.name for v in ir.inputs]}
class MLP(torch.nn.Module):
    def __init__(s):
        super().__init__(); s.fc1 = torch.nn.Linear(128, 256); s.fc2 = torch.nn.Linear(256, 10)
    def forward(s, x):
        return s.fc2(torch.relu(s.fc1(x)))
ir = from_torch(MLP(), torch.randn(1, 128), backend="ir")
res["fx_mlp"] = {"ops": [o.name for o in ir.block.ops]}
ir = from_torch(torch.nn.Sequential(torch.nn.Linear(128, 256), torch.nn.ReLU()), torch.randn(1, 128), backend="ir")
res["fx_sequential"] = {"ops": [o.name for o in ir.block.ops]}
def f(x): return torch.sigmoid(x)
ir = from_torch(f, torch.randn(4, 8), backend="ir")
res["fx_sigmoid"] = {"ops": [o.name for o in ir.block.ops]}
print(json.dumps(res))
'''.replace("REF_SRC", repr(REF_SRC))
    r = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True, timeout=600)
    if r.returncode != 0:
        return {"error": r.stderr.strip().splitlines()[-1:]}
    return json.loads(r.stdout.strip().splitlines()[-1])


if __name__ == "__main__":
    main()
