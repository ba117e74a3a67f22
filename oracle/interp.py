"""CPU IR interpreter — the oracle of the compiled-pipeline path (test infrastructure).

``run_function(fn, inputs, constants)`` executes an IR Function op by op with
torch on the CPU.  Every op's arithmetic is the definition the reference
itself uses for it (cited per op, paths inside the DevProc project):
its Triton templates are checked against exactly these torch functions in
src/devproc/tests/test_triton.py, and its resize/transpose handlers call them
directly.  Floating-point ops compute in fp32 and cast to the IR result type,
which is how the reference's templates accumulate (tl.float32).
"""

from typing import Dict, List

import torch
import torch.nn.functional as F

TD = {"uint8": torch.uint8, "int8": torch.int8, "int16": torch.int16, "int32": torch.int32,
      "int64": torch.int64, "float16": torch.float16, "bfloat16": torch.bfloat16, "float32": torch.float32,
      "float64": torch.float64, "bool": torch.bool}


def _out_dtype(v):
    t = v.type
    return TD[t.dtype]


def op_resize(x, size, layout):
    """Bilinear, align_corners=False, in fp32 with no rounding back to an
    integer type.  The reference's handler calls F.interpolate
    (src/devproc/backend/triton/ops.py:377-386); its CPU result depends on how
    torch splits the work across threads (vector body with FMA vs scalar tail,
    up to 2 ulp apart), so the oracle uses the deterministic restatement of
    that arithmetic in ``preproc_np`` (torch's vectorised path), which
    tests/test_oracle.py checks against F.interpolate."""
    import numpy as np
    from . import preproc_np
    xf = x.float()
    oh, ow = size
    if layout == "HWC":
        return torch.from_numpy(preproc_np.resize_nhwc(xf[None].numpy(), oh, ow)[0])
    if layout == "NHWC":
        return torch.from_numpy(preproc_np.resize_nhwc(xf.numpy(), oh, ow))
    if layout == "CHW":
        y = preproc_np.resize_nhwc(xf.permute(1, 2, 0)[None].numpy(), oh, ow)[0]
        return torch.from_numpy(np.ascontiguousarray(y.transpose(2, 0, 1)))
    if layout == "NCHW":
        y = preproc_np.resize_nhwc(xf.permute(0, 2, 3, 1).numpy(), oh, ow)
        return torch.from_numpy(np.ascontiguousarray(y.transpose(0, 3, 1, 2)))
    if layout == "HW":
        return torch.from_numpy(preproc_np.resize_nhwc(xf[None, :, :, None].numpy(), oh, ow)[0, :, :, 0])
    raise ValueError(layout)


def op_normalize(x, mean, std, channel_dim):
    """fp32 cast (reference normalize_kernel, templates/elementwise.py:11-31)
    then (x - mean[c]) / std[c] along ``channel_dim`` (the build's extension)."""
    xf = x.float()
    if mean is None:
        return xf
    shape = [1] * xf.dim()
    shape[channel_dim] = -1
    m = torch.tensor(mean, dtype=torch.float32).reshape(shape)
    s = torch.tensor(std, dtype=torch.float32).reshape(shape)
    return (xf - m) / s


def run_function(fn, inputs: Dict[str, torch.Tensor], constants: Dict[str, torch.Tensor] = None) -> List[torch.Tensor]:
    env: Dict[str, torch.Tensor] = {}
    constants = dict(getattr(fn, "constants", {}) or {}, **(constants or {}))
    for v in fn.inputs:
        src = constants[v.name] if v.name in constants else inputs[v.name]
        env[v.name] = src.detach().cpu().reshape(v.type.shape).to(TD[v.type.dtype])
    for op in fn.block.ops:
        x = [env[v.name] for v in op.inputs]
        out_v = op.outputs[0]
        env[out_v.name] = _eval(op, x, out_v)
    return [env[v.name] for v in fn.outputs]


def _cast(t, v):
    from devproc_b200.ir.types import ScalarType
    if isinstance(v.type, ScalarType):
        return t.to(TD[v.type.dtype])
    return t.to(_out_dtype(v))


def _eval(op, x, out_v):
    n = op.name
    a = op.attrs
    if n == "resize":
        return _cast(op_resize(x[0], a["size"], a["layout"]), out_v)
    if n == "normalize":
        return op_normalize(x[0], a.get("mean"), a.get("std"), a.get("channel_dim", -1))
    if n == "to":  # reference to_dtype_kernel, templates/elementwise.py:80-101
        return x[0].to(_out_dtype(out_v))
    if n == "transpose":  # reference handle_transpose, ops.py:418-420
        return x[0].permute(*a["dims"]).contiguous()
    if n == "reshape":
        return x[0].reshape(a["shape"])
    if n == "slice":
        idx = [slice(None)] * x[0].dim()
        idx[a["dim"]] = slice(a["start"], a["end"], a["step"])
        return x[0][tuple(idx)].contiguous()
    if n == "expand":
        return x[0].expand(a["shape"]).contiguous()
    if n == "cat":
        return torch.cat(x, dim=a["dim"])
    if n == "rope":  # out = x*cos + rotate_half(x)*sin, rotate_half(x) = [-x2, x1]
        xf, c, s_ = x[0].float(), x[1].float(), x[2].float()
        half = xf.shape[-1] // 2
        if c.shape[-1] == half:
            c = torch.cat([c, c], -1)
        if s_.shape[-1] == half:
            s_ = torch.cat([s_, s_], -1)
        rot = torch.cat([-xf[..., half:], xf[..., :half]], -1)
        return _cast(xf * c + rot * s_, out_v)
    if n == "matmul":  # reference test_triton.py:104 (torch.matmul), fp32 accumulate
        return _cast(torch.matmul(x[0].float(), x[1].float()), out_v)
    if n == "linear":  # reference linear_kernel, templates/matmul.py:152-156; test_triton.py:124
        b = x[2].float() if len(x) > 2 else None
        return _cast(F.linear(x[0].float(), x[1].float(), b), out_v)
    if n == "relu":  # test_triton.py:69
        return _cast(torch.relu(x[0].float()), out_v)
    if n == "sigmoid":  # test_triton.py:86
        return _cast(torch.sigmoid(x[0].float()), out_v)
    if n == "gelu":
        return _cast(F.gelu(x[0].float(), approximate=a.get("approximate", "none")), out_v)
    if n in ("tanh", "exp", "neg", "abs"):
        return _cast(getattr(torch, n)(x[0].float()), out_v)
    if n == "silu":
        return _cast(F.silu(x[0].float()), out_v)
    if n in ("add", "sub", "mul", "div"):  # add: test_triton.py:161
        f = {"add": torch.add, "sub": torch.sub, "mul": torch.mul, "div": torch.div}[n]
        return _cast(f(x[0].float(), x[1].float()), out_v)
    if n.endswith("_scalar"):
        base = n[:-7]
        c = torch.tensor(a["scalar"], dtype=torch.float32)
        l, r = (c, x[0].float()) if a.get("reverse") else (x[0].float(), c)
        f = {"add": torch.add, "sub": torch.sub, "mul": torch.mul, "div": torch.div}[base]
        return _cast(f(l, r), out_v)
    if n == "softmax":  # test_triton.py:178
        return _cast(torch.softmax(x[0].float(), dim=a["dim"]), out_v)
    if n == "argmax":  # test_triton.py:195, first index on ties
        return _cast(torch.argmax(x[0], dim=a["dim"], keepdim=a.get("keepdim", False)), out_v)
    if n in ("sum", "mean"):
        f = torch.sum if n == "sum" else torch.mean
        return _cast(f(x[0].float(), dim=a["dim"], keepdim=a.get("keepdim", False)), out_v)
    if n in ("max", "min"):
        f = torch.amax if n == "max" else torch.amin
        return _cast(f(x[0].float(), dim=a["dim"], keepdim=a.get("keepdim", False)), out_v)
    if n == "layer_norm":
        i = 1
        w = b = None
        if a["has_weight"]:
            w = x[i].float()
            i += 1
        if a["has_bias"]:
            b = x[i].float()
        xf = x[0].float()
        return _cast(F.layer_norm(xf, (xf.shape[-1],), w, b, a["eps"]), out_v)
    if n == "rms_norm":
        xf = x[0].float()
        y = xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + a["eps"])
        if a["has_weight"]:
            y = y * (x[1].float() + a.get("weight_offset", 0.0))
        return _cast(y, out_v)
    if n == "embedding":
        return F.embedding(x[0].long(), x[1])
    if n == "sdpa":
        q, k, v = (t.float() for t in x)
        if k.shape[-3] != q.shape[-3]:
            rep = q.shape[-3] // k.shape[-3]
            k = k.repeat_interleave(rep, dim=-3)
            v = v.repeat_interleave(rep, dim=-3)
        y = F.scaled_dot_product_attention(q, k, v, is_causal=a["is_causal"], scale=a["scale"])
        return _cast(y, out_v)
    raise NotImplementedError(f"oracle: op {n}")
