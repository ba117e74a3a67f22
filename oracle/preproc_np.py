"""numpy restatement of the preprocessing arithmetic (test infrastructure).

The reference's resize handler calls torch's ``F.interpolate(mode="bilinear",
align_corners=False)`` (src/devproc/backend/triton/ops.py:377-386); torch
(torch==2.11.0, the version in this image; the reference pins none) is a
third-party dependency outside the reference tree.  This module restates the
published algorithm of its CPU ``upsample_bilinear2d`` kernel step by step in
fp32 so the oracle's resize can be pinned independently of torch:

  scale = in / out;  src = fma(scale, o + 0.5, -0.5), negative → 0;
  i0 = min(floor(src), in - 1);  l1 = clamp(src - i0, 0, 1);  l0 = 1 - l1;
  i1 = i0 + (i0 < in - 1);  equal sizes copy (i1 = i0, l0 = 1, l1 = 0);
  row = fma(x[i0], l0, x[i1] * l1);  out = fma(row(y0), h0, row(y1) * h1)

(fma = one rounding of the exact a·b + c, emulated in float64, which is exact
for these operand sizes).  Normalisation is ((v - mean) / std) in fp32.
"""

import numpy as np

f32, f64 = np.float32, np.float64


def _fma(a, b, c):
    return (np.asarray(a, f64) * np.asarray(b, f64) + np.asarray(c, f64)).astype(f32)


def coefficients(in_size: int, out_size: int):
    o = np.arange(out_size)
    if in_size == out_size:
        return o, o, np.ones(out_size, f32), np.zeros(out_size, f32)
    scale = f32(in_size) / f32(out_size)
    src = _fma(scale, (o.astype(f32) + f32(0.5)), f32(-0.5))
    src = np.where(src < 0, f32(0), src).astype(f32)
    i0 = np.minimum(np.floor(src).astype(np.int64), in_size - 1)
    l1 = np.clip((src - i0.astype(f32)).astype(f32), f32(0), f32(1)).astype(f32)
    l0 = (f32(1) - l1).astype(f32)
    i1 = i0 + (i0 < in_size - 1)
    return i0, i1, l0, l1


def resize_nhwc(x: np.ndarray, out_h: int, out_w: int) -> np.ndarray:
    """[B, H, W, C] (any real dtype) → fp32 [B, out_h, out_w, C]."""
    xf = x.astype(f32)
    B, H, W, C = xf.shape
    y0, y1, h0, h1 = coefficients(H, out_h)
    x0, x1, w0, w1 = coefficients(W, out_w)
    w0b, w1b = w0[None, None, :, None], w1[None, None, :, None]
    r0 = xf[:, y0]
    r1 = xf[:, y1]
    row0 = _fma(r0[:, :, x0], w0b, (r0[:, :, x1] * w1b).astype(f32))
    row1 = _fma(r1[:, :, x0], w0b, (r1[:, :, x1] * w1b).astype(f32))
    return _fma(row0, h0[None, :, None, None], (row1 * h1[None, :, None, None]).astype(f32))


def preprocess_nhwc(x: np.ndarray, out_h: int, out_w: int, mean, std) -> np.ndarray:
    """Resize + normalise + NHWC→NCHW, fp32 result (cast by the caller)."""
    y = resize_nhwc(x, out_h, out_w)
    y = ((y - np.asarray(mean, f32)).astype(f32) / np.asarray(std, f32)).astype(f32)
    return np.ascontiguousarray(y.transpose(0, 3, 1, 2))
