"""The preprocessing pipeline on the host cores — CPU baseline (test infrastructure).

This is the reference's CPU formulation of the path: its resize handler's
``F.interpolate(mode="bilinear", align_corners=False)``
(src/devproc/backend/triton/ops.py:377-386) on float NCHW, the fp32 cast of
normalize_kernel (templates/elementwise.py:11-31) with the mean/std step,
the transpose (ops.py:418-420) and the final cast (elementwise.py:80-101),
run by torch on every host thread.  ``bench.py`` times it as the
``cpu_baseline`` and as the ``--impl reference`` arm; it is never part of the
product path.
"""

import os

import torch
import torch.nn.functional as F


def use_all_threads() -> int:
    n = os.cpu_count() or 1
    torch.set_num_threads(n)
    return n


def preprocess(images_nhwc_u8: torch.Tensor, out_hw=(224, 224), mean=None, std=None,
               out_dtype=torch.bfloat16) -> torch.Tensor:
    x = images_nhwc_u8.permute(0, 3, 1, 2).float()
    y = F.interpolate(x, size=out_hw, mode="bilinear", align_corners=False)
    if mean is not None:
        m = torch.tensor(mean, dtype=torch.float32).view(1, -1, 1, 1)
        s = torch.tensor(std, dtype=torch.float32).view(1, -1, 1, 1)
        y = (y - m) / s
    return y.contiguous().to(out_dtype)
