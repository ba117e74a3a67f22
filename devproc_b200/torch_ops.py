"""Torch-level ops that a model can call so that capture keeps them whole.

``devproc.rope(x, cos, sin)`` is a torch custom op (``devproc::rope``): in
eager mode it computes the rotary embedding with plain torch ops (the
definition the oracle uses too); under ``devproc.compile`` / Dynamo capture
it stays one graph node, which the FX frontend turns into the IR ``rope`` op
(one fused region on the GPU) instead of the slice / neg / cat / mul / add
chain of the textbook form.
"""

import torch


@torch.library.custom_op("devproc::rope", mutates_args=())
def rope(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
    """Rotate-half rotary embedding: out = x·cos + [-x2, x1]·sin, where x1 and
    x2 are the halves of the last dim; cos / sin broadcast to x and hold
    either the full last dim or its half.  Computed in fp32, returned in
    x's dtype."""
    h = x.shape[-1] // 2
    c, s = cos.float(), sin.float()
    if c.shape[-1] == h:
        c = torch.cat([c, c], -1)
    if s.shape[-1] == h:
        s = torch.cat([s, s], -1)
    xf = x.float()
    rot = torch.cat([-xf[..., h:], xf[..., :h]], -1)
    return (xf * c + rot * s).to(x.dtype)


@rope.register_fake
def _rope_fake(x, cos, sin):
    return torch.empty_like(x)


def rope_tables(positions: int, dim: int, base: float = 10000.0, dtype=torch.float32):
    """cos / sin tables [positions, dim] of the standard inverse-frequency
    schedule base^(-2i/dim), duplicated over the two halves."""
    inv = base ** (-torch.arange(0, dim, 2, dtype=torch.float64) / dim)
    ang = torch.arange(positions, dtype=torch.float64)[:, None] * inv[None, :]
    ang = torch.cat([ang, ang], -1)
    return torch.cos(ang).to(dtype), torch.sin(ang).to(dtype)
