"""Seeded synthetic workloads of the benchmark configurations.

No datasets or checkpoints: inputs are seeded random tensors with the shapes,
dtypes and value distributions of each configuration (data seed 0, weight
seed 1), and models are random-init modules of the stated architecture.

* ``vision_preprocess`` — uint8 NHWC images → bilinear 224×224 → fp32 →
  (x - mean) / std → CHW → bf16 (the 256-image preprocessing pipeline).
* ``TokenPipeline`` — int32 ids [8, 128] → Embedding(32000, 512) → Linear
  512→2048 → GELU → Linear 2048→512 → LayerNorm(512) → Linear 512→32000 →
  argmax → int32 (the fp32 token pipeline).
"""

import math

import torch

from .dsl import ops as dp
from .dsl.kernel import kernel
from .dsl.types import BFloat16, Float32

IMAGENET_MEAN = (0.485 * 255, 0.456 * 255, 0.406 * 255)
IMAGENET_STD = (0.229 * 255, 0.224 * 255, 0.225 * 255)

PREPROC_BATCH, PREPROC_IN_H, PREPROC_IN_W, PREPROC_OUT = 256, 480, 640, 224
# Algorithmic HBM bytes of one preprocessed image: the 448 input rows that the
# 480→224 bilinear touches (every 32-byte sector of each is needed), plus the
# bf16 planar output.
PREPROC_ROWS_TOUCHED = 448
PREPROC_BYTES_PER_IMAGE = PREPROC_ROWS_TOUCHED * PREPROC_IN_W * 3 + 3 * PREPROC_OUT * PREPROC_OUT * 2


@kernel
def vision_preprocess(images):
    x = dp.resize(images, (PREPROC_OUT, PREPROC_OUT))
    x = dp.to(x, Float32)
    x = dp.normalize(x, IMAGENET_MEAN, IMAGENET_STD)
    x = dp.transpose(x, (0, 3, 1, 2))
    return dp.to(x, BFloat16)


def preprocess_images(batch: int = PREPROC_BATCH, h: int = PREPROC_IN_H, w: int = PREPROC_IN_W,
                      seed: int = 0) -> torch.Tensor:
    g = torch.Generator().manual_seed(seed)
    return torch.randint(0, 256, (batch, h, w, 3), generator=g, dtype=torch.uint8)


def rows_touched(in_size: int, out_size: int) -> int:
    """Distinct input rows a bilinear resize reads (for the bytes model)."""
    scale = in_size / out_size
    rows = set()
    for o in range(out_size):
        src = max(scale * (o + 0.5) - 0.5, 0.0)
        i0 = min(int(src), in_size - 1)
        rows.add(i0)
        rows.add(min(i0 + 1, in_size - 1))
    return len(rows)


class TokenPipeline(torch.nn.Module):
    VOCAB, DIM, FFN = 32000, 512, 2048

    def __init__(self, seed: int = 1):
        super().__init__()
        self.emb = torch.nn.Embedding(self.VOCAB, self.DIM)
        self.fc1 = torch.nn.Linear(self.DIM, self.FFN)
        self.fc2 = torch.nn.Linear(self.FFN, self.DIM)
        self.ln = torch.nn.LayerNorm(self.DIM)
        self.head = torch.nn.Linear(self.DIM, self.VOCAB)
        g = torch.Generator().manual_seed(seed)
        with torch.no_grad():
            for lin in (self.fc1, self.fc2, self.head):
                lin.weight.copy_(torch.randn(lin.weight.shape, generator=g) * 0.02)
                lin.bias.zero_()
            self.emb.weight.copy_(torch.randn(self.emb.weight.shape, generator=g) * 0.02)
            self.ln.weight.fill_(1.0)
            self.ln.bias.zero_()

    def forward(self, ids):
        x = self.emb(ids)
        x = torch.nn.functional.gelu(self.fc1(x))
        x = self.fc2(x)
        x = self.ln(x)
        return self.head(x).argmax(-1).to(torch.int32)


def token_ids(batch: int = 8, length: int = 128, seed: int = 0) -> torch.Tensor:
    g = torch.Generator().manual_seed(seed)
    return torch.randint(0, TokenPipeline.VOCAB, (batch, length), generator=g, dtype=torch.int32)


class VitAttention(torch.nn.Module):
    def __init__(self, dim: int, heads: int):
        super().__init__()
        self.heads = heads
        self.q = torch.nn.Linear(dim, dim)
        self.k = torch.nn.Linear(dim, dim)
        self.v = torch.nn.Linear(dim, dim)
        self.o = torch.nn.Linear(dim, dim)

    def forward(self, x):
        b, n, d = x.shape
        h = self.heads
        q = self.q(x).view(b, n, h, d // h).transpose(1, 2)
        k = self.k(x).view(b, n, h, d // h).transpose(1, 2)
        v = self.v(x).view(b, n, h, d // h).transpose(1, 2)
        o = torch.nn.functional.scaled_dot_product_attention(q, k, v)
        return self.o(o.transpose(1, 2).reshape(b, n, d))


class VitBlock(torch.nn.Module):
    def __init__(self, dim: int, heads: int, mlp: int, eps: float):
        super().__init__()
        self.ln1 = torch.nn.LayerNorm(dim, eps=eps)
        self.attn = VitAttention(dim, heads)
        self.ln2 = torch.nn.LayerNorm(dim, eps=eps)
        self.fc1 = torch.nn.Linear(dim, mlp)
        self.fc2 = torch.nn.Linear(mlp, dim)

    def forward(self, x):
        x = x + self.attn(self.ln1(x))
        return x + self.fc2(torch.nn.functional.gelu(self.fc1(self.ln2(x)), approximate="tanh"))


class VitClassifier(torch.nn.Module):
    """SigLIP-So400m/14-shaped encoder + mean-pool + linear head + argmax.

    Defaults are the benchmark's shape: patch 14 on 224×224 (256 tokens),
    width 1152, 27 layers, 16 heads, MLP 4304, GELU-tanh, LayerNorm (eps 1e-6),
    1000 classes; weights N(0, 0.02), biases 0, LayerNorm γ=1, β=0.
    """

    def __init__(self, layers: int = 27, dim: int = 1152, heads: int = 16, mlp: int = 4304, classes: int = 1000,
                 patch: int = 14, image: int = 224, seed: int = 1, dtype=torch.bfloat16, logits: bool = False,
                 device=None):
        super().__init__()
        self.logits = logits
        self.patch = torch.nn.Conv2d(3, dim, kernel_size=patch, stride=patch)
        tokens = (image // patch) ** 2
        self.pos = torch.nn.Parameter(torch.zeros(1, tokens, dim))
        self.blocks = torch.nn.ModuleList([VitBlock(dim, heads, mlp, 1e-6) for _ in range(layers)])
        self.post_ln = torch.nn.LayerNorm(dim, eps=1e-6)
        self.head = torch.nn.Linear(dim, classes)
        g = torch.Generator(device=device or "cpu").manual_seed(seed)
        with torch.no_grad():
            for name, prm in self.named_parameters():
                if name.endswith("bias"):
                    prm.zero_()
                elif ".ln" in name or name.startswith("post_ln"):
                    prm.fill_(1.0)
                else:
                    prm.copy_(torch.randn(prm.shape, generator=g, dtype=torch.float32, device=g.device) * 0.02)
        self.to(dtype)

    def encode(self, pixels):
        """Token features [B, tokens, dim] after the final LayerNorm."""
        x = self.patch(pixels).flatten(2).transpose(1, 2)
        x = x + self.pos
        for blk in self.blocks:
            x = blk(x)
        return self.post_ln(x)

    def forward(self, pixels):
        x = self.encode(pixels)
        y = self.head(x.mean(dim=1))
        return y if self.logits else y.argmax(-1)


def vit_flops_per_image(layers=27, dim=1152, mlp=4304, tokens=256, heads=16, classes=1000, patch_k=588):
    per_layer = 2 * tokens * dim * dim * 4 + 2 * tokens * dim * mlp * 2 + 2 * 2 * tokens * tokens * dim
    return layers * per_layer + 2 * tokens * patch_k * dim + 2 * dim * classes


# --------------------------------------------------------------- pi0.5-shaped
class DecoderBlock(torch.nn.Module):
    """Pre-norm decoder block of the Gemma family: RMSNorm → grouped-query
    attention with rotary embeddings → RMSNorm → GeGLU MLP (tanh GELU).
    ``forward`` returns the new hidden state and this layer's post-rotary
    keys and values; given ``prefix_kv`` the queries attend to the prefix
    keys / values followed by the block's own (bidirectionally)."""

    def __init__(self, dim: int, heads: int, kv_heads: int, head_dim: int, mlp: int, eps: float = 1e-6):
        super().__init__()
        self.heads, self.kv_heads, self.head_dim = heads, kv_heads, head_dim
        self.ln1 = torch.nn.RMSNorm(dim, eps=eps)
        self.q = torch.nn.Linear(dim, heads * head_dim, bias=False)
        self.k = torch.nn.Linear(dim, kv_heads * head_dim, bias=False)
        self.v = torch.nn.Linear(dim, kv_heads * head_dim, bias=False)
        self.o = torch.nn.Linear(heads * head_dim, dim, bias=False)
        self.ln2 = torch.nn.RMSNorm(dim, eps=eps)
        self.gate = torch.nn.Linear(dim, mlp, bias=False)
        self.up = torch.nn.Linear(dim, mlp, bias=False)
        self.down = torch.nn.Linear(mlp, dim, bias=False)

    def forward(self, x, cos, sin, prefix_k=None, prefix_v=None):
        from .torch_ops import rope
        b, n, _ = x.shape
        h = self.ln1(x)
        q = rope(self.q(h).view(b, n, self.heads, self.head_dim).transpose(1, 2), cos, sin)
        k = rope(self.k(h).view(b, n, self.kv_heads, self.head_dim).transpose(1, 2), cos, sin)
        v = self.v(h).view(b, n, self.kv_heads, self.head_dim).transpose(1, 2)
        ka, va = k, v
        if prefix_k is not None:
            ka = torch.cat([prefix_k, k], dim=2)
            va = torch.cat([prefix_v, v], dim=2)
        a = torch.nn.functional.scaled_dot_product_attention(q, ka, va, enable_gqa=True)
        x = x + self.o(a.transpose(1, 2).reshape(b, n, self.heads * self.head_dim))
        h = self.ln2(x)
        x = x + self.down(torch.nn.functional.gelu(self.gate(h), approximate="tanh") * self.up(h))
        return x, k, v


class Pi05Policy(torch.nn.Module):
    """pi0.5-shaped vision-language-action policy with random-init weights.

    Per sample: ``cams`` camera images (already preprocessed, bf16
    [3, 224, 224]) → the SigLIP-shaped encoder (no head) → projection to the
    language width; ``text`` token ids → embedding · √width; one prefill over
    image + text tokens through the Gemma-2B-shaped decoder (18 layers, width
    2048, 8 query heads sharing 1 key/value head of 256, GeGLU 16384) whose
    per-layer keys / values the action expert reads; then ``steps`` flow-
    matching denoise steps from N(0, 1) noise [horizon, action_dim] through
    the action expert (18 layers, width 1024, same heads, MLP 4096), each
    step x ← x − v(x, t) / steps with t = 1, 1 − 1/steps, …  Time enters as a
    sinusoidal embedding through a SiLU MLP added to the action tokens.
    Returns the denoised actions (fp32).
    """

    def __init__(self, cams: int = 3, text: int = 48, vocab: int = 257152, width: int = 2048, layers: int = 18,
                 heads: int = 8, kv_heads: int = 1, head_dim: int = 256, mlp: int = 16384,
                 expert_width: int = 1024, expert_layers: int = 18, expert_mlp: int = 4096,
                 horizon: int = 50, action_dim: int = 32, steps: int = 10, vit: dict = None, seed: int = 1,
                 dtype=torch.bfloat16, device=None):
        super().__init__()
        prev = torch.get_default_dtype()
        torch.set_default_dtype(dtype)  # build in the target dtype: no fp32 copy of ~3 B weights
        try:
            with torch.device(device or "cpu"):
                self._build(cams, text, vocab, width, layers, heads, kv_heads, head_dim, mlp, expert_width,
                            expert_layers, expert_mlp, horizon, action_dim, steps, dict(vit or {}), seed, dtype,
                            device)
        finally:
            torch.set_default_dtype(prev)

    def _build(self, cams, text, vocab, width, layers, heads, kv_heads, head_dim, mlp, expert_width, expert_layers,
               expert_mlp, horizon, action_dim, steps, vit, seed, dtype, device):
        from .torch_ops import rope_tables
        self.cams, self.steps = cams, steps
        self.width = width
        self.vision = VitClassifier(seed=seed, dtype=dtype, logits=True, device=device, **vit)
        vdim = self.vision.post_ln.normalized_shape[0]
        self.vision.head = torch.nn.Identity()
        self.img_tokens = cams * self.vision.pos.shape[1]
        self.proj = torch.nn.Linear(vdim, width)
        self.embed = torch.nn.Embedding(vocab, width)
        self.blocks = torch.nn.ModuleList([DecoderBlock(width, heads, kv_heads, head_dim, mlp) for _ in range(layers)])
        self.expert = torch.nn.ModuleList([DecoderBlock(expert_width, heads, kv_heads, head_dim, expert_mlp)
                                           for _ in range(expert_layers)])
        self.action_in = torch.nn.Linear(action_dim, expert_width)
        self.time_mlp = torch.nn.Sequential(torch.nn.Linear(expert_width, expert_width), torch.nn.SiLU(),
                                            torch.nn.Linear(expert_width, expert_width))
        self.final_ln = torch.nn.RMSNorm(expert_width, eps=1e-6)
        self.action_out = torch.nn.Linear(expert_width, action_dim)
        prefix = self.img_tokens + text
        cos, sin = rope_tables(prefix + horizon, head_dim)
        self.register_buffer("cos", cos.to(dtype))
        self.register_buffer("sin", sin.to(dtype))
        # sinusoidal embedding of t = 1, 1 - 1/steps, ..., 1/steps
        t = 1.0 - torch.arange(steps, dtype=torch.float64) / steps
        freq = torch.exp(-math.log(10000.0) * torch.arange(expert_width // 2, dtype=torch.float64) /
                         (expert_width // 2))
        ang = t[:, None] * 1000.0 * freq[None, :]
        self.register_buffer("t_emb", torch.cat([torch.sin(ang), torch.cos(ang)], -1).to(dtype))
        self.prefix = prefix
        # With ``device`` the draws come from that device's generator (a different
        # stream than the CPU default, which keeps building on a GPU fast).
        g = torch.Generator(device=device or "cpu").manual_seed(seed + 1)
        with torch.no_grad():
            for name, prm in self.named_parameters():
                if name.startswith("vision."):
                    continue
                if name.endswith("bias"):
                    prm.zero_()
                elif ".ln" in name or name.startswith("final_ln"):
                    prm.fill_(1.0)
                else:  # N(0, 0.02), drawn in fp32 one tensor at a time
                    prm.copy_(torch.randn(prm.shape, generator=g, dtype=torch.float32, device=g.device) * 0.02)

    def forward(self, pixels, text_ids, noise):
        b = text_ids.shape[0]
        vis = self.vision.encode(pixels)  # [b * cams, tokens, vdim]
        img = self.proj(vis.reshape(b, self.img_tokens, -1))
        txt = self.embed(text_ids) * math.sqrt(self.width)
        x = torch.cat([img, txt], dim=1)
        cos_p, sin_p = self.cos[: self.prefix], self.sin[: self.prefix]
        cos_e, sin_e = self.cos[self.prefix:], self.sin[self.prefix:]
        kv = []
        for blk in self.blocks:
            x, k, v = blk(x, cos_p, sin_p)
            kv.append((k, v))
        a = noise
        for s in range(self.steps):
            h = self.action_in(a.to(self.action_in.weight.dtype)) + self.time_mlp(self.t_emb[s])
            for blk, (k, v) in zip(self.expert, kv):
                h, _, _ = blk(h, cos_e, sin_e, k, v)
            vel = self.action_out(self.final_ln(h)).float()
            a = a - vel * (1.0 / self.steps)
        return a


def pi05_inputs(batch: int = 64, cams: int = 3, text: int = 48, vocab: int = 257152, horizon: int = 50,
                action_dim: int = 32, seed: int = 0):
    """(uint8 camera images [batch·cams, 480, 640, 3], int32 ids [batch, text], fp32 noise)."""
    g = torch.Generator().manual_seed(seed)
    imgs = torch.randint(0, 256, (batch * cams, PREPROC_IN_H, PREPROC_IN_W, 3), generator=g, dtype=torch.uint8)
    ids = torch.randint(0, vocab, (batch, text), generator=g, dtype=torch.int32)
    noise = torch.randn(batch, horizon, action_dim, generator=g)
    return imgs, ids, noise


def pi05_flops_per_sample(cams=3, text=48, width=2048, layers=18, heads=8, kv_heads=1, head_dim=256, mlp=16384,
                          expert_width=1024, expert_layers=18, expert_mlp=4096, horizon=50, action_dim=32, steps=10,
                          vit_layers=27):
    """Multiply-add FLOPs (2 per MAC) of one sample: vision, projection,
    prefill and the denoise steps (GEMMs and attention)."""
    img = cams * 256
    prefix = img + text
    vision = cams * vit_flops_per_image(layers=vit_layers, classes=0)
    proj = 2 * img * 1152 * width
    qkvo = 2 * width * head_dim * (2 * heads + 2 * kv_heads)
    prefill = layers * (prefix * (qkvo + 2 * 3 * width * mlp) + 2 * 2 * heads * prefix * prefix * head_dim)
    eq = 2 * expert_width * head_dim * (2 * heads + 2 * kv_heads)
    per_step = expert_layers * (horizon * (eq + 2 * 3 * expert_width * expert_mlp)
                                + 2 * 2 * heads * horizon * (prefix + horizon) * head_dim)
    per_step += 2 * horizon * (action_dim * expert_width * 2) + 2 * 2 * expert_width * expert_width
    return vision + proj + prefill + steps * per_step
