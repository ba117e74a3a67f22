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
                 patch: int = 14, image: int = 224, seed: int = 1, dtype=torch.bfloat16, logits: bool = False):
        super().__init__()
        self.logits = logits
        self.patch = torch.nn.Conv2d(3, dim, kernel_size=patch, stride=patch)
        tokens = (image // patch) ** 2
        self.pos = torch.nn.Parameter(torch.zeros(1, tokens, dim))
        self.blocks = torch.nn.ModuleList([VitBlock(dim, heads, mlp, 1e-6) for _ in range(layers)])
        self.post_ln = torch.nn.LayerNorm(dim, eps=1e-6)
        self.head = torch.nn.Linear(dim, classes)
        g = torch.Generator().manual_seed(seed)
        with torch.no_grad():
            for name, prm in self.named_parameters():
                if name.endswith("bias"):
                    prm.zero_()
                elif ".ln" in name or name.startswith("post_ln"):
                    prm.fill_(1.0)
                else:
                    prm.copy_(torch.randn(prm.shape, generator=g) * 0.02)
        self.to(dtype)

    def forward(self, pixels):
        x = self.patch(pixels).flatten(2).transpose(1, 2)
        x = x + self.pos
        for blk in self.blocks:
            x = blk(x)
        x = self.post_ln(x)
        y = self.head(x.mean(dim=1))
        return y if self.logits else y.argmax(-1)


def vit_flops_per_image(layers=27, dim=1152, mlp=4304, tokens=256, heads=16, classes=1000, patch_k=588):
    per_layer = 2 * tokens * dim * dim * 4 + 2 * tokens * dim * mlp * 2 + 2 * 2 * tokens * tokens * dim
    return layers * per_layer + 2 * tokens * patch_k * dim + 2 * dim * classes
