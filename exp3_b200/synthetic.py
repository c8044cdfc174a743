"""Seeded synthetic inputs with the shapes of the benchmark configurations.

The reference measures on RULER / LongBench prompts through Qwen2.5-7B; none of
that data is used here. These generators stand in for it with the shapes and
value distributions the benchmark configurations name: Q/K/V ~ N(0, 1) in bf16,
NeoX-style RoPE (theta 1e6, as HF Qwen2) on Q and K, and planted "needle" key
rows that copy a later query row of the same KV group scaled by 4, so a
query-to-key match exists far back in the sequence.

``structured_sigma`` adds a labelled block-structured variant: every key block
of a KV head is offset along one random direction by a per-block amount
a_b ~ N(0, sigma^2), and the queries of that group lean on the same direction.
With iid inputs every selector keeps ~100% of causal blocks (block means of iid
keys are all alike); the structured variant gives the routing real sparsity.
"""

from __future__ import annotations

import hashlib
from dataclasses import dataclass

import torch


@dataclass(frozen=True)
class LayerShape:
    batch: int
    length: int
    heads: int
    kv_heads: int
    head_dim: int = 128


# Benchmark configurations 1, 2, 4 and 5 (single attention layer shapes).
CONFIGS = {
    "c1": (LayerShape(1, 4096, 28, 4), 8),
    "c2": (LayerShape(1, 32768, 28, 4), 32),
    "c4": (LayerShape(1, 131072, 28, 4), 128),
    "c5": (LayerShape(2, 65536, 40, 8), 0),
}


def generator(seed: int, device="cpu") -> torch.Generator:
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    return g


def randn_bf16(shape, seed: int, device="cpu") -> torch.Tensor:
    """N(0, 1) rounded to bf16, from a seeded generator on ``device``."""
    return torch.randn(shape, generator=generator(seed, device), device=device,
                       dtype=torch.float32).to(torch.bfloat16)


def rope(x: torch.Tensor, theta: float = 1e6, offset: int = 0) -> torch.Tensor:
    """NeoX half-rotation RoPE on [B, L, H, d] (HF Qwen2 ``apply_rotary_pos_emb``)."""
    d = x.shape[-1]
    inv_freq = 1.0 / (theta ** (torch.arange(0, d, 2, device=x.device, dtype=torch.float32) / d))
    pos = torch.arange(offset, offset + x.shape[1], device=x.device, dtype=torch.float32)
    freqs = torch.outer(pos, inv_freq)
    emb = torch.cat((freqs, freqs), dim=-1)
    cos, sin = emb.cos()[None, :, None, :], emb.sin()[None, :, None, :]
    xf = x.float()
    half = d // 2
    rotated = torch.cat((-xf[..., half:], xf[..., :half]), dim=-1)
    return (xf * cos + rotated * sin).to(x.dtype)


def attention_inputs(shape: LayerShape, seed: int = 0, needles: int = 0, device="cpu",
                     apply_rope: bool = True, structured_sigma: float = 0.0,
                     key_lognormal_sigma: float = 0.0):
    """q [B, L, H, d], k / v [B, L, Hkv, d] bf16, contiguous."""
    b, length, h, hkv, d = shape.batch, shape.length, shape.heads, shape.kv_heads, shape.head_dim
    q = randn_bf16((b, length, h, d), seed, device)
    k = randn_bf16((b, length, hkv, d), seed + 1, device)
    v = randn_bf16((b, length, hkv, d), seed + 2, device)
    g = generator(seed + 3, "cpu")
    group = h // hkv
    if structured_sigma > 0:
        blocks = (length + 127) // 128
        direction = torch.randn(b, 1, hkv, d, generator=g)
        direction = direction / direction.norm(dim=-1, keepdim=True) * d ** 0.5
        offsets = torch.randn(b, blocks, hkv, 1, generator=g) * structured_sigma
        shift = (offsets * direction).repeat_interleave(128, dim=1)[:, :length]
        k = (k.float() + shift.to(device)).to(torch.bfloat16)
        lean = direction.repeat_interleave(group, dim=2) * 0.25
        q = (q.float() + lean.to(device)).to(torch.bfloat16)
    if key_lognormal_sigma > 0:
        norms = torch.exp(torch.randn(b, length, hkv, 1, generator=g) * key_lognormal_sigma)
        k = (k.float() * norms.to(device)).to(torch.bfloat16)
    for n in range(needles):
        kv = n % hkv
        pos = int(torch.randint(0, max(1, length - 128), (1,), generator=g))
        row = int(torch.randint(pos + 1, length, (1,), generator=g)) if pos + 1 < length else pos
        head = kv * group + int(torch.randint(0, group, (1,), generator=g))
        bi = int(torch.randint(0, b, (1,), generator=g))
        k[bi, pos, kv] = (q[bi, row, head].float() * 4.0).to(torch.bfloat16)
    if apply_rope:
        q, k = rope(q), rope(k)
    return q.contiguous(), k.contiguous(), v.contiguous()


def config_inputs(name: str, seed: int = 0, device="cpu", **overrides):
    shape, needles = CONFIGS[name]
    kwargs = {"needles": needles}
    if name == "c5":
        kwargs["key_lognormal_sigma"] = 0.5
    kwargs.update(overrides)
    return attention_inputs(shape, seed=seed, device=device, **kwargs)


def tensor_digest(*tensors: torch.Tensor) -> str:
    """sha256 over the raw bytes of CPU tensors (pins regenerated fixture inputs)."""
    h = hashlib.sha256()
    for t in tensors:
        t = t.detach().cpu().contiguous()
        if t.dtype == torch.bfloat16:
            t = t.view(torch.int16)
        h.update(t.numpy().tobytes())
    return h.hexdigest()
