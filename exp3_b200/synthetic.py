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

import numpy as np
import torch


@dataclass(frozen=True)
class LayerShape:
    batch: int
    length: int
    heads: int
    kv_heads: int
    head_dim: int = 128


# Benchmark configurations 1, 2, 4 and 5 (single attention layer shapes), and the head-dim-256 layer.
CONFIGS = {
    "c1": (LayerShape(1, 4096, 28, 4), 8),
    "c2": (LayerShape(1, 32768, 28, 4), 32),
    "c4": (LayerShape(1, 131072, 28, 4), 128),
    "c5": (LayerShape(2, 65536, 40, 8), 0),
    "q35": (LayerShape(1, 32768, 16, 4, 256), 32),  # head dim 256 (Qwen3.5-4B full-attention layers)
}


def generator(seed: int, device="cpu") -> torch.Generator:
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    return g


def _np_rng(seed: int) -> np.random.Generator:
    return np.random.Generator(np.random.PCG64(seed))


def randn_bf16(shape, seed: int, device="cpu") -> torch.Tensor:
    """N(0, 1) rounded to bf16.

    On the CPU the draws come from numpy's PCG64 stream in float64 (generated in slices, so
    memory stays bounded) and are rounded to fp32 and then bf16: the bits are the same on
    every x86-64 host, which the golden fixtures rely on (torch's CPU sampler uses vectorised
    fp32 math whose last bits depend on the instruction set). On a GPU the device's own
    generator is used (fast, deterministic for a given GPU type)."""
    if torch.device(device).type != "cpu":
        return torch.randn(shape, generator=generator(seed, device), device=device,
                           dtype=torch.float32).to(torch.bfloat16)
    out = torch.empty(shape, dtype=torch.bfloat16)
    flat = out.view(-1)
    rng = _np_rng(seed)
    step = 1 << 24
    for lo in range(0, flat.numel(), step):
        n = min(step, flat.numel() - lo)
        flat[lo:lo + n] = torch.from_numpy(rng.standard_normal(n).astype(np.float32)).to(torch.bfloat16)
    return out


def rope_tables(length: int, d: int, theta: float = 1e6, offset: int = 0):
    """fp32 cos / sin [length, d] of NeoX RoPE, evaluated in float64 and rounded once."""
    inv_freq = 1.0 / (theta ** (np.arange(0, d, 2, dtype=np.float64) / d))
    freqs = np.outer(np.arange(offset, offset + length, dtype=np.float64), inv_freq)
    emb = np.concatenate((freqs, freqs), axis=-1)
    return torch.from_numpy(np.cos(emb).astype(np.float32)), torch.from_numpy(np.sin(emb).astype(np.float32))


def rope(x: torch.Tensor, theta: float = 1e6, offset: int = 0) -> torch.Tensor:
    """NeoX half-rotation RoPE on [B, L, H, d] (HF Qwen2 ``apply_rotary_pos_emb``)."""
    d = x.shape[-1]
    cos, sin = rope_tables(x.shape[1], d, theta, offset)
    cos, sin = cos.to(x.device)[None, :, None, :], sin.to(x.device)[None, :, None, :]
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
    rng = _np_rng(seed + 3)
    group = h // hkv
    if structured_sigma > 0:
        blocks = (length + 127) // 128
        direction = rng.standard_normal((b, 1, hkv, d))
        direction = direction / np.linalg.norm(direction, axis=-1, keepdims=True) * d ** 0.5
        offsets = rng.standard_normal((b, blocks, hkv, 1)) * structured_sigma
        shift = torch.from_numpy((offsets * direction).astype(np.float32))
        shift = shift.repeat_interleave(128, dim=1)[:, :length]
        k = (k.float() + shift.to(device)).to(torch.bfloat16)
        lean = torch.from_numpy((direction * 0.25).astype(np.float32)).repeat_interleave(group, dim=2)
        q = (q.float() + lean.to(device)).to(torch.bfloat16)
    if key_lognormal_sigma > 0:
        norms = np.exp(rng.standard_normal((b, length, hkv, 1)) * key_lognormal_sigma)
        k = (k.float() * torch.from_numpy(norms.astype(np.float32)).to(device)).to(torch.bfloat16)
    for n in range(needles):
        kv = n % hkv
        pos = int(rng.integers(0, max(1, length - 128)))
        row = int(rng.integers(pos + 1, length)) if pos + 1 < length else pos
        head = kv * group + int(rng.integers(0, group))
        bi = int(rng.integers(0, b))
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
