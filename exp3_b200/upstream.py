"""The public entry points of exp3's ``upstream/flashprefill_native_forward.py`` on libfpx.

Same names, arguments, return types and layouts ([batch, sequence, heads, dim]) as
the reference module (``upstream:420-533``); every op allocates fresh outputs and
never mutates its inputs. The Triton kernels and ``torch.compile`` helpers of the
reference are replaced by the CUDA kernels of libfpx (routing: csrc/route.cu;
exact path: csrc/attn_*.cu). Each op is also the PyTorch custom op
``torch.ops.fpx.<name>`` (with a fake implementation), which the public functions call.
"""

from __future__ import annotations

import torch

from . import _capi
from ._capi import call, ptr, require_cuda, stream, strides3

SCORE_IMPL = "v1_kmean_qt_row_reduce"
LSE_IMPL = "natural_log_exact_lse"

# Physical tiles of the kernels, reported like the reference's autotuned configs
# (upstream:524-533): the exact kernel runs 128-row query tiles over 64-key sub-tiles,
# the V1 scoring kernel scores 8 key blocks per tensor-core tile.
Q_TILE_SIZE, K_TILE_SIZE, SCORE_K_TILE_SIZE = 128, 64, 8


def _blocks(length: int, block_size: int) -> int:
    return (length + block_size - 1) // block_size


def _check_bf16(*tensors):
    for t in tensors:
        if t.dtype != torch.bfloat16:
            raise TypeError(f"expected bfloat16 tensors, got {t.dtype}")


@torch.library.custom_op("fpx::block_mean_k", mutates_args=())
def _block_mean_k(k: torch.Tensor, block_size: int) -> torch.Tensor:
    dev = require_cuda(k)
    _check_bf16(k)
    batch, sequence, kv_heads, head_dim = k.shape
    mean = torch.empty(batch, _blocks(sequence, block_size), kv_heads, head_dim, dtype=k.dtype, device=dev)
    call("fpx_block_mean_k", ptr(k), *strides3(k), batch, sequence, kv_heads, head_dim, block_size,
         ptr(mean), stream(dev))
    return mean


@_block_mean_k.register_fake
def _(k, block_size):
    batch, sequence, kv_heads, head_dim = k.shape
    return k.new_empty(batch, _blocks(sequence, block_size), kv_heads, head_dim)


@torch.no_grad()
def block_mean_k(k: torch.Tensor, block_size: int = 128) -> torch.Tensor:
    """``upstream:420-442``: bf16 mean of each (block, KV head) -> [B, nb, Hkv, d]."""
    return torch.ops.fpx.block_mean_k(k, block_size)


@torch.library.custom_op("fpx::v1_scores", mutates_args=())
def _v1_scores(q: torch.Tensor, mean_k: torch.Tensor, scale: float, block_size: int) -> torch.Tensor:
    dev = require_cuda(q, mean_k)
    _check_bf16(q, mean_k)
    batch, sequence, heads, head_dim = q.shape
    blocks, kv_heads = mean_k.shape[1], mean_k.shape[2]
    mean_k = mean_k.contiguous()
    score = torch.empty(batch, blocks, blocks, heads, dtype=torch.float32, device=dev)
    call("fpx_v1_scores", ptr(q), *strides3(q), ptr(mean_k), batch, sequence, heads, kv_heads, head_dim,
         block_size, float(scale), ptr(score), stream(dev))
    return score


@_v1_scores.register_fake
def _(q, mean_k, scale, block_size):
    blocks = mean_k.shape[1]
    return q.new_empty(q.shape[0], blocks, blocks, q.shape[2], dtype=torch.float32)


@torch.no_grad()
def v1_scores(q: torch.Tensor, mean_k: torch.Tensor, scale: float, block_size: int = 128) -> torch.Tensor:
    """``upstream:445-475``: normalised V1 proxy scores [B, nb, nb, H] fp32."""
    return torch.ops.fpx.v1_scores(q, mean_k, float(scale), block_size)


@torch.library.custom_op("fpx::deal_output_score", mutates_args=())
def _deal_output_score(score: torch.Tensor, attention_sink: int, window: int, alpha: float,
                       last_n_blocks_full: int, min_budget: int) -> tuple[torch.Tensor, torch.Tensor]:
    dev = require_cuda(score)
    score = score.float().contiguous()
    batch, query_blocks, key_blocks, heads = score.shape
    if query_blocks != key_blocks:
        raise ValueError("score must be [B, nb, nb, H]")
    indices = torch.empty(batch, query_blocks, key_blocks, heads, dtype=torch.int64, device=dev)
    counts = torch.empty(batch, query_blocks, heads, dtype=torch.int32, device=dev)
    call("fpx_deal_output_score", ptr(score), batch, key_blocks, heads, attention_sink, window, float(alpha),
         last_n_blocks_full, min_budget, ptr(indices), ptr(counts), stream(dev))
    return indices, counts


@_deal_output_score.register_fake
def _(score, attention_sink, window, alpha, last_n_blocks_full, min_budget):
    batch, query_blocks, _, heads = score.shape
    return (score.new_empty(score.shape, dtype=torch.int64),
            score.new_empty(batch, query_blocks, heads, dtype=torch.int32))


@torch.no_grad()
def deal_output_score(score: torch.Tensor, attention_sink: int, window: int, alpha: float = 0.1,
                      last_n_blocks_full: int = 2, min_budget: int = 0):
    """``upstream:388-407``: (int64 indices [B, nb, nb, H] with sentinel nb, int32 counts [B, nb, H])."""
    return torch.ops.fpx.deal_output_score(score, attention_sink, window, float(alpha), last_n_blocks_full,
                                           min_budget)


@torch.library.custom_op("fpx::exact_attention", mutates_args=())
def _exact_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, indices: torch.Tensor,
                     counts: torch.Tensor, scale: float, block_size: int) -> tuple[torch.Tensor, torch.Tensor]:
    dev = require_cuda(q, k, v, indices, counts)
    _check_bf16(q, k, v)
    batch, sequence, heads, head_dim = q.shape
    output = torch.empty(batch, sequence, heads, head_dim, dtype=q.dtype, device=dev)
    lse = torch.empty(batch, sequence, heads, dtype=torch.float32, device=dev)
    indices = indices.to(torch.int64).contiguous()
    counts = counts.to(torch.int32).contiguous()
    call("fpx_exact_attention", ptr(q), *strides3(q), ptr(k), *strides3(k), ptr(v), *strides3(v),
         ptr(indices), ptr(counts), batch, sequence, heads, k.shape[2], head_dim, block_size, float(scale),
         ptr(output), ptr(lse), stream(dev))
    return output, lse


@_exact_attention.register_fake
def _(q, k, v, indices, counts, scale, block_size):
    return torch.empty_like(q, memory_format=torch.contiguous_format), q.new_empty(q.shape[:3], dtype=torch.float32)


@torch.no_grad()
def exact_attention(q, k, v, indices, counts, scale: float, block_size: int = 128):
    """``upstream:478-521``: (bf16 output [B, L, H, d], fp32 natural LSE [B, L, H])."""
    return torch.ops.fpx.exact_attention(q, k, v, indices, counts, float(scale), block_size)


def attention_tile_sizes():
    """``upstream:524-528``: (query tile, key tile) of the exact kernel."""
    return Q_TILE_SIZE, K_TILE_SIZE


def score_tile_size():
    """``upstream:531-533``: key blocks per scoring tile."""
    return SCORE_K_TILE_SIZE


__all__ = ["SCORE_IMPL", "LSE_IMPL", "block_mean_k", "v1_scores", "deal_output_score", "exact_attention",
           "attention_tile_sizes", "score_tile_size"]
_ = _capi
