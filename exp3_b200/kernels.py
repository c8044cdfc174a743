"""The public entry points of exp3's ``kernels.py`` on libfpx.

Same names, arguments, return types and layouts as the reference (``kernels.py:10-407``).
Each op allocates fresh outputs and never mutates its inputs; the work runs in the
CUDA kernels of libfpx on the current stream. ``chunk_tiles`` is accepted for
signature compatibility: the kernels need no host-side chunking.

Every tensor op is also a PyTorch custom op (``torch.ops.fpx.<name>``, with a fake
implementation for shape propagation), and the public functions call through it, so
``torch.compile`` and fake-tensor tracing see each op as one opaque node.
"""

from __future__ import annotations

import math
from dataclasses import dataclass

import torch

from ._capi import METHOD_IDS, call, lib, ptr, require_cuda, stream, strides3

BLOCK_SIZE = 128
SELECTORS = ("mean_balanced", "cgf_mean", "dispersion_mean")


@dataclass
class BlockDescriptors:
    """``kernels.py:13-19``."""

    mean_k: torch.Tensor
    mean_v: torch.Tensor
    var_k: torch.Tensor
    sigma_v: torch.Tensor
    counts: torch.Tensor


def _blocks(length, block_size):
    return (length + block_size - 1) // block_size


@torch.library.custom_op("fpx::block_descriptors", mutates_args=())
def _block_descriptors(k: torch.Tensor, v: torch.Tensor, block_size: int) -> tuple[
        torch.Tensor, torch.Tensor, torch.Tensor, torch.Tensor, torch.Tensor]:
    dev = require_cuda(k, v)
    batch, sequence, kv_heads, head_dim = k.shape
    blocks = _blocks(sequence, block_size)
    f32 = dict(dtype=torch.float32, device=dev)
    mean_k = torch.empty(batch, blocks, kv_heads, head_dim, **f32)
    mean_v, var_k = torch.empty_like(mean_k), torch.empty_like(mean_k)
    sigma_v = torch.empty(batch, blocks, kv_heads, **f32)
    counts = torch.empty(blocks, dtype=torch.int32, device=dev)
    call("fpx_block_descriptors", ptr(k), *strides3(k), ptr(v), *strides3(v), batch, sequence, kv_heads,
         head_dim, block_size, ptr(mean_k), ptr(mean_v), ptr(var_k), ptr(sigma_v), ptr(counts), stream(dev))
    return mean_k, mean_v, var_k, sigma_v, counts


@_block_descriptors.register_fake
def _(k, v, block_size):
    batch, sequence, kv_heads, head_dim = k.shape
    blocks = _blocks(sequence, block_size)
    mean_k = k.new_empty(batch, blocks, kv_heads, head_dim, dtype=torch.float32)
    return (mean_k, torch.empty_like(mean_k), torch.empty_like(mean_k),
            k.new_empty(batch, blocks, kv_heads, dtype=torch.float32), k.new_empty(blocks, dtype=torch.int32))


@torch.no_grad()
def block_descriptors(k: torch.Tensor, v: torch.Tensor, block_size: int = BLOCK_SIZE) -> BlockDescriptors:
    """``kernels.py:22-46``: fp32 mean/var of K, mean of V, sigma_v, valid-row counts."""
    return BlockDescriptors(*torch.ops.fpx.block_descriptors(k, v, block_size))


@torch.library.custom_op("fpx::selector_scores", mutates_args=())
def _selector_scores(q: torch.Tensor, mean_k: torch.Tensor, var_k: torch.Tensor, sigma_v: torch.Tensor,
                     counts: torch.Tensor, scale: float, selector: str, block_size: int) -> torch.Tensor:
    if selector not in SELECTORS:
        raise ValueError(f"unsupported selector: {selector}")
    dev = require_cuda(q)
    batch, sequence, heads, head_dim = q.shape
    blocks, kv_heads = mean_k.shape[1], mean_k.shape[2]
    scores = torch.empty(batch, blocks, blocks, heads, dtype=torch.float32, device=dev)
    mk, vk, sv = (x.float().contiguous() for x in (mean_k, var_k, sigma_v))
    call("fpx_selector_scores", ptr(q), *strides3(q), ptr(mk), ptr(vk), ptr(sv), ptr(counts.contiguous()),
         batch, sequence, heads, kv_heads, head_dim, block_size, METHOD_IDS[selector], float(scale),
         ptr(scores), stream(dev))
    return scores


@_selector_scores.register_fake
def _(q, mean_k, var_k, sigma_v, counts, scale, selector, block_size):
    blocks = mean_k.shape[1]
    return q.new_empty(q.shape[0], blocks, blocks, q.shape[2], dtype=torch.float32)


@torch.no_grad()
def selector_scores(q, descriptors: BlockDescriptors, scale: float, selector: str,
                    block_size: int = BLOCK_SIZE, chunk_tiles: int = 8) -> torch.Tensor:
    """``kernels.py:49-126``: [B, query block, key block, H] fp32."""
    if selector not in SELECTORS:
        raise ValueError(f"unsupported selector: {selector}")
    d = descriptors
    return torch.ops.fpx.selector_scores(q, d.mean_k, d.var_k, d.sigma_v, d.counts, float(scale), selector,
                                         block_size)


@torch.library.custom_op("fpx::protected_selection", mutates_args=())
def _protected_selection(scores: torch.Tensor, alpha: float, sink_blocks: int, window_blocks: int,
                         last_full_blocks: int) -> torch.Tensor:
    dev = require_cuda(scores)
    scores = scores.float().contiguous()
    batch, query_blocks, key_blocks, heads = scores.shape
    selected = torch.empty(scores.shape, dtype=torch.bool, device=dev)
    call("fpx_protected_selection", ptr(scores), batch, key_blocks, heads, float(alpha), sink_blocks,
         window_blocks, last_full_blocks, ptr(selected), stream(dev))
    return selected


@_protected_selection.register_fake
def _(scores, alpha, sink_blocks, window_blocks, last_full_blocks):
    return scores.new_empty(scores.shape, dtype=torch.bool)


@torch.no_grad()
def protected_selection(scores, alpha, sink_blocks, window_blocks, last_full_blocks) -> torch.Tensor:
    """``kernels.py:129-151``: bool [B, nb, nb, H]."""
    return torch.ops.fpx.protected_selection(scores, float(alpha), sink_blocks, window_blocks, last_full_blocks)


@torch.library.custom_op("fpx::indices_from_mask", mutates_args=())
def _indices_from_mask(selected: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    dev = require_cuda(selected)
    selected = selected.to(torch.bool).contiguous()
    batch, query_blocks, key_blocks, heads = selected.shape
    indices = torch.empty(selected.shape, dtype=torch.int64, device=dev)
    counts = torch.empty(batch, query_blocks, heads, dtype=torch.int32, device=dev)
    call("fpx_indices_from_mask", ptr(selected), batch, key_blocks, heads, ptr(indices), ptr(counts), stream(dev))
    return indices, counts


@_indices_from_mask.register_fake
def _(selected):
    batch, query_blocks, _, heads = selected.shape
    return (selected.new_empty(selected.shape, dtype=torch.int64),
            selected.new_empty(batch, query_blocks, heads, dtype=torch.int32))


@torch.no_grad()
def indices_from_mask(selected: torch.Tensor):
    """``kernels.py:154-160``."""
    return torch.ops.fpx.indices_from_mask(selected)


@torch.library.custom_op("fpx::mask_from_indices", mutates_args=())
def _mask_from_indices(indices: torch.Tensor, counts: torch.Tensor) -> torch.Tensor:
    dev = require_cuda(indices, counts)
    indices = indices.to(torch.int64).contiguous()
    counts = counts.to(torch.int32).contiguous()
    batch, query_blocks, key_blocks, heads = indices.shape
    selected = torch.empty(indices.shape, dtype=torch.bool, device=dev)
    call("fpx_mask_from_indices", ptr(indices), ptr(counts), batch, key_blocks, heads, ptr(selected), stream(dev))
    return selected


@_mask_from_indices.register_fake
def _(indices, counts):
    return indices.new_empty(indices.shape, dtype=torch.bool)


@torch.no_grad()
def mask_from_indices(indices: torch.Tensor, counts: torch.Tensor) -> torch.Tensor:
    """``kernels.py:163-176``."""
    return torch.ops.fpx.mask_from_indices(indices, counts)


@torch.library.custom_op("fpx::mean_tail", mutates_args=())
def _mean_tail(q: torch.Tensor, mean_k: torch.Tensor, mean_v: torch.Tensor, counts: torch.Tensor,
               selected: torch.Tensor, scale: float, block_size: int) -> tuple[torch.Tensor, torch.Tensor]:
    dev = require_cuda(q, selected)
    batch, sequence, heads, head_dim = q.shape
    kv_heads = mean_k.shape[2]
    out = torch.empty(batch, sequence, heads, head_dim, dtype=torch.float32, device=dev)
    lse = torch.empty(batch, sequence, heads, dtype=torch.float32, device=dev)
    mk, mv = mean_k.float().contiguous(), mean_v.float().contiguous()
    selected = selected.to(torch.bool).contiguous()
    call("fpx_mean_tail", ptr(q), *strides3(q), ptr(mk), ptr(mv), ptr(counts.contiguous()), ptr(selected),
         batch, sequence, heads, kv_heads, head_dim, block_size, float(scale), ptr(out), ptr(lse), stream(dev))
    return out, lse


def _fake_o_lse(q):
    return q.new_empty(q.shape, dtype=torch.float32), q.new_empty(q.shape[:3], dtype=torch.float32)


@_mean_tail.register_fake
def _(q, mean_k, mean_v, counts, selected, scale, block_size):
    return _fake_o_lse(q)


@torch.no_grad()
def mean_tail(q, descriptors: BlockDescriptors, selected, scale: float, block_size: int = BLOCK_SIZE,
              chunk_tiles: int = 8):
    """``kernels.py:179-230``: (fp32 output [B, L, H, d], fp32 LSE [B, L, H])."""
    d = descriptors
    return torch.ops.fpx.mean_tail(q, d.mean_k, d.mean_v, d.counts, selected, float(scale), block_size)


@torch.library.custom_op("fpx::rescue_tail", mutates_args=())
def _rescue_tail(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, selected: torch.Tensor, scale: float,
                 block_size: int, remainder: bool) -> tuple[torch.Tensor, torch.Tensor]:
    dev = require_cuda(q, k, v, selected)
    batch, sequence, heads, head_dim = q.shape
    kv_heads = k.shape[2]
    out = torch.empty(batch, sequence, heads, head_dim, dtype=torch.float32, device=dev)
    lse = torch.empty(batch, sequence, heads, dtype=torch.float32, device=dev)
    nbytes = lib().fpx_rescue_tail_workspace_bytes(batch, sequence, heads, kv_heads, head_dim, block_size)
    ws = torch.empty(max(nbytes, 1), dtype=torch.uint8, device=dev)
    selected = selected.to(torch.bool).contiguous()
    call("fpx_rescue_tail", ptr(q), *strides3(q), ptr(k), *strides3(k), ptr(v), *strides3(v), ptr(selected),
         batch, sequence, heads, kv_heads, head_dim, block_size, float(scale), 1 if remainder else 0,
         ptr(out), ptr(lse), ptr(ws), ws.numel(), stream(dev))
    return out, lse


@_rescue_tail.register_fake
def _(q, k, v, selected, scale, block_size, remainder):
    return _fake_o_lse(q)


@torch.no_grad()
def rescue_tail(q, k, v, selected, scale, block_size=BLOCK_SIZE, chunk_tiles=8, remainder=False):
    """``kernels.py:233-309``: exact attention to one rescue token per unselected full-history
    block (the key maximising the tile's mean query . k), with ``remainder`` also the block's
    other tokens through their mean with weight B - 1. Returns (fp32 O, fp32 natural LSE) over
    these entries only, for ``merge_exact_mean``. ``chunk_tiles`` only batches the reference's
    torch work and does not change the result."""
    return torch.ops.fpx.rescue_tail(q, k, v, selected, float(scale), block_size, bool(remainder))


@torch.library.custom_op("fpx::merge_exact_mean", mutates_args=())
def _merge_exact_mean(exact_output: torch.Tensor, exact_lse: torch.Tensor, mean_output: torch.Tensor,
                      mean_lse: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    dev = require_cuda(exact_output, exact_lse, mean_output, mean_lse)
    if exact_output.dtype != torch.bfloat16:
        raise TypeError("exact_output must be bfloat16")
    exact_output = exact_output.contiguous()
    mean_output = mean_output.float().contiguous()
    out = torch.empty_like(exact_output)
    lse = torch.empty(exact_lse.shape, dtype=torch.float32, device=dev)
    rows = exact_output.numel() // exact_output.shape[-1]
    call("fpx_merge_exact_mean", ptr(exact_output), ptr(exact_lse.float().contiguous()), ptr(mean_output),
         ptr(mean_lse.float().contiguous()), rows, exact_output.shape[-1], ptr(out), ptr(lse), stream(dev))
    return out, lse


@_merge_exact_mean.register_fake
def _(exact_output, exact_lse, mean_output, mean_lse):
    return torch.empty_like(exact_output), exact_lse.new_empty(exact_lse.shape, dtype=torch.float32)


@torch.no_grad()
def merge_exact_mean(exact_output, exact_lse, mean_output, mean_lse):
    """``kernels.py:312-325``: (output in exact_output's dtype, fp32 LSE)."""
    return torch.ops.fpx.merge_exact_mean(exact_output, exact_lse, mean_output, mean_lse)


@torch.library.custom_op("fpx::selection_counters", mutates_args=())
def _selection_counters(selected: torch.Tensor, sequence: int, block_size: int) -> torch.Tensor:
    """[exact token pairs, selected block entries, mean proxy entries] as int64 on the device."""
    dev = require_cuda(selected)
    selected = selected.to(torch.bool).contiguous()
    batch, blocks, _, heads = selected.shape
    counters = torch.empty(3, dtype=torch.int64, device=dev)
    call("fpx_selection_accounting", ptr(selected), batch, blocks, heads, sequence, block_size, ptr(counters),
         stream(dev))
    return counters


@_selection_counters.register_fake
def _(selected, sequence, block_size):
    return selected.new_empty(3, dtype=torch.int64)


@torch.no_grad()
def selection_accounting(selected, sequence, q_tile_size, k_tile_size, method, score_k_tile_size,
                         block_size: int = BLOCK_SIZE):
    """``kernels.py:328-407``; scalar device tensors where the reference returns tensors."""
    dev = require_cuda(selected)
    batch, blocks, _, heads = selected.shape
    counters = torch.ops.fpx.selection_counters(selected, sequence, block_size)
    exact_pairs, selected_blocks, mean_proxy_entries = counters[0], counters[1], counters[2]
    counts = [block_size] * (blocks - 1) + [sequence - (blocks - 1) * block_size]
    total_pairs = batch * heads * sequence * (sequence + 1) // 2
    causal_blocks = batch * heads * blocks * (blocks + 1) // 2
    history = sum(counts[qb] * qb for qb in range(blocks))  # rows x strictly-earlier blocks
    selector_proxy_entries = torch.tensor(history * batch * heads, dtype=torch.int64, device=dev)
    physical_tiles = None
    if q_tile_size is not None and k_tile_size is not None:
        programs = torch.tensor([(n + q_tile_size - 1) // q_tile_size for n in counts], dtype=torch.int64,
                                device=dev)
        per_row = selected.sum(dim=(0, 2, 3))
        physical_tiles = (per_row * programs).sum() * math.ceil(block_size / k_tile_size)
    mean_method = method in {"mean_native", "mean_balanced", "cgf_mean", "dispersion_mean",
                             "fp_v1_rescue", "fp_v1_rescue_v2"}
    executed_mean_entries = batch * sequence * heads * blocks if mean_method else 0
    selector_executed_entries = 0
    selector_physical_tiles = None
    if method in SELECTORS:
        selector_executed_entries = batch * sequence * heads * blocks * (1 if method == "mean_balanced" else 2)
    elif method in {"fp_v1", "mean_native", "fp_v1_rescue", "fp_v1_rescue_v2"} and score_k_tile_size is not None:
        selector_physical_tiles = sum(math.ceil((qb + 1) / score_k_tile_size) for qb in range(blocks)) * batch * heads
        selector_executed_entries = selector_physical_tiles * score_k_tile_size * block_size
    return {
        "effective_exact_token_pair_ratio": exact_pairs / total_pairs,
        "exact_token_pairs": exact_pairs,
        "causal_token_pairs": total_pairs,
        "legacy_block_density": selected_blocks / causal_blocks,
        "selected_block_entries": selected_blocks,
        "causal_block_entries": causal_blocks,
        "exact_physical_qk_tiles": physical_tiles,
        "mean_proxy_entries": mean_proxy_entries,
        "selector_proxy_entries": selector_proxy_entries,
        "mean_executed_logit_entries": executed_mean_entries,
        "mean_executed_value_entries": executed_mean_entries,
        "selector_executed_dot_entries": selector_executed_entries,
        "selector_physical_qk_tiles": selector_physical_tiles,
        "q_tile_size": q_tile_size,
        "k_tile_size": k_tile_size,
        "score_k_tile_size": score_k_tile_size,
    }
