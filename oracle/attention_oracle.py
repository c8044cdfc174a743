"""CPU restatement of exp3's block-sparse prefill attention — the parity checker.

TEST INFRASTRUCTURE ONLY. Only ``tests/``, ``__graft_entry__.smoke()`` and the
CPU legs of ``bench.py`` may import this module; the product never routes
through it.

Every function restates one reference function (file:line in the exp3 tree,
``upstream/`` meaning ``upstream/flashprefill_native_forward.py``) in plain
PyTorch on the CPU, in fp32 like the reference, and works one 128-row query
tile at a time so that 32K–128K sequences never materialise an ``[L, L]``
matrix. Functions that take ``tiles=`` compute only those query tiles, which is
how full-size parity tests and the timed CPU baseline sample a layer.

Pinning: ``tests/golden/make_golden.py`` runs the reference itself (its torch
functions on the CPU, and its Triton kernels under ``TRITON_INTERPRET=1`` in
fp32) and stores the outputs under ``tests/golden/``;
``tests/test_oracle_golden.py`` checks this module against them.

One deliberate definition: the reference's V1 block mean (``upstream:27-69``)
sums bf16 rows in bf16 in an order fixed by the autotuned warp count, so it
has no single bit pattern. Here (and in the CUDA kernel) it is the fp32
sequential sum over the block's valid rows, divided in fp32 by the row count
and rounded to bf16 (round-to-nearest-even); this meets the reference's own
block-mean check (``check_math.py:292-300``) and makes the V1 masks
reproducible bit for bit.
"""

from __future__ import annotations

import math
from dataclasses import dataclass

import numpy as np
import torch

BLOCK_SIZE = 128
LOG2E = 1.4426950408889634
LN2 = 0.6931471805599453
NEG_INF = float("-inf")

METHODS = (
    "dense",
    "fp_v1",
    "mean_native",
    "mean_balanced",
    "cgf_mean",
    "dispersion_mean",
    "fp_v1_rescue",
    "fp_v1_rescue_v2",
)
V1_ROUTED_METHODS = {"fp_v1", "mean_native", "fp_v1_rescue", "fp_v1_rescue_v2"}
MEAN_METHODS = {"mean_native", "mean_balanced", "cgf_mean", "dispersion_mean"}
RESCUE_METHODS = {"fp_v1_rescue", "fp_v1_rescue_v2"}
SELECTORS = ("mean_balanced", "cgf_mean", "dispersion_mean")

__all__ = [
    "BLOCK_SIZE", "METHODS", "V1_ROUTED_METHODS", "MEAN_METHODS", "RESCUE_METHODS", "SELECTORS",
    "BlockDescriptors", "num_blocks", "f32", "block_mean_k", "v1_scores",
    "deal_output_score", "block_descriptors", "selector_scores",
    "protected_selection", "indices_from_mask", "mask_from_indices",
    "exact_attention", "exact_attention_tiles", "mean_tail", "mean_tail_tiles",
    "merge_exact_mean", "selection_accounting", "dense_attention", "route",
    "prefill_attention_tiles", "exact_token_pairs", "threshold_band",
    "rescue_choice", "rescue_tail", "rescue_tail_tiles",
]


def num_blocks(length: int, block_size: int = BLOCK_SIZE) -> int:
    return (length + block_size - 1) // block_size


def f32(x: float) -> float:
    """Round a Python float to the nearest fp32 value."""
    return float(np.float32(x))


def _tile_rows(t: int, length: int, block_size: int) -> tuple[int, int]:
    return t * block_size, min(length, (t + 1) * block_size)


def _grouped(q_tile: torch.Tensor, kv_heads: int) -> torch.Tensor:
    """[B, rows, H, d] -> [B, rows, Hkv, G, d] with head h = kv * G + g."""
    b, rows, heads, d = q_tile.shape
    return q_tile.reshape(b, rows, kv_heads, heads // kv_heads, d)


# --------------------------------------------------------------------------- V1 routing


def block_mean_k(k: torch.Tensor, block_size: int = BLOCK_SIZE) -> torch.Tensor:
    """bf16 mean of the valid K rows of each (block, KV head).

    Reference: ``upstream:27-69`` (``compute_mean_vector``) and ``upstream:420-442``
    (``block_mean_k``). Order defined in the module docstring: fp32 sequential
    sum over rows, fp32 division by the valid count, RNE rounding to bf16.
    """
    batch, length, kv_heads, d = k.shape
    blocks = num_blocks(length, block_size)
    padded = np.zeros((batch, blocks * block_size, kv_heads, d), dtype=np.float32)
    padded[:, :length] = k.float().numpy()
    padded = padded.reshape(batch, blocks, block_size, kv_heads, d)
    acc = np.zeros((batch, blocks, kv_heads, d), dtype=np.float32)
    for r in range(block_size):  # sequential fp32 adds; padding rows add +0.0
        acc = acc + padded[:, :, r]
    counts = np.full((blocks,), block_size, dtype=np.float32)
    counts[-1] = length - (blocks - 1) * block_size
    mean = acc / counts.reshape(1, blocks, 1, 1)
    return torch.from_numpy(mean).to(torch.bfloat16)


def _v1_tile_scores(q_tile, mean_k, t, scale, block_size):
    """Normalised V1 proxy scores of one query tile: [B, nb, H] fp32.

    ``upstream:137-175``: x = (mk_b . q_i) * (scale * log2 e) for rows i with
    i >= 128 b + 127; per block M = max_i x and S = sum_i exp2(x - M).
    ``upstream:410-417``: score = S exp2(M - max M) / (sum + 1e-9); blocks with
    M = -inf score 0.
    """
    batch, rows, heads, _ = q_tile.shape
    blocks, kv_heads = mean_k.shape[1], mean_k.shape[2]
    scale_log2 = f32(f32(scale) * f32(LOG2E))
    x = torch.einsum(
        "brkgd,bnkd->bkgrn", _grouped(q_tile.float(), kv_heads), mean_k.float()
    ).reshape(batch, heads, rows, blocks) * scale_log2
    row_pos = t * block_size + torch.arange(rows)
    key_end = torch.arange(blocks) * block_size + block_size - 1
    causal = row_pos[:, None] >= key_end[None, :]
    x = x.masked_fill(~causal, NEG_INF)
    maximum = x.amax(dim=2)  # [B, H, nb]
    finite = maximum != NEG_INF
    safe_max = torch.where(finite, maximum, 0.0)
    mass = torch.where(causal, torch.exp2(x - safe_max[:, :, None, :]), 0.0).sum(dim=2)
    global_max = maximum.amax(dim=2, keepdim=True)
    rescaled = torch.where(finite, torch.exp2(maximum - global_max), 1.0)
    score = torch.where(finite, mass, 0.0) * rescaled
    score = score / (score.sum(dim=2, keepdim=True) + 1e-9)
    return score.permute(0, 2, 1).contiguous()  # [B, nb, H]


def v1_scores(q, mean_k, scale, block_size=BLOCK_SIZE, tiles=None):
    """``upstream:445-475`` (``v1_scores``) -> [B, nb, nb, H] fp32 (rows of ``tiles`` only)."""
    batch, length, heads, _ = q.shape
    blocks = mean_k.shape[1]
    out = torch.zeros(batch, blocks, blocks, heads, dtype=torch.float32)
    for t in range(blocks) if tiles is None else tiles:
        lo, hi = _tile_rows(t, length, block_size)
        out[:, t] = _v1_tile_scores(q[:, lo:hi], mean_k, t, scale, block_size)
    return out


def _protected(query_blocks, key_blocks, sink, window, last_full, rows=None):
    query_ids = torch.arange(query_blocks).view(1, query_blocks, 1, 1)
    if rows is not None:
        query_ids = torch.as_tensor(rows).view(1, -1, 1, 1)
    key_ids = torch.arange(key_blocks).view(1, 1, key_blocks, 1)
    distance = query_ids - key_ids
    protected = (
        (key_ids < sink)
        | ((distance >= 0) & (distance < window))
        | (query_ids >= query_blocks - last_full)
    )
    return protected, distance >= 0


def deal_output_score(score, attention_sink, window, alpha=0.1, last_n_blocks_full=2, min_budget=0):
    """``upstream:357-407``: threshold + protected regions -> sorted indices (sentinel nb), counts."""
    batch, query_blocks, key_blocks, heads = score.shape
    key_ids = torch.arange(key_blocks).view(1, 1, key_blocks, 1)
    if min_budget > 0:
        top_values, top_indices = torch.topk(score, k=min_budget, dim=2)
        keep = score >= top_values[:, :, :1, :] * alpha
        keep.scatter_(2, top_indices, True)
    else:
        keep = score >= score.amax(dim=2, keepdim=True) * alpha
    protected, causal = _protected(query_blocks, key_blocks, attention_sink, window, last_n_blocks_full)
    active = (keep | protected) & causal
    counts = active.sum(dim=2).to(torch.int32)
    indices = key_ids.expand(batch, query_blocks, key_blocks, heads)
    indices = indices.masked_fill(~active, key_blocks).sort(dim=2).values
    return indices.contiguous(), counts.contiguous()


def threshold_band(score, alpha):
    """|score - alpha * max_kb score| for V1 / new-selector thresholds (fp32, like the reference)."""
    return (score - score.amax(dim=2, keepdim=True) * alpha).abs()


# --------------------------------------------------------------------------- descriptors, selectors


@dataclass
class BlockDescriptors:
    """``kernels.py:13-19``."""

    mean_k: torch.Tensor
    mean_v: torch.Tensor
    var_k: torch.Tensor
    sigma_v: torch.Tensor
    counts: torch.Tensor


def block_descriptors(k, v, block_size=BLOCK_SIZE):
    """``kernels.py:22-46``: fp32 mean/var of K, mean of V, sigma_v = sqrt(sum_d var V)."""
    batch, length, kv_heads, d = k.shape
    blocks = num_blocks(length, block_size)
    padding = blocks * block_size - length
    kf = torch.nn.functional.pad(k.float(), (0, 0, 0, 0, 0, padding))
    vf = torch.nn.functional.pad(v.float(), (0, 0, 0, 0, 0, padding))
    kf = kf.reshape(batch, blocks, block_size, kv_heads, d)
    vf = vf.reshape(batch, blocks, block_size, kv_heads, d)
    counts = torch.full((blocks,), block_size, dtype=torch.int32)
    counts[-1] = length - (blocks - 1) * block_size
    den = counts.to(torch.float32).view(1, blocks, 1, 1)
    mean_k = kf.sum(dim=2) / den
    var_k = (kf.square().sum(dim=2) / den - mean_k.square()).clamp_min_(0)
    mean_v = vf.sum(dim=2) / den
    var_v = (vf.square().sum(dim=2) / den - mean_v.square()).clamp_min_(0)
    sigma_v = var_v.sum(dim=-1).sqrt_()
    return BlockDescriptors(mean_k, mean_v, var_k, sigma_v, counts)


def _selector_tile_scores(q_tile, desc, t, scale, selector):
    """``kernels.py:82-125`` for one tile: per-row softmax over blocks b < t, mean over rows."""
    batch, rows, heads, _ = q_tile.shape
    blocks, kv_heads = desc.mean_k.shape[1], desc.mean_k.shape[2]
    group = heads // kv_heads
    qg = _grouped(q_tile.float(), kv_heads)
    log_counts = desc.counts.to(torch.float32).log()
    visible = (torch.arange(blocks) < t).view(1, 1, 1, blocks)
    ell0 = torch.einsum("brkgd,bnkd->brkgn", qg, desc.mean_k).reshape(batch, rows, heads, blocks)
    ell0 = ell0 * scale + log_counts.view(1, 1, 1, blocks)
    dispersion = None
    if selector == "mean_balanced":
        logits = ell0
    else:
        u = torch.einsum("brkgd,bnkd->brkgn", qg.square(), desc.var_k).reshape(batch, rows, heads, blocks)
        u = (u * (scale * scale)).clamp_min(0)
        logits = ell0 + 0.5 * u
        if selector == "dispersion_mean":
            dispersion = u.sqrt()
    masked = logits.masked_fill(~visible, NEG_INF)
    normalizer = torch.logsumexp(masked, dim=-1, keepdim=True)
    probability = torch.where(visible, torch.exp(masked - normalizer), 0.0)
    if dispersion is not None:
        sigma_v = desc.sigma_v.repeat_interleave(group, dim=2).permute(0, 2, 1)  # [B, H, nb]
        probability = probability * dispersion * sigma_v[:, None]
    return probability.sum(dim=1) / float(rows)  # [B, H, nb]


def selector_scores(q, desc, scale, selector, block_size=BLOCK_SIZE, chunk_tiles=8, tiles=None):
    """``kernels.py:49-126`` -> [B, nb(query), nb(key), H] fp32."""
    if selector not in SELECTORS:
        raise ValueError(f"unsupported selector: {selector}")
    batch, length, heads, _ = q.shape
    blocks = desc.mean_k.shape[1]
    out = torch.zeros(batch, blocks, blocks, heads, dtype=torch.float32)
    for t in range(blocks) if tiles is None else tiles:
        lo, hi = _tile_rows(t, length, block_size)
        out[:, t] = _selector_tile_scores(q[:, lo:hi], desc, t, scale, selector).permute(0, 2, 1)
    return out


def protected_selection(scores, alpha, sink_blocks, window_blocks, last_full_blocks):
    """``kernels.py:129-151``."""
    batch, query_blocks, key_blocks, _ = scores.shape
    protected, causal = _protected(query_blocks, key_blocks, sink_blocks, window_blocks, last_full_blocks)
    if alpha == 0:
        return causal.expand_as(scores).clone()
    maximum = scores.amax(dim=2, keepdim=True)
    routed = (scores > 0) & (scores >= alpha * maximum)
    return (routed | protected) & causal


def indices_from_mask(selected):
    """``kernels.py:154-160``."""
    batch, query_blocks, key_blocks, heads = selected.shape
    key_ids = torch.arange(key_blocks).view(1, 1, key_blocks, 1)
    indices = key_ids.expand(batch, query_blocks, key_blocks, heads)
    indices = indices.masked_fill(~selected, key_blocks).sort(dim=2).values
    return indices.contiguous(), selected.sum(dim=2).to(torch.int32).contiguous()


def mask_from_indices(indices, counts):
    """``kernels.py:163-176``."""
    batch, query_blocks, key_blocks, heads = indices.shape
    positions = torch.arange(key_blocks).view(1, 1, key_blocks, 1)
    valid = positions < counts.unsqueeze(2)
    full = torch.zeros(batch, query_blocks, key_blocks + 1, heads, dtype=torch.bool)
    full.scatter_(2, indices.long(), valid)
    return full[:, :, :key_blocks]


# --------------------------------------------------------------------------- exact / mean / merge


def _exact_tile(q_tile, k, v, active_t, t, scale, block_size):
    """Exact attention of one query tile over its selected blocks (``upstream:291-354``).

    Returns fp32 O [B, rows, H, d] and natural-log LSE [B, rows, H]. Rows with no
    allowed key get O = 0 and LSE = -inf, as the reference kernel does.
    """
    batch, rows, heads, d = q_tile.shape
    kv_heads = k.shape[2]
    group = heads // kv_heads
    row_lo = t * block_size
    keys = min(k.shape[1], (t + 1) * block_size)
    key_pos = torch.arange(keys)
    kf, vf = k[:, :keys].float(), v[:, :keys].float()
    logits = torch.einsum("brkgd,bjkd->bkgrj", _grouped(q_tile.float(), kv_heads), kf) * scale
    allowed = active_t[:, key_pos // block_size, :]  # [B, keys, H]
    allowed = allowed.permute(0, 2, 1).reshape(batch, kv_heads, group, 1, keys)
    causal = key_pos[None, :] <= (row_lo + torch.arange(rows))[:, None]
    logits = logits.masked_fill(~(allowed & causal), NEG_INF)
    lse = torch.logsumexp(logits, dim=-1)  # [B, Hkv, G, rows]
    finite = lse != NEG_INF
    p = torch.where(finite[..., None], torch.exp(logits - torch.where(finite, lse, 0.0)[..., None]), 0.0)
    out = torch.einsum("bkgrj,bjkd->brkgd", p, vf).reshape(batch, rows, heads, d)
    return out, lse.reshape(batch, heads, rows).permute(0, 2, 1)


def exact_attention_tiles(q, k, v, selected, scale, block_size=BLOCK_SIZE, tiles=None):
    """Exact path over the tiles in ``tiles``: dict t -> (O fp32, LSE fp32)."""
    length = q.shape[1]
    blocks = num_blocks(length, block_size)
    result = {}
    for t in range(blocks) if tiles is None else tiles:
        lo, hi = _tile_rows(t, length, block_size)
        result[t] = _exact_tile(q[:, lo:hi], k, v, selected[:, t], t, scale, block_size)
    return result


def exact_attention(q, k, v, indices, counts, scale, block_size=BLOCK_SIZE):
    """``upstream:478-521``: bf16 O [B, L, H, d] and fp32 natural LSE [B, L, H]."""
    selected = mask_from_indices(indices, counts)
    out = torch.empty(q.shape, dtype=torch.float32)
    lse = torch.empty(q.shape[:3], dtype=torch.float32)
    for t, (o_t, l_t) in exact_attention_tiles(q, k, v, selected, scale, block_size).items():
        lo, hi = _tile_rows(t, q.shape[1], block_size)
        out[:, lo:hi], lse[:, lo:hi] = o_t, l_t
    return out.to(q.dtype), lse


def _mean_tile(q_tile, desc, active_t, t, scale):
    """``kernels.py:211-229`` for one tile: unselected blocks b < t via fp32 block means."""
    batch, rows, heads, d = q_tile.shape
    blocks, kv_heads = desc.mean_k.shape[1], desc.mean_k.shape[2]
    group = heads // kv_heads
    visible = (torch.arange(blocks) < t).view(1, blocks, 1)
    tail = (visible & ~active_t).view(batch, 1, blocks, heads).permute(0, 1, 3, 2)  # [B,1,H,nb]
    logits = torch.einsum("brkgd,bnkd->brkgn", _grouped(q_tile.float(), kv_heads), desc.mean_k)
    logits = logits.reshape(batch, rows, heads, blocks) * scale
    logits = logits + desc.counts.to(torch.float32).log().view(1, 1, 1, blocks)
    masked = logits.masked_fill(~tail, NEG_INF)
    lse = torch.logsumexp(masked, dim=-1)
    weights = torch.where(tail, torch.exp(masked - lse.unsqueeze(-1)), 0.0)
    mean_v = desc.mean_v.repeat_interleave(group, dim=2)
    out = torch.einsum("brhk,bkhd->brhd", weights, mean_v)
    return out, lse


def mean_tail_tiles(q, desc, selected, scale, block_size=BLOCK_SIZE, tiles=None):
    length = q.shape[1]
    blocks = desc.mean_k.shape[1]
    result = {}
    for t in range(blocks) if tiles is None else tiles:
        lo, hi = _tile_rows(t, length, block_size)
        result[t] = _mean_tile(q[:, lo:hi], desc, selected[:, t], t, scale)
    return result


def mean_tail(q, desc, selected, scale, block_size=BLOCK_SIZE, chunk_tiles=8):
    """``kernels.py:179-230``: fp32 O [B, L, H, d] and LSE [B, L, H] of the unselected tail."""
    out = torch.zeros(q.shape, dtype=torch.float32)
    lse = torch.full(q.shape[:3], NEG_INF, dtype=torch.float32)
    for t, (o_t, l_t) in mean_tail_tiles(q, desc, selected, scale, block_size).items():
        lo, hi = _tile_rows(t, q.shape[1], block_size)
        out[:, lo:hi], lse[:, lo:hi] = o_t, l_t
    return out, lse


def rescue_choice(q_tile, k, t, block_size=BLOCK_SIZE):
    """``kernels.py:276-285`` for one query tile: for every key block kb < t and head h, the
    token of kb maximising q_mean . k_j, with q_mean the fp32 mean of the tile's valid query
    rows. Returns int64 [B, H, t] token offsets (ties: the first maximum, as torch.argmax)."""
    batch, rows, heads, d = q_tile.shape
    kv_heads = k.shape[2]
    q_mean = q_tile.float().sum(dim=1) / float(rows)  # [B, H, d]
    k_blocks = k[:, : t * block_size].float().view(batch, t, block_size, kv_heads, d)
    scores = torch.einsum("bkgd,bnjkd->bkgnj", q_mean.view(batch, kv_heads, heads // kv_heads, d), k_blocks)
    return scores.argmax(dim=-1).reshape(batch, heads, t)


def _rescue_tile(q_tile, k, v, active_t, t, scale, block_size, remainder, choice=None):
    """``kernels.py:233-309`` (``rescue_tail``) for one tile: exact attention to one rescue
    token per unselected block kb < t, and with ``remainder`` the block's other B - 1 tokens
    through their mean K/V with weight B - 1. fp32 O [B, rows, H, d] and natural LSE."""
    batch, rows, heads, d = q_tile.shape
    kv_heads = k.shape[2]
    group = heads // kv_heads
    out = torch.zeros(batch, rows, heads, d)
    lse = torch.full((batch, rows, heads), NEG_INF)
    if t == 0:
        return out, lse
    if choice is None:
        choice = rescue_choice(q_tile, k, t, block_size)
    k_blocks = k[:, : t * block_size].float().view(batch, t, block_size, kv_heads, d)
    v_blocks = v[:, : t * block_size].float().view(batch, t, block_size, kv_heads, d)
    head_kv = torch.arange(heads) // group
    bi = torch.arange(batch).view(batch, 1, 1)
    ni = torch.arange(t).view(1, 1, t)
    ki = head_kv.view(1, heads, 1)
    k_res = k_blocks[bi, ni, choice, ki]  # [B, H, t, d]
    v_res = v_blocks[bi, ni, choice, ki]
    tail = (~active_t[:, :t, :]).permute(0, 2, 1)  # [B, H, t]
    qf = q_tile.float()
    logits = torch.einsum("brhd,bhnd->brhn", qf, k_res) * scale
    values = v_res
    mask = tail.unsqueeze(1)
    if remainder:
        k_sum = k_blocks.sum(dim=2)[:, :, head_kv].permute(0, 2, 1, 3)  # [B, H, t, d]
        v_sum = v_blocks.sum(dim=2)[:, :, head_kv].permute(0, 2, 1, 3)
        k_rest = (k_sum - k_res) / (block_size - 1)
        v_rest = (v_sum - v_res) / (block_size - 1)
        rest = torch.einsum("brhd,bhnd->brhn", qf, k_rest) * scale
        logits = torch.cat((logits, rest + math.log(block_size - 1)), dim=-1)
        values = torch.cat((values, v_rest), dim=2)
        mask = torch.cat((mask, mask), dim=-1)
    masked = logits.masked_fill(~mask, NEG_INF)
    lse = torch.logsumexp(masked, dim=-1)
    weights = torch.where(mask, torch.exp(masked - lse.unsqueeze(-1)), 0.0)
    out = torch.einsum("brhn,bhnd->brhd", weights, values)
    return out, lse


def rescue_tail_tiles(q, k, v, selected, scale, remainder=False, block_size=BLOCK_SIZE, tiles=None):
    """``kernels.py:233-309`` over the tiles in ``tiles``: dict t -> (O fp32, LSE fp32)."""
    length = q.shape[1]
    blocks = num_blocks(length, block_size)
    result = {}
    for t in range(blocks) if tiles is None else tiles:
        lo, hi = _tile_rows(t, length, block_size)
        result[t] = _rescue_tile(q[:, lo:hi], k, v, selected[:, t], t, scale, block_size, remainder)
    return result


def rescue_tail(q, k, v, selected, scale, block_size=BLOCK_SIZE, remainder=False):
    """``kernels.py:233-309``: fp32 O [B, L, H, d] and LSE [B, L, H] of the rescue entries."""
    out = torch.zeros(q.shape, dtype=torch.float32)
    lse = torch.full(q.shape[:3], NEG_INF, dtype=torch.float32)
    for t, (o_t, l_t) in rescue_tail_tiles(q, k, v, selected, scale, remainder, block_size).items():
        lo, hi = _tile_rows(t, q.shape[1], block_size)
        out[:, lo:hi], lse[:, lo:hi] = o_t, l_t
    return out, lse


def merge_exact_mean(exact_output, exact_lse, mean_output, mean_lse):
    """``kernels.py:312-325``: logaddexp merge; the exact output enters at its stored dtype."""
    total_lse = torch.logaddexp(exact_lse, mean_lse)
    exact_weight = torch.exp(exact_lse - total_lse)
    mean_weight = torch.exp(mean_lse - total_lse)
    output = exact_output.float() * exact_weight.unsqueeze(-1) + mean_output * mean_weight.unsqueeze(-1)
    return output.to(exact_output.dtype), total_lse


def dense_attention(q, k, v, scale, block_size=BLOCK_SIZE, tiles=None):
    """``check_math.py:33-42`` (causal dense, fp32), tile by tile: dict t -> (O, LSE)."""
    batch, length, heads, _ = q.shape
    blocks = num_blocks(length, block_size)
    every = torch.ones(batch, blocks, heads, dtype=torch.bool)
    result = {}
    for t in range(blocks) if tiles is None else tiles:
        lo, hi = _tile_rows(t, length, block_size)
        result[t] = _exact_tile(q[:, lo:hi], k, v, every, t, scale, block_size)
    return result


# --------------------------------------------------------------------------- accounting


def exact_token_pairs(selected, length, block_size=BLOCK_SIZE):
    """Exact (query, key) pairs of a selection, ``kernels.py:339-350``: full history
    blocks count n_q * n_k, the diagonal n (n + 1) / 2, summed over batch and heads."""
    batch, blocks, _, heads = selected.shape
    counts = torch.full((blocks,), block_size, dtype=torch.int64)
    counts[-1] = length - (blocks - 1) * block_size
    q_ids = torch.arange(blocks).view(blocks, 1)
    k_ids = torch.arange(blocks).view(1, blocks)
    weights = torch.where(
        k_ids < q_ids,
        counts.view(-1, 1) * counts.view(1, -1),
        torch.where(k_ids == q_ids, (counts * (counts + 1) // 2).view(-1, 1), 0),
    )
    return int((selected.to(torch.int64) * weights.view(1, blocks, blocks, 1)).sum())


def selection_accounting(selected, sequence, q_tile_size, k_tile_size, method, score_k_tile_size,
                         block_size=BLOCK_SIZE):
    """``kernels.py:328-407`` with Python ints."""
    batch, blocks, _, heads = selected.shape
    counts = torch.full((blocks,), block_size, dtype=torch.int64)
    counts[-1] = sequence - (blocks - 1) * block_size
    exact_pairs = exact_token_pairs(selected, sequence, block_size)
    total_pairs = batch * heads * sequence * (sequence + 1) // 2
    causal_blocks = batch * heads * blocks * (blocks + 1) // 2
    selected_blocks = int(selected.sum())
    q_ids = torch.arange(blocks).view(blocks, 1)
    k_ids = torch.arange(blocks).view(1, blocks)
    full_history = k_ids < q_ids
    tail = full_history.view(1, blocks, blocks, 1) & ~selected
    mean_proxy_entries = int((tail.to(torch.int64) * counts.view(1, blocks, 1, 1)).sum())
    selector_proxy_entries = int((full_history.to(torch.int64) * counts.view(blocks, 1)).sum()) * batch * heads
    physical_tiles = None
    if q_tile_size is not None and k_tile_size is not None:
        q_programs = (counts + q_tile_size - 1) // q_tile_size
        physical_tiles = int((selected.to(torch.int64) * q_programs.view(1, blocks, 1, 1)).sum()) * math.ceil(
            block_size / k_tile_size)
    mean_method = method in MEAN_METHODS | {"fp_v1_rescue", "fp_v1_rescue_v2"}
    executed_mean_entries = batch * sequence * heads * blocks if mean_method else 0
    selector_executed_entries = 0
    selector_physical_tiles = None
    if method in SELECTORS:
        selector_executed_entries = batch * sequence * heads * blocks * (1 if method == "mean_balanced" else 2)
    elif method in V1_ROUTED_METHODS and score_k_tile_size is not None:
        selector_physical_tiles = sum(
            math.ceil((qb + 1) / score_k_tile_size) for qb in range(blocks)) * batch * heads
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


# --------------------------------------------------------------------------- whole path


def route(method, q, k, v, scale, alpha, sink=2, window=4, last_full=2, block_size=BLOCK_SIZE, tiles=None):
    """Routing of ``attention.py:77-152``: returns (selected [B,nb,nb,H] bool, scores, descriptors).

    Only the rows of ``tiles`` (all when None) are filled; ``selected`` rows of
    other tiles are False.
    """
    length = q.shape[1]
    blocks = num_blocks(length, block_size)
    rows = list(range(blocks)) if tiles is None else list(tiles)
    desc = block_descriptors(k, v, block_size)
    if method == "dense":
        protected, causal = _protected(blocks, blocks, sink, window, last_full)
        selected = causal.expand(q.shape[0], blocks, blocks, q.shape[2]).clone()
        return selected, None, desc
    if method in V1_ROUTED_METHODS:
        mean_k = block_mean_k(k, block_size)
        scores = v1_scores(q, mean_k, scale, block_size, tiles=rows)
        keep = scores >= scores.amax(dim=2, keepdim=True) * alpha
    else:
        if alpha == 0:
            scores = torch.zeros(q.shape[0], blocks, blocks, q.shape[2])
        else:
            scores = selector_scores(q, desc, scale, method, block_size, tiles=rows)
        keep = (scores > 0) & (scores >= alpha * scores.amax(dim=2, keepdim=True))
    protected, causal = _protected(blocks, blocks, sink, window, last_full)
    if method not in V1_ROUTED_METHODS and alpha == 0:
        selected = causal.expand_as(scores).clone()
    else:
        selected = (keep | protected) & causal
    row_mask = torch.zeros(blocks, dtype=torch.bool)
    row_mask[rows] = True
    selected &= row_mask.view(1, blocks, 1, 1)
    return selected, scores, desc


def prefill_attention_tiles(method, q, k, v, scale, alpha, sink=2, window=4, last_full=2,
                            block_size=BLOCK_SIZE, tiles=None, routing=None):
    """``attention.py:210-333`` for the query tiles in ``tiles``.

    Returns (outputs, selected, scores): outputs maps t -> (O bf16, LSE fp32).
    Mean methods merge the exact path (stored bf16, ``kernels.py:322``) with the
    block-mean tail. ``routing`` may pass a precomputed (selected, scores, desc).
    """
    if method not in METHODS:
        raise ValueError(f"unsupported method {method!r}")
    selected, scores, desc = routing or route(method, q, k, v, scale, alpha, sink, window, last_full,
                                              block_size, tiles)
    exact = exact_attention_tiles(q, k, v, selected, scale, block_size, tiles)
    outputs = {}
    for t, (o_e, l_e) in exact.items():
        o_e = o_e.to(q.dtype)
        lo, hi = _tile_rows(t, q.shape[1], block_size)
        if method in MEAN_METHODS:
            o_m, l_m = _mean_tile(q[:, lo:hi], desc, selected[:, t], t, scale)
            outputs[t] = merge_exact_mean(o_e, l_e, o_m, l_m)
        elif method in RESCUE_METHODS:  # attention.py:306-331
            o_r, l_r = _rescue_tile(q[:, lo:hi], k, v, selected[:, t], t, scale, block_size,
                                    method == "fp_v1_rescue_v2")
            outputs[t] = merge_exact_mean(o_e, l_e, o_r, l_r)
        else:
            outputs[t] = (o_e, l_e)
    return outputs, selected, scores
