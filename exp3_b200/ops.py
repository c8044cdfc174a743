"""The fused prefill attention op (route -> exact -> mean + merge) on libfpx.

``prefill_attention`` is the call the drop-in ``AttentionBackend`` makes per layer; it
is also registered as the PyTorch custom op ``fpx::prefill_attention``. Its device
workspace (routing lists, descriptors, LSE) is cached per device and reused across
calls on the same stream.
"""

from __future__ import annotations

import torch

from ._capi import (METHOD_IDS, STAGE_ALL, FpxError, call, lib, ptr, require_cuda, stream as cur_stream,
                    strides3)

BLOCK_SIZE = 128
_workspaces: dict[int, torch.Tensor] = {}


def workspace_bytes(method: str, batch, length, heads, kv_heads, head_dim=128, block_size=BLOCK_SIZE) -> int:
    return int(lib().fpx_prefill_workspace_bytes(METHOD_IDS[method], batch, length, heads, kv_heads, head_dim,
                                                 block_size))


def workspace(device: torch.device, nbytes: int) -> torch.Tensor:
    """A cached uint8 device buffer of at least ``nbytes`` (256-byte aligned)."""
    idx = device.index if device.index is not None else torch.cuda.current_device()
    buf = _workspaces.get(idx)
    if buf is None or buf.numel() < nbytes:
        buf = torch.empty(max(nbytes, 1 << 20), dtype=torch.uint8, device=torch.device("cuda", idx))
        _workspaces[idx] = buf
    return buf


def release_workspaces():
    _workspaces.clear()


@torch.no_grad()
def prefill_attention(q, k, v, method: str, alpha: float, scale: float, sink: int = 2, window: int = 4,
                      last_full: int = 2, block_size: int = BLOCK_SIZE, out=None, lse=None,
                      kv_range=None, tile_range=None, stages: int = STAGE_ALL, ws=None):
    """The prefill branch of ``AttentionBackend.forward`` (``attention.py:210-333``).

    q [B, L, H, d], k / v [B, L, Hkv, d] bf16 with the last dim contiguous (any other
    strides, so HF's [B, H, L, d] tensors can be passed as ``x.transpose(1, 2)``).
    Returns the bf16 output [B, L, H, d] (``out`` if given; it may be a strided view).
    ``kv_range`` / ``tile_range`` restrict the work to KV heads / query tiles (the
    work units of a sharded layer).
    """
    if method not in METHOD_IDS:
        raise ValueError(f"unknown method {method!r}")
    dev = require_cuda(q, k, v)
    for t in (q, k, v):
        if t.dtype != torch.bfloat16:
            raise TypeError("q, k, v must be bfloat16")
    batch, length, heads, head_dim = q.shape
    kv_heads = k.shape[2]
    blocks = (length + block_size - 1) // block_size
    kv0, kv1 = kv_range or (0, kv_heads)
    t0, t1 = tile_range or (0, blocks)
    if out is None:
        out = torch.empty(batch, length, heads, head_dim, dtype=q.dtype, device=dev)
    if ws is None:
        ws = workspace(dev, workspace_bytes(method, batch, length, heads, kv_heads, head_dim, block_size))
    call("fpx_prefill_attention", METHOD_IDS[method], float(alpha), sink, window, last_full,
         ptr(q), *strides3(q), ptr(k), *strides3(k), ptr(v), *strides3(v),
         batch, length, heads, kv_heads, head_dim, block_size, float(scale), kv0, kv1, t0, t1,
         ptr(out), *strides3(out), ptr(lse), ptr(ws), ws.numel(), stages, cur_stream(dev))
    return out


@torch.no_grad()
def export_routing(method: str, batch, length, heads, kv_heads, ws: torch.Tensor | None = None,
                   head_dim: int = 128, block_size: int = BLOCK_SIZE, device=None):
    """The last routing on ``ws`` in the reference's layouts: (bool mask, int64 indices, int32 counts)."""
    device = device or torch.device("cuda", torch.cuda.current_device())
    if ws is None:
        ws = workspace(device, workspace_bytes(method, batch, length, heads, kv_heads, head_dim, block_size))
    blocks = (length + block_size - 1) // block_size
    selected = torch.empty(batch, blocks, blocks, heads, dtype=torch.bool, device=device)
    indices = torch.empty(batch, blocks, blocks, heads, dtype=torch.int64, device=device)
    counts = torch.empty(batch, blocks, heads, dtype=torch.int32, device=device)
    call("fpx_prefill_export_routing", METHOD_IDS[method], batch, length, heads, kv_heads, head_dim, block_size,
         ptr(ws), ws.numel(), ptr(selected), ptr(indices), ptr(counts), cur_stream(device))
    return selected, indices, counts


@torch.library.custom_op("fpx::prefill_attention", mutates_args=())
def prefill_attention_op(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, method: str, alpha: float,
                         scale: float, sink: int, window: int, last_full: int) -> torch.Tensor:
    return prefill_attention(q, k, v, method, alpha, scale, sink, window, last_full)


@prefill_attention_op.register_fake
def _(q, k, v, method, alpha, scale, sink, window, last_full):
    return q.new_empty(q.shape)


__all__ = ["prefill_attention", "prefill_attention_op", "export_routing", "workspace", "workspace_bytes",
           "release_workspaces", "FpxError"]
