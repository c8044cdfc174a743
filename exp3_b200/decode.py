"""Dense decode attention (the reference's q_len != k_len branch, attention.py:178-189) on libfpx."""

from __future__ import annotations

import torch

from ._capi import call, lib, ptr, require_cuda, stream, strides3

_workspaces: dict[int, torch.Tensor] = {}


@torch.library.custom_op("fpx::decode_attention", mutates_args=())
def _decode_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, scale: float) -> torch.Tensor:
    return _decode(q, k, v, scale, None, None)


@_decode_attention.register_fake
def _(q, k, v, scale):
    return q.new_empty(q.shape)


@torch.no_grad()
def decode_attention(q, k, v, scale: float, out=None, lse=None):
    """q [B, Lq, H, d]; k / v [B, S, Hkv, d] (views of HF's [B, Hkv, S, d] cache work).

    Non-causal: every query row sees all S keys, as SDPA(is_causal=False) does in the
    reference's decode call. Returns bf16 [B, Lq, H, d] (``out`` if given). Without ``out``
    and ``lse`` it runs as the custom op ``torch.ops.fpx.decode_attention``.
    """
    if out is None and lse is None:
        return torch.ops.fpx.decode_attention(q, k, v, float(scale))
    return _decode(q, k, v, scale, out, lse)


def _decode(q, k, v, scale, out, lse):
    dev = require_cuda(q, k, v)
    batch, lq, heads, head_dim = q.shape
    s_len, kv_heads = k.shape[1], k.shape[2]
    if out is None:
        out = torch.empty(batch, lq, heads, head_dim, dtype=q.dtype, device=dev)
    need = int(lib().fpx_decode_workspace_bytes(batch, lq, heads, kv_heads, s_len, head_dim))
    idx = dev.index if dev.index is not None else torch.cuda.current_device()
    ws = _workspaces.get(idx)
    if ws is None or ws.numel() < need:
        ws = torch.empty(max(need, 1 << 20), dtype=torch.uint8, device=dev)
        _workspaces[idx] = ws
    call("fpx_decode_attention", ptr(q), *strides3(q), ptr(k), *strides3(k), ptr(v), *strides3(v),
         batch, lq, s_len, heads, kv_heads, head_dim, float(scale), ptr(out), *strides3(out), ptr(lse),
         ptr(ws), ws.numel(), stream(dev))
    return out
