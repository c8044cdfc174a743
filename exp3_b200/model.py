"""Qwen2.5-7B-shaped full-model prefill and greedy decode on libfpx, one GPU or tensor-parallel.

The model exp3 times is HF ``Qwen2ForCausalLM`` driven by ``evaluate.prefill``
(``evaluate.py:323-345``: one forward with ``logits_to_keep=1`` then argmax) and
``evaluate.generate`` (``evaluate.py:357-405``: dense greedy decode on the KV cache), with
the sparse prefill attention plugged in (``attention.py:57``). This module runs the same
computation without the HF module graph:

- the projections are plain cuBLAS GEMMs (through torch);
- residual add + RMSNorm, RoPE and SwiGLU are libfpx kernels that keep HF's bf16 rounding
  points;
- attention is the fused libfpx prefill op on zero-copy views of the QKV output, and libfpx's
  split-K decode kernel on the KV cache.

Weights are random (seeded, normal(0, 0.02) like HF's initializer) because no checkpoint is
available.

Tensor parallelism (``tp_size`` > 1, one process per GPU, NCCL):
- ranks own whole KV groups, or for ``tp_size`` > Hkv an equal split of one group's query
  heads (Qwen2.5-7B on 8 GPUs: each KV head on two ranks with 4 + 3 query heads);
- QKV and gate/up are column-sharded, o_proj and down_proj row-sharded;
- o_proj and down_proj are each followed by an all-reduce.

The tensor-parallel prefill overlaps those all-reduces with compute. Routing and attention
of a query tile read only that tile's rows and the K/V rows before it, and every other op is
row-wise, so each layer runs as ``prefill_chunks`` row chunks (whole 128-row tiles): chunk c
goes through RMSNorm, QKV, RoPE, attention on its tile range and o_proj, and its o_proj
all-reduce is issued asynchronously while chunk c + 1 computes; the MLP of chunk c runs after
that, and its down all-reduce overlaps the following chunks (and the next layer's first ones).
Only the last chunk's o_proj all-reduce of each layer is left exposed.

The embedding and LM head are replicated; only the last token's logits are computed.
"""

from __future__ import annotations

import math
from dataclasses import dataclass

import torch

from . import decode as _decode
from . import ops
from ._capi import FpxError, call, lib, ptr, stream, strides3


@dataclass
class _GraphStep:
    """Device state of a captured decode step: the new token's position (int32 for the kernels,
    int64 for the cache write), the key count after it, the input token and the decode workspace."""
    pos32: torch.Tensor
    pos64: torch.Tensor
    keys32: torch.Tensor
    token: torch.Tensor
    ws: torch.Tensor


@dataclass(frozen=True)
class Qwen2Config:
    vocab_size: int = 152064
    hidden_size: int = 3584
    intermediate_size: int = 18944
    num_hidden_layers: int = 28
    num_attention_heads: int = 28
    num_key_value_heads: int = 4
    head_dim: int = 128
    rope_theta: float = 1e6
    rms_norm_eps: float = 1e-6
    initializer_range: float = 0.02


QWEN25_7B = Qwen2Config()


def head_partition(cfg: Qwen2Config, rank: int, world: int):
    """(kv heads, query heads) owned by ``rank``: whole KV groups, or a split of one group."""
    hkv, heads = cfg.num_key_value_heads, cfg.num_attention_heads
    group = heads // hkv
    if world <= hkv:
        if hkv % world:
            raise ValueError(f"{hkv} KV heads do not split over {world} ranks")
        per = hkv // world
        kv = list(range(rank * per, (rank + 1) * per))
        return kv, [h for k in kv for h in range(k * group, (k + 1) * group)]
    if world % hkv:
        raise ValueError(f"{world} ranks do not split {hkv} KV heads evenly")
    parts = world // hkv
    kv = rank // parts
    j = rank % parts
    size = [group // parts + (1 if i < group % parts else 0) for i in range(parts)]
    start = kv * group + sum(size[:j])
    return [kv], list(range(start, start + size[j]))


def ffn_partition(cfg: Qwen2Config, rank: int, world: int):
    per = cfg.intermediate_size // world
    if cfg.intermediate_size % world:
        raise ValueError("intermediate size does not split evenly")
    return rank * per, (rank + 1) * per


class _Init:
    """Seeded normal(0, std) tensors, identical on every rank (each generates, then slices)."""

    def __init__(self, seed: int, device):
        self.gen = torch.Generator(device=device)
        self.gen.manual_seed(seed)
        self.device = device

    def normal(self, shape, std):
        return (torch.randn(shape, generator=self.gen, device=self.device, dtype=torch.float32) * std).to(
            torch.bfloat16)


class LayerWeights:
    def __init__(self, cfg: Qwen2Config, layer: int, seed: int, device, kv, qh, ffn):
        d, hid = cfg.head_dim, cfg.hidden_size
        init = _Init(seed * 1000 + layer, device)
        std = cfg.initializer_range
        wq = init.normal((cfg.num_attention_heads * d, hid), std)
        wk = init.normal((cfg.num_key_value_heads * d, hid), std)
        wv = init.normal((cfg.num_key_value_heads * d, hid), std)
        bq = init.normal((cfg.num_attention_heads * d,), std)
        bk = init.normal((cfg.num_key_value_heads * d,), std)
        bv = init.normal((cfg.num_key_value_heads * d,), std)
        wo = init.normal((hid, cfg.num_attention_heads * d), std)
        wg = init.normal((cfg.intermediate_size, hid), std)
        wu = init.normal((cfg.intermediate_size, hid), std)
        wd = init.normal((hid, cfg.intermediate_size), std)
        rows = lambda heads: torch.cat([torch.arange(h * d, (h + 1) * d, device=device) for h in heads])
        qr, kr = rows(qh), rows(kv)
        self.w_qkv = torch.cat([wq[qr], wk[kr], wv[kr]]).contiguous()
        self.b_qkv = torch.cat([bq[qr], bk[kr], bv[kr]]).contiguous()
        self.w_o = wo[:, qr].contiguous()
        f0, f1 = ffn
        self.w_gu = torch.cat([wg[f0:f1], wu[f0:f1]]).contiguous()
        self.w_down = wd[:, f0:f1].contiguous()
        self.ln1 = torch.ones(hid, dtype=torch.bfloat16, device=device)
        self.ln2 = torch.ones(hid, dtype=torch.bfloat16, device=device)
        # full tensors kept only for tests that rebuild an HF model from the same weights
        self.full = dict(wq=wq, wk=wk, wv=wv, bq=bq, bk=bk, bv=bv, wo=wo, wg=wg, wu=wu, wd=wd)


@dataclass
class AttentionSettings:
    method: str = "mean_native"
    alpha: float = 0.08
    sink: int = 2
    window: int = 4
    last_full: int = 2


class Qwen2Model:
    def __init__(self, cfg: Qwen2Config = QWEN25_7B, device=None, seed: int = 0, tp_rank: int = 0,
                 tp_size: int = 1, group=None, attention: AttentionSettings | None = None, keep_full=False):
        self.cfg = cfg
        self.device = torch.device(device or "cuda")
        self.tp_rank, self.tp_size, self.group = tp_rank, tp_size, group
        self.attn = attention or AttentionSettings()
        self.kv, self.qh = head_partition(cfg, tp_rank, tp_size)
        self.ffn = ffn_partition(cfg, tp_rank, tp_size)
        init = _Init(seed, self.device)
        self.embed = init.normal((cfg.vocab_size, cfg.hidden_size), cfg.initializer_range)
        self.layers = []
        for i in range(cfg.num_hidden_layers):
            lw = LayerWeights(cfg, i, seed, self.device, self.kv, self.qh, self.ffn)
            if not keep_full:
                lw.full = None
            self.layers.append(lw)
        self.norm = torch.ones(cfg.hidden_size, dtype=torch.bfloat16, device=self.device)
        lm_head = _Init(seed + 7, self.device).normal((cfg.vocab_size, cfg.hidden_size), cfg.initializer_range)
        # Vocab-sharded LM head under tensor parallelism: each rank holds vocab / N rows and the
        # last token's logits are all-gathered (the head is 1.09 GB: replicated, it would be
        # read in full by every rank at every decode step).
        if tp_size > 1 and cfg.vocab_size % tp_size == 0:
            rows = cfg.vocab_size // tp_size
            self.lm_head = lm_head[tp_rank * rows:(tp_rank + 1) * rows].contiguous()
            self.vocab_sharded = True
        else:
            self.lm_head = lm_head
            self.vocab_sharded = False
        del lm_head
        self.scale = cfg.head_dim ** -0.5
        self.k_cache = self.v_cache = None
        self.length = 0
        self.peer_all_reduce = True
        self._peer_ar = None
        # Row chunks of the tensor-parallel prefill pipeline (1 = one pass per layer, no overlap).
        self.prefill_chunks = 4 if tp_size > 1 else 1
        self.replay_events = None  # (start, end, replays) of the last decode_graph

    # ---------------------------------------------------------------- pieces
    def _rmsnorm(self, x, weight, residual=None):
        rows, hid = x.shape
        out = torch.empty_like(x)
        call("fpx_rmsnorm", ptr(x), ptr(residual), ptr(weight), self.cfg.rms_norm_eps, rows, hid, ptr(out),
             ptr(residual), stream(self.device))
        return out

    def _rope(self, t, pos0):
        if isinstance(pos0, torch.Tensor):  # device position (captured decode step)
            call("fpx_rope_neox_at", ptr(t), *strides3(t), t.shape[0], t.shape[1], t.shape[2], t.shape[3],
                 ptr(pos0), self.cfg.rope_theta, stream(self.device))
        else:
            call("fpx_rope_neox", ptr(t), *strides3(t), t.shape[0], t.shape[1], t.shape[2], t.shape[3], pos0,
                 self.cfg.rope_theta, stream(self.device))

    def _silu_mul(self, gu):
        rows, two_i = gu.shape
        out = torch.empty(rows, two_i // 2, dtype=gu.dtype, device=gu.device)
        call("fpx_silu_mul", ptr(gu), rows, two_i // 2, ptr(out), stream(self.device))
        return out

    def _all_reduce(self, t):
        if self.tp_size > 1:
            if self._peer_ar is not None and self._peer_ar.fits(t):  # decode: one-shot over peer memory
                self._peer_ar.all_reduce_(t)
            else:
                torch.distributed.all_reduce(t, group=self.group)
        return t

    def _decode_comm(self):
        """The decode step's small all-reduces go over NVLink peer memory (exp3_b200.comm) when
        ``peer_all_reduce`` is set and the model is tensor parallel."""
        if self.tp_size > 1 and self.peer_all_reduce and self._peer_ar is None:
            from .comm import PeerAllReduce
            self._peer_ar = PeerAllReduce(self.group, self.device, max_elems=8 * self.cfg.hidden_size)

    def _alloc_cache(self, capacity):
        shape = (self.cfg.num_hidden_layers, 1, capacity, len(self.kv), self.cfg.head_dim)
        self.k_cache = torch.empty(shape, dtype=torch.bfloat16, device=self.device)
        self.v_cache = torch.empty(shape, dtype=torch.bfloat16, device=self.device)

    def _layer(self, i, h, x, pos0, length, decoding, step=None):
        """One decoder layer: x = normed input rows; returns (h, partial down output). ``step``
        (a _GraphStep) replaces the host position by device tensors, for captured decode steps."""
        cfg, lw = self.cfg, self.layers[i]
        d = cfg.head_dim
        hq, hkv = len(self.qh), len(self.kv)
        qkv = torch.addmm(lw.b_qkv, x, lw.w_qkv.t())
        q = qkv[:, : hq * d].view(1, length, hq, d)
        k = qkv[:, hq * d:(hq + hkv) * d].view(1, length, hkv, d)
        v = qkv[:, (hq + hkv) * d:].view(1, length, hkv, d)
        if step is not None:
            self._rope(q, step.pos32)
            self._rope(k, step.pos32)
            self.k_cache[i, 0].index_copy_(0, step.pos64, k[0])
            self.v_cache[i, 0].index_copy_(0, step.pos64, v[0])
            attn = torch.empty_like(q)
            call("fpx_decode_attention_at", ptr(q), *strides3(q), ptr(self.k_cache[i]), *strides3(self.k_cache[i]),
                 ptr(self.v_cache[i]), *strides3(self.v_cache[i]), 1, length, self.k_cache.shape[2],
                 ptr(step.keys32), hq, hkv, d, float(self.scale), ptr(attn), *strides3(attn), None,
                 ptr(step.ws), step.ws.numel(), stream(self.device))
            o = self._all_reduce(attn.view(length, hq * d) @ lw.w_o.t())
            x2 = self._rmsnorm(o, lw.ln2, residual=h)
            gu = x2 @ lw.w_gu.t()
            down = self._all_reduce(self._silu_mul(gu) @ lw.w_down.t())
            return h, down
        self._rope(q, pos0)
        self._rope(k, pos0)
        self.k_cache[i, :, pos0:pos0 + length] = k
        self.v_cache[i, :, pos0:pos0 + length] = v
        if decoding:
            kc, vc = self.k_cache[i, :, :pos0 + length], self.v_cache[i, :, :pos0 + length]
            attn = _decode.decode_attention(q, kc, vc, self.scale)
        else:
            a = self.attn
            attn = ops.prefill_attention(q, k, v, a.method, a.alpha, self.scale, a.sink, a.window, a.last_full)
        o = self._all_reduce(attn.view(length, hq * d) @ lw.w_o.t())
        x2 = self._rmsnorm(o, lw.ln2, residual=h)  # h += o
        gu = x2 @ lw.w_gu.t()
        down = self._all_reduce(self._silu_mul(gu) @ lw.w_down.t())
        return h, down

    def _forward(self, ids, pos0, decoding, step=None):
        length = ids.shape[0]
        h = torch.nn.functional.embedding(ids, self.embed)
        x = self._rmsnorm(h, self.layers[0].ln1)
        down = None
        for i in range(self.cfg.num_hidden_layers):
            if i > 0:
                x = self._rmsnorm(down, self.layers[i].ln1, residual=h)  # h += down
            h, down = self._layer(i, h, x, pos0, length, decoding, step)
        last = self._rmsnorm(down[-1:].contiguous(), self.norm, residual=h[-1:].contiguous())
        logits = (last @ self.lm_head.t()).float()  # bf16 LM head, as HF's lm_head
        if self.vocab_sharded:
            full = torch.empty(self.tp_size * logits.shape[-1], dtype=logits.dtype, device=logits.device)
            torch.distributed.all_gather_into_tensor(full, logits.view(-1), group=self.group)
            return full
        return logits[-1]

    def _chunk_bounds(self, length: int):
        """Row ranges [r0, r1) of the prefill pipeline: ``prefill_chunks`` runs of whole tiles."""
        tiles = (length + 127) // 128
        n = max(1, min(self.prefill_chunks, tiles))
        cuts = [round(tiles * c / n) for c in range(n + 1)]
        return [(128 * a, min(length, 128 * b)) for a, b in zip(cuts, cuts[1:]) if b > a]

    def _forward_pipelined(self, ids):
        """The tensor-parallel prefill as a row-chunk pipeline (see the module docstring): the
        same computation as ``_forward(ids, 0, decoding=False)``, with each chunk's all-reduces
        issued asynchronously and waited for only by the compute that reads them."""
        cfg = self.cfg
        d, hid = cfg.head_dim, cfg.hidden_size
        hq, hkv = len(self.qh), len(self.kv)
        length = ids.shape[0]
        bounds = self._chunk_bounds(length)
        dev = self.device
        h = torch.nn.functional.embedding(ids, self.embed)
        x = torch.empty_like(h)
        o = torch.empty_like(h)
        down = torch.empty_like(h)
        qkv = torch.empty(length, (hq + 2 * hkv) * d, dtype=torch.bfloat16, device=dev)
        attn = torch.empty(length, hq * d, dtype=torch.bfloat16, device=dev)
        q = qkv[:, : hq * d].view(1, length, hq, d)
        k = qkv[:, hq * d:(hq + hkv) * d].view(1, length, hkv, d)
        v = qkv[:, (hq + hkv) * d:].view(1, length, hkv, d)
        a = self.attn
        pending_down = [None] * len(bounds)  # down all-reduce of chunk c, previous layer
        work_o = [None] * len(bounds)

        def attention_part(i, c):
            lw = self.layers[i]
            r0, r1 = bounds[c]
            if pending_down[c] is not None:
                pending_down[c].wait()
                pending_down[c] = None
            if i == 0:
                x[r0:r1] = self._rmsnorm(h[r0:r1], lw.ln1)
            else:
                x[r0:r1] = self._rmsnorm(down[r0:r1], lw.ln1, residual=h[r0:r1])  # h += down
            torch.addmm(lw.b_qkv, x[r0:r1], lw.w_qkv.t(), out=qkv[r0:r1])
            self._rope(q[:, r0:r1], r0)
            self._rope(k[:, r0:r1], r0)
            self.k_cache[i, :, r0:r1] = k[:, r0:r1]
            self.v_cache[i, :, r0:r1] = v[:, r0:r1]
            ops.prefill_attention(q, k, v, a.method, a.alpha, self.scale, a.sink, a.window, a.last_full,
                                  out=attn.view(1, length, hq, d), tile_range=(r0 // 128, (r1 + 127) // 128))
            torch.mm(attn[r0:r1], lw.w_o.t(), out=o[r0:r1])
            work_o[c] = torch.distributed.all_reduce(o[r0:r1], group=self.group, async_op=True)

        def mlp_part(i, c):
            lw = self.layers[i]
            r0, r1 = bounds[c]
            work_o[c].wait()
            work_o[c] = None
            x2 = self._rmsnorm(o[r0:r1], lw.ln2, residual=h[r0:r1])  # h += o
            torch.mm(self._silu_mul(x2 @ lw.w_gu.t()), lw.w_down.t(), out=down[r0:r1])
            pending_down[c] = torch.distributed.all_reduce(down[r0:r1], group=self.group, async_op=True)

        for i in range(cfg.num_hidden_layers):
            for c in range(len(bounds)):
                attention_part(i, c)
                if c > 0:
                    mlp_part(i, c - 1)
            mlp_part(i, len(bounds) - 1)
        for c, work in enumerate(pending_down):
            if work is not None:
                work.wait()
        last = self._rmsnorm(down[-1:].contiguous(), self.norm, residual=h[-1:].contiguous())
        logits = (last @ self.lm_head.t()).float()
        if self.vocab_sharded:
            full = torch.empty(self.tp_size * logits.shape[-1], dtype=logits.dtype, device=logits.device)
            torch.distributed.all_gather_into_tensor(full, logits.view(-1), group=self.group)
            return full
        return logits[-1]

    # ---------------------------------------------------------------- public
    @torch.inference_mode()
    def prefill_logits(self, input_ids: torch.Tensor, max_new_tokens: int = 0):
        """One forward over the prompt (filling the KV cache); returns the last token's fp32
        logits over the whole vocabulary, on the device."""
        if input_ids.dim() != 1:
            raise ValueError("input_ids must be 1-D (batch 1, as exp3)")
        length = input_ids.shape[0]
        if self.k_cache is None or self.k_cache.shape[2] < length + max_new_tokens:
            self._alloc_cache(length + max_new_tokens)
        if self.tp_size > 1 and self.prefill_chunks > 1:
            logits = self._forward_pipelined(input_ids)
        else:
            logits = self._forward(input_ids, 0, decoding=False)
        self.length = length
        return logits

    @torch.inference_mode()
    def prefill(self, input_ids: torch.Tensor, max_new_tokens: int = 0):
        """``evaluate.prefill``: one forward over the prompt; returns the first generated token (device)."""
        return self.prefill_logits(input_ids, max_new_tokens).argmax()

    @torch.inference_mode()
    def decode_step(self, token: torch.Tensor):
        """One dense greedy decode step (``evaluate.py:384-400``); returns the next token (device)."""
        self._decode_comm()
        logits = self._forward(token.view(1), self.length, decoding=True)
        self.length += 1
        return logits.argmax()

    @torch.inference_mode()
    def decode_graph(self, first_token: torch.Tensor, steps: int):
        """``steps`` greedy decode tokens after ``prefill`` (the first is ``first_token``), the
        same computation as ``decode_step`` but each step one replay of a CUDA graph: the step's
        position and key count live in device memory and advance inside the graph, and the next
        token is written back into the graph's input, so no step waits for the host. Returns the
        [steps] int64 tokens on the device."""
        cap = self.k_cache.shape[2]
        if self.length + steps - 1 > cap:
            raise ValueError("KV cache too small: prefill with max_new_tokens >= steps")
        dev = self.device
        out = torch.empty(steps, dtype=torch.int64, device=dev)
        out[0] = first_token.view(())
        if steps == 1:
            return out
        cfg = self.cfg
        self._decode_comm()
        need = int(lib().fpx_decode_workspace_bytes(1, 1, len(self.qh), len(self.kv), cap, cfg.head_dim))
        step = _GraphStep(
            pos32=torch.tensor([self.length], dtype=torch.int32, device=dev),
            pos64=torch.tensor([self.length], dtype=torch.int64, device=dev),
            keys32=torch.tensor([self.length + 1], dtype=torch.int32, device=dev),
            token=first_token.view(1).clone(),
            ws=torch.empty(max(need, 256), dtype=torch.uint8, device=dev))

        def one_step():
            logits = self._forward(step.token, None, decoding=True, step=step)
            step.token.copy_(logits.argmax().view(1))
            step.pos32.add_(1)
            step.pos64.add_(1)
            step.keys32.add_(1)

        side = torch.cuda.Stream(device=dev)  # the eager first step warms the allocator up
        side.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(side):
            one_step()
        torch.cuda.current_stream(dev).wait_stream(side)
        out[1] = step.token[0]
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            one_step()
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record()
        for i in range(2, steps):
            graph.replay()
            out[i] = step.token[0]
        end.record()
        self.replay_events = (start, end, steps - 2)
        del graph  # a graph holding NCCL calls must go before the process group
        self.length += steps - 1
        return out

    @torch.inference_mode()
    def generate(self, input_ids: torch.Tensor, max_new_tokens: int):
        token = self.prefill(input_ids, max_new_tokens)
        out = [token]
        for _ in range(max_new_tokens - 1):
            token = self.decode_step(token)
            out.append(token)
        return torch.stack(out)

    def close_comm(self):
        """Unmaps the peer all-reduce buffers (every rank calls it; no kernel of theirs may be
        in flight, hence the synchronize and barrier first)."""
        if self._peer_ar is not None:
            torch.cuda.synchronize(self.device)
            torch.distributed.barrier(group=self.group)
            self._peer_ar.close()
            self._peer_ar = None

    def replay_ms_per_token(self) -> float | None:
        """Device time per step of the last ``decode_graph``'s replays (after its eager warm-up
        step and the capture), or None."""
        if not self.replay_events or self.replay_events[2] <= 0:
            return None
        start, end, n = self.replay_events
        end.synchronize()
        return start.elapsed_time(end) / n

    def prefill_flops(self, length: int, exact_pairs: int | None = None) -> float:
        """Algorithmic FLOPs of one prefill: 2 x params x L for the linear layers (last-token LM
        head) plus 4 d x exact pairs per layer (all causal pairs when ``exact_pairs`` is None)."""
        cfg = self.cfg
        d, hid = cfg.head_dim, cfg.hidden_size
        per_layer = hid * (cfg.num_attention_heads + 2 * cfg.num_key_value_heads) * d + \
            cfg.num_attention_heads * d * hid + 3 * hid * cfg.intermediate_size
        linear = 2 * per_layer * cfg.num_hidden_layers * length + 2 * hid * cfg.vocab_size
        pairs = exact_pairs if exact_pairs is not None else \
            cfg.num_attention_heads * length * (length + 1) // 2
        return linear + 4 * d * pairs * cfg.num_hidden_layers


def synthetic_prompt(length: int = 32640, vocab: int = 152064, spans: int = 64, span_len: int = 16,
                     seed: int = 0) -> torch.Tensor:
    """Uniform random token ids with ``spans`` planted repeated key -> value spans of
    ``span_len`` tokens (each span appears twice, its copy later in the prompt)."""
    g = torch.Generator().manual_seed(seed)
    ids = torch.randint(0, vocab, (length,), generator=g)
    half = length // 2
    for _ in range(spans):
        src = int(torch.randint(0, half - span_len, (1,), generator=g))
        dst = int(torch.randint(half, length - span_len, (1,), generator=g))
        ids[dst:dst + span_len] = ids[src:src + span_len]
    return ids


__all__ = ["Qwen2Config", "QWEN25_7B", "Qwen2Model", "AttentionSettings", "head_partition", "ffn_partition",
           "synthetic_prompt", "FpxError", "math"]
