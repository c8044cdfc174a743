"""Drop-in ``AttentionBackend`` (exp3 ``attention.py:37-369``) on libfpx.

Same constructor, ``configure``, ``forward``, profile and capture hooks as the
reference; construction registers ``forward`` as transformers'
``ALL_ATTENTION_FUNCTIONS["sdpa"]`` exactly as ``attention.py:57`` does. Prefill
runs the fused CUDA path (route -> exact -> mean + merge) of ``ops.prefill_attention``
on views of HF's [B, H, L, d] tensors (no transpose copies); decode (q_len != k_len)
runs libfpx's dense decode kernel. There is no Triton, no backend dispatch and no
CPU fallback.

Profile rows keep the reference's stage schema (``attention.py:352-369``); the
routing kernels fuse the "descriptor", "selector" and "indices" stages, so their
time is reported under "selector", and "merge" is fused into "mean".
"""

from __future__ import annotations

import torch

from . import decode as _decode
from . import kernels, ops, upstream
from ._capi import STAGE_EXACT, STAGE_MEAN, STAGE_ROUTE

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
RESCUE_METHODS = {"fp_v1_rescue", "fp_v1_rescue_v2"}
MEAN_METHODS = {"mean_native", "mean_balanced", "cgf_mean", "dispersion_mean"}


def _register(forward):
    try:
        from transformers.modeling_utils import ALL_ATTENTION_FUNCTIONS
    except ImportError:  # transformers is only needed for the HF model path
        return
    ALL_ATTENTION_FUNCTIONS["sdpa"] = forward


class AttentionBackend:
    def __init__(self, alpha: float = 0.08, sink_blocks: int = 2, window_blocks: int = 4,
                 last_full_blocks: int = 2, block_size: int = 128, selector_chunk_tiles: int = 8):
        self.method = "dense"
        self.alpha = alpha
        self.sink_blocks = sink_blocks
        self.window_blocks = window_blocks
        self.last_full_blocks = last_full_blocks
        self.block_size = block_size
        self.selector_chunk_tiles = selector_chunk_tiles
        self.record = False
        self.profile_records = []
        self.capture_callback = None
        _register(self.forward)

    def configure(self, method: str, alpha: float | None = None):
        if method not in METHODS:
            raise ValueError(f"unknown method {method!r}; choose from {METHODS}")
        self.method = method
        if alpha is not None:
            self.alpha = alpha

    def _event(self):
        ev = torch.cuda.Event(enable_timing=True)
        ev.record()
        return ev

    def _prefill(self, q, k, v, scale, record):
        method = self.method
        args = (q, k, v, method, self.alpha, scale, self.sink_blocks, self.window_blocks,
                self.last_full_blocks, self.block_size)
        if not self.record:
            return ops.prefill_attention(*args)
        out = torch.empty(q.shape, dtype=q.dtype, device=q.device)
        events = record["events"]
        e0 = self._event()
        ops.prefill_attention(*args, out=out, stages=STAGE_ROUTE)
        e1 = self._event()
        ops.prefill_attention(*args, out=out, stages=STAGE_EXACT)
        e2 = self._event()
        events["selector"] = (e0, e1)
        events["exact"] = (e1, e2)
        if method in MEAN_METHODS or method in RESCUE_METHODS:  # the rescue tail is timed as "mean"
            ops.prefill_attention(*args, out=out, stages=STAGE_MEAN)
            events["mean"] = (e2, self._event())
        batch, length, heads, _ = q.shape
        selected, _, _ = ops.export_routing(method, batch, length, heads, k.shape[2], device=q.device)
        q_tile, k_tile = upstream.attention_tile_sizes()
        record["accounting"] = kernels.selection_accounting(
            selected, length, q_tile, k_tile, method,
            upstream.score_tile_size() if method in V1_ROUTED_METHODS else None, self.block_size)
        return out

    def _capture_fp_v1(self, module, q, k, v, scale):
        """The reference's V1 capture path (``attention.py:215-251``), through the mirror ops."""
        mean_k = upstream.block_mean_k(k.contiguous(), self.block_size)
        scores = upstream.v1_scores(q, mean_k, scale, self.block_size)
        indices, counts = upstream.deal_output_score(scores, self.sink_blocks, self.window_blocks, self.alpha,
                                                     self.last_full_blocks, 0)
        selected = kernels.mask_from_indices(indices, counts)
        self.capture_callback(layer=int(module.layer_idx), q=q, k=k, v=v, mean_k=mean_k, scores=scores,
                              indices=indices, counts=counts, selected=selected, scale=scale)
        out, _ = upstream.exact_attention(q, k, v, indices, counts, scale, self.block_size)
        return out

    def forward(self, module, query, key, value, attention_mask, scaling, dropout=0.0, **kwargs):
        record = {"layer": getattr(module, "layer_idx", None), "method": self.method, "events": {},
                  "accounting": None}
        overall_start = self._event() if self.record else None
        is_prefill = query.shape[2] == key.shape[2]
        scale = float(scaling)
        q, k, v = query.transpose(1, 2), key.transpose(1, 2), value.transpose(1, 2)
        if not is_prefill:
            output = _decode.decode_attention(q, k, v, scale)
        elif self.capture_callback is not None and self.method == "fp_v1":
            output = self._capture_fp_v1(module, q, k, v, scale)
        else:
            output = self._prefill(q, k, v, scale, record)
            if self.record and self.method == "dense":
                sequence = query.shape[2]
                pairs = query.shape[0] * query.shape[1] * sequence * (sequence + 1) // 2
                record["accounting"] = {"effective_exact_token_pair_ratio": 1.0, "exact_token_pairs": pairs,
                                        "causal_token_pairs": pairs, "legacy_block_density": 1.0}
        if self.record and is_prefill:
            record["events"]["attention"] = (overall_start, self._event())
            self.profile_records.append(record)
        return output, None

    def start_profile(self):
        self.profile_records.clear()
        self.record = True

    def start_capture(self, callback):
        """Attach a synchronous V1-prefill diagnostic callback."""
        self.capture_callback = callback

    def finish_capture(self):
        self.capture_callback = None

    def finish_profile(self):
        self.record = False
        torch.cuda.synchronize()
        rows = []
        stage_names = ("descriptor", "selector", "indices", "exact", "mean", "merge", "attention")
        for record in self.profile_records:
            row = {"layer": record["layer"], "method": record["method"]}
            for name in stage_names:
                event = record["events"].get(name)
                row[f"{name}_ms"] = event[0].elapsed_time(event[1]) if event else 0.0
            for key, value in (record["accounting"] or {}).items():
                row[key] = value.item() if isinstance(value, torch.Tensor) else value
            rows.append(row)
        self.profile_records.clear()
        return rows
