"""The decode entry point that allocates nothing (fpx_decode_attention_noalloc).

It is for callers that cannot allocate device memory where they decode, such as an engine
that only hands out memory from its own fixed pool. This file is named to be collected last,
so a run that stops at the first failure has already run every other test; it also passes
alone in a fresh process.
"""

import ctypes

import pytest
import torch

from exp3_b200 import _capi

pytestmark = pytest.mark.gpu
O_TOL, LSE_TOL = 2e-2, 1e-3


def _inputs(seed, batch, lq, s_len, heads, kv_heads, d=128):
    g = torch.Generator().manual_seed(seed)
    q = torch.randn(batch, lq, heads, d, generator=g).to(torch.bfloat16).cuda()
    # The cache as HF keeps it, [B, Hkv, S, d], passed as a [B, S, Hkv, d] view.
    k = torch.randn(batch, kv_heads, s_len, d, generator=g).to(torch.bfloat16).cuda().transpose(1, 2)
    v = torch.randn(batch, kv_heads, s_len, d, generator=g).to(torch.bfloat16).cuda().transpose(1, 2)
    return q, k, v


def _call(name, q, k, v, workspace=None):
    lib = _capi.lib()
    batch, lq, heads, d = q.shape
    s_len, kv_heads = k.shape[1], k.shape[2]
    out = torch.empty(batch, lq, heads, d, dtype=torch.bfloat16, device="cuda")
    lse = torch.empty(batch, lq, heads, dtype=torch.float32, device="cuda")
    args = [_capi.ptr(q), *_capi.strides3(q), _capi.ptr(k), *_capi.strides3(k), _capi.ptr(v), *_capi.strides3(v),
            batch, lq, s_len, heads, kv_heads, d, d ** -0.5, _capi.ptr(out), *_capi.strides3(out), _capi.ptr(lse)]
    if workspace is not None:
        args += [_capi.ptr(workspace), workspace.numel()]
    rc = getattr(lib, name)(*args, _capi.stream(q.device))
    return rc, out, lse


def test_noalloc_decode_matches_workspace_decode_on_two_calls_in_a_row():
    lib = _capi.lib()
    # Two different problems back to back: the second reuses the scratch the first left behind.
    for seed, shape in ((1, (1, 1, 32768, 28, 4)), (2, (2, 3, 1000, 40, 8))):
        q, k, v = _inputs(seed, *shape)
        need = lib.fpx_decode_workspace_bytes(shape[0], shape[1], shape[3], shape[4], shape[2], 128)
        ws = torch.empty(need, dtype=torch.uint8, device="cuda")
        rc_ref, ref, ref_lse = _call("fpx_decode_attention", q, k, v, ws)
        rc, out, lse = _call("fpx_decode_attention_noalloc", q, k, v)
        torch.cuda.synchronize()
        assert rc_ref == 0 and rc == 0
        torch.testing.assert_close(out.float(), ref.float(), atol=O_TOL, rtol=0)
        torch.testing.assert_close(lse, ref_lse, atol=LSE_TOL, rtol=0)


def test_noalloc_decode_at_head_dim_256_matches_workspace_decode():
    # The Qwen3.5 shape (16 query heads over 4 KV heads, d = 256): twice the partials per row
    # and another kernel instance. Two calls in a row, the second on a longer cache.
    lib = _capi.lib()
    for seed, s_len in ((4, 4096), (5, 6000)):
        q, k, v = _inputs(seed, 1, 1, s_len, 16, 4, d=256)
        need = lib.fpx_decode_workspace_bytes(1, 1, 16, 4, s_len, 256)
        assert 0 < need <= 2 << 20
        ws = torch.empty(need, dtype=torch.uint8, device="cuda")
        rc_ref, ref, ref_lse = _call("fpx_decode_attention", q, k, v, ws)
        rc, out, lse = _call("fpx_decode_attention_noalloc", q, k, v)
        torch.cuda.synchronize()
        assert rc_ref == 0 and rc == 0
        torch.testing.assert_close(out.float(), ref.float(), atol=O_TOL, rtol=0)
        torch.testing.assert_close(lse, ref_lse, atol=LSE_TOL, rtol=0)
        # and against a plain fp32 softmax over the whole cache
        qf = q[0, 0].float().view(4, 4, 256)                       # [Hkv, G, d]
        kf, vf = k[0].float().transpose(0, 1), v[0].float().transpose(0, 1)  # [Hkv, S, d]
        logits = torch.einsum("hgd,hsd->hgs", qf, kf) * 256 ** -0.5
        dense = torch.einsum("hgs,hsd->hgd", logits.softmax(-1), vf).reshape(16, 256)
        torch.testing.assert_close(out[0, 0].float(), dense, atol=O_TOL, rtol=0)
        torch.testing.assert_close(lse[0, 0], logits.logsumexp(-1).reshape(16), atol=LSE_TOL, rtol=0)


def test_noalloc_decode_refuses_problems_beyond_its_scratch():
    lib = _capi.lib()
    # 512 query rows x 28 heads of split partials need far more than the fixed array holds.
    q, k, v = _inputs(3, 1, 512, 4096, 28, 4)
    need = lib.fpx_decode_workspace_bytes(1, 512, 28, 4, 4096, 128)
    limit = 2 << 20  # FPX_DECODE_NOALLOC_SCRATCH_BYTES
    assert need > limit
    rc, _, _ = _call("fpx_decode_attention_noalloc", q, k, v)
    assert rc == -5  # FPX_ERR_WORKSPACE
    assert lib.fpx_status_string(rc) == b"workspace too small or misaligned"
    _ = ctypes
