"""Head dim 256 (the Qwen3.5 shape: 16 query heads over 4 KV heads, check_qwen35_math.py:93-185).

The reference's fp_v1 path at d = 256 through the C ABI: the bf16 block mean, the V1 scores and
selection against the reference's golden vectors, the tcgen05 d = 256 exact kernel in the
reference layout (all causal blocks, and a fixed mask), and the fused fp_v1 / dense prefill
against the oracle; also mean_native (descriptors, the block-mean tail and the merge) and decode
at d = 256. Bars as for d = 128: masks bit-exact outside the 1e-6 band, O 2e-2, LSE 1e-3.
"""

import pytest
import torch

import oracle
from exp3_b200 import _capi, ops, synthetic, upstream
from exp3_b200.attention import AttentionBackend
from golden_cases import load, t

pytestmark = pytest.mark.gpu
DEV = "cuda"
SCALE = 256 ** -0.5
O_TOL, LSE_TOL, BAND = 2e-2, 1e-3, 1e-6


def test_block_mean_and_scores_match_reference():
    data, q, k, v = load("qwen35_routing_l1025.npz")
    mine = upstream.block_mean_k(k.to(DEV)).cpu()
    assert torch.equal(mine.view(torch.int16), oracle.block_mean_k(k).view(torch.int16))
    torch.testing.assert_close(mine.float(), t(data["block_mean_fp32"]), atol=2e-3, rtol=2e-2)
    mk = t(data["mean_k_bf16_bits"]).view(torch.bfloat16)
    scores = upstream.v1_scores(q.to(DEV), mk.to(DEV), SCALE).cpu()
    torch.testing.assert_close(scores, t(data["scores"]), atol=1e-6, rtol=1e-5)
    idx, cnt = upstream.deal_output_score(t(data["scores"]).to(DEV).square().square(), 2, 4, 0.8, 2, 0)
    assert torch.equal(idx.cpu(), t(data["indices_pow4_a08"])) and torch.equal(cnt.cpu(), t(data["counts_pow4_a08"]))


def test_exact_attention_matches_reference():
    data, q, k, v = load("qwen35_exact_l385.npz")
    qd, kd, vd = q.to(DEV), k.to(DEV), v.to(DEV)
    rows, heads = t(data["rows"]), t(data["out_heads"])
    for tag in ("fixed", "all"):
        if tag == "fixed":
            idx, cnt = t(data["indices_fixed"]), t(data["counts_fixed"])
        else:
            idx, cnt = oracle.indices_from_mask(oracle.protected_selection(torch.zeros(1, 4, 4, 16), 0.0, 2, 4, 2))
        out, lse = upstream.exact_attention(qd, kd, vd, idx.to(DEV), cnt.to(DEV), SCALE)
        assert out.shape == (1, 385, 16, 256)
        torch.testing.assert_close(lse.cpu(), t(data[f"lse_{tag}"]), atol=LSE_TOL, rtol=0)
        torch.testing.assert_close(out.cpu().float()[:, rows][:, :, heads], t(data[f"out_{tag}_rows"]),
                                   atol=O_TOL, rtol=0)
        # every row and head against the oracle
        o_ref, l_ref = oracle.exact_attention(q.float(), k.float(), v.float(), idx, cnt, SCALE)
        torch.testing.assert_close(out.cpu().float(), o_ref, atol=O_TOL, rtol=0)
    assert _capi.device_error() == 0


def _fused_vs_oracle(method, q, k, v, alpha, tiles):
    qd, kd, vd = q.to(DEV), k.to(DEV), v.to(DEV)
    batch, length, heads, d = q.shape
    lse = torch.empty(batch, length, heads, device=DEV)
    out = ops.prefill_attention(qd, kd, vd, method, alpha, SCALE, lse=lse)
    sel, _, cnt = ops.export_routing(method, batch, length, heads, k.shape[2], head_dim=d)
    sel = sel.cpu()
    outs, ref_sel, ref_scores = oracle.prefill_attention_tiles(method, q, k, v, SCALE, alpha, tiles=tiles)
    compared = 0
    for tile in tiles:
        diff = sel[:, tile] != ref_sel[:, tile]
        if diff.any():
            s = ref_scores[:, tile]
            band = (s - s.amax(dim=1, keepdim=True) * alpha).abs() <= BAND
            assert bool((diff <= band).all()), f"{method}: mask differs outside the band on tile {tile}"
            continue
        lo, hi = 128 * tile, min(length, 128 * tile + 128)
        o_ref, l_ref = outs[tile]
        torch.testing.assert_close(out[:, lo:hi].cpu().float(), o_ref.float(), atol=O_TOL, rtol=0)
        torch.testing.assert_close(lse[:, lo:hi].cpu(), l_ref, atol=LSE_TOL, rtol=0)
        compared += 1
    assert compared >= len(tiles) // 2
    return sel


@pytest.mark.parametrize("method", ["fp_v1", "dense"])
def test_fused_prefill_head_dim_256(method):
    shape = synthetic.LayerShape(1, 2177, 16, 4, 256)  # 18 blocks, the last with one row
    q, k, v = synthetic.attention_inputs(shape, seed=41, needles=4, structured_sigma=0.5)
    blocks = oracle.num_blocks(2177)
    sel = _fused_vs_oracle(method, q, k, v, 0.08, list(range(blocks)))
    if method == "fp_v1":
        assert int(sel.sum()) < 16 * blocks * (blocks + 1) // 2  # structured inputs route blocks away


def test_fused_prefill_head_dim_256_batch_and_edges():
    for length in (1, 129, 385):
        shape = synthetic.LayerShape(2, length, 8, 2, 256)
        q, k, v = synthetic.attention_inputs(shape, seed=length, needles=1)
        _fused_vs_oracle("fp_v1", q, k, v, 0.08, list(range(oracle.num_blocks(length))))


def test_backend_fp_v1_at_head_dim_256():
    """The reference's own gate (check_qwen35_math.py:153-168): the backend at alpha 0 equals dense."""
    shape = synthetic.LayerShape(1, 257, 16, 4, 256)
    q, k, v = synthetic.attention_inputs(shape, seed=35)
    backend = AttentionBackend(alpha=0.0)
    backend.configure("fp_v1", 0.0)

    class Layer:
        layer_idx = 3

    qd, kd, vd = q.to(DEV), k.to(DEV), v.to(DEV)
    out, _ = backend.forward(Layer(), qd.transpose(1, 2).contiguous(), kd.transpose(1, 2).contiguous(),
                             vd.transpose(1, 2).contiguous(), None, SCALE)
    tiles = oracle.dense_attention(q.float(), k.float(), v.float(), SCALE)
    ref = torch.cat([tiles[i][0] for i in sorted(tiles)], dim=1)
    torch.testing.assert_close(out.cpu().float(), ref, atol=0.03, rtol=0.03)


def test_fused_mean_native_at_head_dim_256():
    """mean_native on the Qwen3.5 shape: V1 routing, the d = 256 exact kernel, the fp32
    block-mean tail (four threads per row) merged in place; structured inputs so tails exist."""
    shape = synthetic.LayerShape(1, 2177, 16, 4, 256)
    q, k, v = synthetic.attention_inputs(shape, seed=43, needles=4, structured_sigma=0.5)
    blocks = oracle.num_blocks(2177)
    sel = _fused_vs_oracle("mean_native", q, k, v, 0.08, list(range(blocks)))
    assert int(sel.sum()) < 16 * blocks * (blocks + 1) // 2  # tails exist


def test_descriptors_mean_tail_and_merge_ops_at_head_dim_256():
    from exp3_b200 import kernels
    shape = synthetic.LayerShape(1, 385, 8, 2, 256)
    q, k, v = synthetic.attention_inputs(shape, seed=44, needles=1)
    qd, kd, vd = q.to(DEV), k.to(DEV), v.to(DEV)
    desc = kernels.block_descriptors(kd, vd)
    ref = oracle.block_descriptors(k.float(), v.float())
    for name in ("mean_k", "mean_v", "var_k", "sigma_v"):
        torch.testing.assert_close(getattr(desc, name).cpu(), getattr(ref, name), atol=2e-6, rtol=1e-5)
    selected = oracle.protected_selection(torch.zeros(1, 4, 4, 8), 0.0, 2, 4, 2)
    selected[:, 3, 1, ::2] = False
    selected[:, 3, 0, 1::3] = False
    mo, ml = kernels.mean_tail(qd, desc, selected.to(DEV), SCALE)
    mo_ref, ml_ref = oracle.mean_tail(q.float(), ref, selected, SCALE)
    torch.testing.assert_close(ml.cpu(), ml_ref, atol=LSE_TOL, rtol=0)
    torch.testing.assert_close(mo.cpu(), mo_ref, atol=O_TOL, rtol=0)
    idx, cnt = oracle.indices_from_mask(selected)
    eo, el = upstream.exact_attention(qd, kd, vd, idx.to(DEV), cnt.to(DEV), SCALE)
    merged, merged_lse = kernels.merge_exact_mean(eo, el, mo, ml)
    m_ref, ml2_ref = oracle.merge_exact_mean(eo.cpu(), el.cpu(), mo_ref, ml_ref)
    torch.testing.assert_close(merged.cpu().float(), m_ref.float(), atol=O_TOL, rtol=0)
    torch.testing.assert_close(merged_lse.cpu(), ml2_ref, atol=LSE_TOL, rtol=0)


@pytest.mark.parametrize("method", ["mean_balanced", "cgf_mean", "dispersion_mean"])
def test_fused_new_selectors_at_head_dim_256(method):
    """The new selectors on the Qwen3.5 shape: fp32 selector routing (q row in registers, 256
    dimensions), the d = 256 exact kernel and the fp32 block-mean tail, against the oracle.
    (Log-normal K row norms are exercised at d = 128 on the config-5 shape; at d = 256 they push
    single outputs near 2.0, where the bar of 2e-2 is three bf16 steps.)"""
    shape = synthetic.LayerShape(1, 1409, 16, 4, 256)  # 12 blocks, the last with one row
    q, k, v = synthetic.attention_inputs(shape, seed=45, needles=2, structured_sigma=0.5)
    _fused_vs_oracle(method, q, k, v, 0.08, list(range(oracle.num_blocks(1409))))


def test_selector_scores_op_at_head_dim_256():
    from exp3_b200 import kernels
    shape = synthetic.LayerShape(1, 385, 8, 2, 256)
    q, k, v = synthetic.attention_inputs(shape, seed=46, needles=1)
    desc = kernels.block_descriptors(k.to(DEV), v.to(DEV))
    ref_desc = oracle.block_descriptors(k.float(), v.float())
    for selector in oracle.SELECTORS:
        got = kernels.selector_scores(q.to(DEV), desc, SCALE, selector).cpu()
        ref = oracle.selector_scores(q.float(), ref_desc, SCALE, selector)
        torch.testing.assert_close(got, ref, atol=2e-6, rtol=1e-5)


@pytest.mark.parametrize("method", ["fp_v1_rescue", "fp_v1_rescue_v2"])
def test_fused_rescue_methods_at_head_dim_256(method):
    """The rescue methods on the Qwen3.5 shape: V1 routing, the d = 256 exact kernel, the rescue
    choice (a thread pair per token, 128 dimensions each) and the fp32 rescue tail."""
    shape = synthetic.LayerShape(1, 1409, 16, 4, 256)
    q, k, v = synthetic.attention_inputs(shape, seed=47, needles=2, structured_sigma=0.5)
    _fused_vs_oracle(method, q, k, v, 0.08, list(range(oracle.num_blocks(1409))))


def test_rescue_tail_op_at_head_dim_256():
    from exp3_b200 import kernels
    shape = synthetic.LayerShape(1, 1153, 8, 2, 256)
    q, k, v = synthetic.attention_inputs(shape, seed=48, needles=1)
    g = torch.Generator().manual_seed(48)
    selected = oracle.protected_selection(torch.rand(1, 10, 10, 8, generator=g), 0.6, 1, 1, 1)
    for remainder in (False, True):
        o, lse = kernels.rescue_tail(q.to(DEV), k.to(DEV), v.to(DEV), selected.to(DEV), SCALE, remainder=remainder)
        o_ref, l_ref = oracle.rescue_tail(q.float(), k.float(), v.float(), selected, SCALE, remainder=remainder)
        torch.testing.assert_close(lse.cpu(), l_ref, atol=LSE_TOL, rtol=0)
        torch.testing.assert_close(o.cpu(), o_ref, atol=O_TOL, rtol=0)


def test_decode_at_head_dim_256_matches_dense_softmax():
    """The backend's decode branch (attention.py:178-189) at head dim 256: the split-K decode
    kernel against a dense fp32 softmax, one and three query rows, 16:4 GQA."""
    from exp3_b200 import decode
    g = torch.Generator().manual_seed(256)
    for lq, s_len in ((1, 4097), (3, 300)):
        q = torch.randn(2, lq, 16, 256, generator=g).to(torch.bfloat16)
        k = torch.randn(2, s_len, 4, 256, generator=g).to(torch.bfloat16)
        v = torch.randn(2, s_len, 4, 256, generator=g).to(torch.bfloat16)
        out = decode.decode_attention(q.to(DEV), k.to(DEV), v.to(DEV), SCALE).cpu().float()
        kf = k.float().repeat_interleave(4, dim=2)
        vf = v.float().repeat_interleave(4, dim=2)
        w = torch.einsum("bqhd,bkhd->bhqk", q.float(), kf).mul(SCALE).softmax(-1)
        ref = torch.einsum("bhqk,bkhd->bqhd", w, vf)
        torch.testing.assert_close(out, ref, atol=O_TOL, rtol=0)


@pytest.mark.parametrize("length,heads,kv", [(2049, 16, 4), (32768, 16, 4), (40000, 8, 4), (65536, 4, 2)])
def test_tcgen05_and_mma_route_kernels_agree_at_head_dim_256(length, heads, kv):
    """The tensor-core V1 routing at d = 256 (16 K-steps per chunk, one 64 KB Q stage, two
    resident block-mean chunks) against the mma.sync kernel: scores within fp32 rounding, masks
    bit-exact outside the threshold band. 40000 tokens give 313 blocks, so tiles past 256
    blocks stream their block means; 65536 tokens give 512 blocks, the most the kernel holds at
    d = 256."""
    from test_gpu_parity import assert_masks_match
    shape = synthetic.LayerShape(1, length, heads, kv, 256)
    q, k, v = (x.to(DEV) for x in synthetic.attention_inputs(shape, seed=length + 256, needles=3,
                                                              structured_sigma=0.5))
    mk = upstream.block_mean_k(k)
    scores, sels = [], []
    try:
        for which in ("mma", "tcgen05"):
            _capi.set_route_kernel(which)
            scores.append(upstream.v1_scores(q, mk, SCALE).cpu())
            ops.prefill_attention(q, k, v, "fp_v1", 0.08, SCALE)
            sels.append(ops.export_routing("fp_v1", 1, length, heads, kv, head_dim=256)[0].cpu())
    finally:
        _capi.set_route_kernel("tcgen05")
    torch.testing.assert_close(scores[1], scores[0], atol=1e-6, rtol=1e-5)
    blocks = oracle.num_blocks(length)
    assert_masks_match("fp_v1", sels[1], sels[0], scores[0], 0.08, list(range(blocks)))
    assert _capi.device_error() == 0
