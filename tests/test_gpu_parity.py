"""Parity of the CUDA path (through the C ABI) with the CPU oracle and the reference's golden vectors.

Bars (the benchmark contract): routing masks / indices bit-exact except blocks whose fp32
score lies within 1e-6 of the threshold; outputs within 2e-2 max-abs (bf16); LSE within 1e-3.
"""

import math

import pytest
import torch

import oracle
from exp3_b200 import _capi, decode, kernels, ops, synthetic, upstream
from exp3_b200.attention import AttentionBackend
from golden_cases import SCALE, load, t

pytestmark = pytest.mark.gpu
DEV = "cuda"
O_TOL, LSE_TOL, BAND = 2e-2, 1e-3, 1e-6


def cuda(*xs):
    return [x.to(DEV) for x in xs]


# --------------------------------------------------------------------------- golden vectors


def test_block_mean_k_bit_exact_with_oracle():
    data, q, k, v = load("v1_routing_l1089.npz")
    mine = upstream.block_mean_k(k.to(DEV)).cpu()
    assert torch.equal(mine.view(torch.int16), oracle.block_mean_k(k).view(torch.int16))
    torch.testing.assert_close(mine.float(), t(data["block_mean_fp32"]), atol=2e-3, rtol=2e-2)


def test_v1_scores_match_reference_kernel():
    data, q, k, v = load("v1_routing_l1089.npz")
    mk = t(data["mean_k_bf16_bits"]).view(torch.bfloat16)
    scores = upstream.v1_scores(q.to(DEV), mk.to(DEV), SCALE).cpu()
    torch.testing.assert_close(scores, t(data["scores"]), atol=1e-6, rtol=1e-5)


def test_deal_output_score_bit_exact():
    data, *_ = load("v1_routing_l1089.npz")
    scores = t(data["scores"]).to(DEV)
    idx, cnt = upstream.deal_output_score(scores, 2, 4, 0.08, 2, 0)
    assert torch.equal(idx.cpu(), t(data["indices_a008"])) and torch.equal(cnt.cpu(), t(data["counts_a008"]))
    idx, cnt = upstream.deal_output_score(scores.square().square(), 2, 4, 0.8, 2, 0)
    assert torch.equal(idx.cpu(), t(data["indices_pow4_a08"]))
    assert torch.equal(cnt.cpu(), t(data["counts_pow4_a08"]))


def test_deal_output_score_min_budget_top_k():
    g = torch.Generator().manual_seed(5)
    scores = torch.rand(2, 12, 12, 3, generator=g)  # distinct values: no ties at the k-th place
    for budget in (1, 3, 5):
        idx, cnt = upstream.deal_output_score(scores.to(DEV), 2, 4, 0.5, 2, budget)
        ref_i, ref_c = oracle.deal_output_score(scores, 2, 4, 0.5, 2, budget)
        assert torch.equal(idx.cpu(), ref_i) and torch.equal(cnt.cpu(), ref_c)


def test_descriptors_match_reference():
    data, q, k, v = load("exact_mean_l257.npz")
    desc = kernels.block_descriptors(*cuda(k, v))
    for name in ("mean_k", "mean_v", "var_k", "sigma_v"):
        torch.testing.assert_close(getattr(desc, name).cpu(), t(data[f"desc_{name}"]), atol=2e-6, rtol=1e-5)
    assert torch.equal(desc.counts.cpu(), t(data["desc_counts"]))


def test_selectors_and_selection_match_reference():
    data, q, k, v = load("selectors_l385.npz")
    qd, kd, vd = cuda(q, k, v)
    desc = kernels.block_descriptors(kd, vd)
    for selector in oracle.SELECTORS:
        scores = kernels.selector_scores(qd, desc, SCALE, selector).cpu()
        torch.testing.assert_close(scores, t(data[f"{selector}_scores"]), atol=2e-6, rtol=1e-5)
        ref_scores = t(data[f"{selector}_scores"])
        selected = kernels.protected_selection(ref_scores.to(DEV), 0.08, 2, 4, 2).cpu()
        assert torch.equal(selected, t(data[f"{selector}_selected"]))
        idx, cnt = kernels.indices_from_mask(selected.to(DEV))
        assert torch.equal(idx.cpu(), t(data[f"{selector}_indices"]))
        assert torch.equal(cnt.cpu(), t(data[f"{selector}_counts"]))
        assert torch.equal(kernels.mask_from_indices(idx, cnt).cpu(), selected)
    with pytest.raises(ValueError):
        kernels.selector_scores(qd, desc, SCALE, "nope")


def test_exact_mean_and_merge_match_reference():
    data, q, k, v = load("exact_mean_l257.npz")
    qd, kd, vd = cuda(q, k, v)
    idx, cnt = t(data["indices_fixed"]).to(DEV), t(data["counts_fixed"]).to(DEV)
    out, lse = upstream.exact_attention(qd, kd, vd, idx, cnt, SCALE)
    torch.testing.assert_close(out.cpu().float(), t(data["out_fixed"]), atol=O_TOL, rtol=0)
    torch.testing.assert_close(lse.cpu(), t(data["lse_fixed"]), atol=LSE_TOL, rtol=0)
    desc = kernels.block_descriptors(kd, vd)
    selected = t(data["selected_fixed"]).to(DEV)
    mo, ml = kernels.mean_tail(qd, desc, selected, SCALE)
    torch.testing.assert_close(ml.cpu(), t(data["mean_lse"]), atol=LSE_TOL, rtol=0)
    merged, merged_lse = kernels.merge_exact_mean(out, lse, mo, ml)
    torch.testing.assert_close(merged.cpu().float(), t(data["merged"]), atol=O_TOL, rtol=0)
    torch.testing.assert_close(merged_lse.cpu(), t(data["merged_lse"]), atol=LSE_TOL, rtol=0)
    acc = kernels.selection_accounting(selected, 257, 64, 64, "mean_native", 64)
    ref = oracle.selection_accounting(selected.cpu(), 257, 64, 64, "mean_native", 64)
    for key in ("exact_token_pairs", "selected_block_entries", "mean_proxy_entries", "selector_proxy_entries",
                "exact_physical_qk_tiles"):
        assert int(acc[key]) == int(ref[key]), key


def test_rescue_tails_match_reference():
    data, q, k, v = load("rescue_l1153.npz")
    selected = t(data["selected"])
    rows = t(data["rows"])
    for name, remainder in (("rescue", False), ("rescue_v2", True)):
        out, lse = kernels.rescue_tail(*cuda(q, k, v, selected), SCALE, remainder=remainder)
        torch.testing.assert_close(lse.cpu(), t(data[f"{name}_lse"]), atol=LSE_TOL, rtol=0)
        torch.testing.assert_close(out.cpu()[:, rows], t(data[f"{name}_out_rows"]), atol=O_TOL, rtol=0)


# --------------------------------------------------------------------------- fused path vs oracle


def assert_masks_match(method, gpu_sel, ref_sel, ref_scores, alpha, tiles):
    """Bit-exact on the sampled tiles except entries within BAND of the threshold."""
    for tile in tiles:
        g, r = gpu_sel[:, tile], ref_sel[:, tile]
        diff = g != r
        if not diff.any():
            continue
        assert ref_scores is not None, f"{method}: mask differs on tile {tile}"
        s = ref_scores[:, tile]
        band = (s - s.amax(dim=1, keepdim=True) * alpha).abs() <= BAND
        assert bool((diff <= band).all()), f"{method}: {int(diff.sum())} mask entries differ outside the band"


def run_fused_vs_oracle(method, q, k, v, alpha, tiles):
    qd, kd, vd = cuda(q, k, v)
    batch, length, heads, _ = q.shape
    lse = torch.empty(batch, length, heads, device=DEV)
    out = ops.prefill_attention(qd, kd, vd, method, alpha, SCALE, lse=lse)
    gpu_sel, gpu_idx, gpu_cnt = ops.export_routing(method, batch, length, heads, k.shape[2])
    outs, ref_sel, ref_scores = oracle.prefill_attention_tiles(method, q, k, v, SCALE, alpha, tiles=tiles)
    assert_masks_match(method, gpu_sel.cpu(), ref_sel, ref_scores, alpha, tiles)
    # Compare outputs on tiles where the masks agree exactly.
    agree = [tile for tile in tiles if torch.equal(gpu_sel.cpu()[:, tile], ref_sel[:, tile])]
    assert agree, "no tile with an identical mask to compare outputs on"
    for tile in agree:
        lo, hi = tile * 128, min(length, tile * 128 + 128)
        o_ref, l_ref = outs[tile]
        torch.testing.assert_close(out[:, lo:hi].cpu().float(), o_ref.float(), atol=O_TOL, rtol=0)
        torch.testing.assert_close(lse[:, lo:hi].cpu(), l_ref, atol=LSE_TOL, rtol=0)
    return gpu_sel.cpu()


@pytest.mark.parametrize("method", ["dense", "fp_v1", "mean_native", "mean_balanced", "cgf_mean",
                                    "dispersion_mean", "fp_v1_rescue", "fp_v1_rescue_v2"])
def test_fused_prefill_small(method):
    shape = synthetic.LayerShape(1, 2049, 14, 2)
    q, k, v = synthetic.attention_inputs(shape, seed=31, needles=4, structured_sigma=0.5)
    blocks = oracle.num_blocks(2049)
    sel = run_fused_vs_oracle(method, q, k, v, 0.08, list(range(blocks)))
    if method != "dense":
        density = sel.sum().item() / (14 * blocks * (blocks + 1) / 2)
        assert density <= 1.0


def test_fused_prefill_structured_is_sparse_and_merges_tail():
    shape = synthetic.LayerShape(1, 4096, 7, 1)
    q, k, v = synthetic.attention_inputs(shape, seed=7, needles=2, structured_sigma=0.5)
    sel = run_fused_vs_oracle("mean_native", q, k, v, 0.08, [5, 17, 31])
    assert sel.sum().item() < 7 * 32 * 33 / 2  # the structured variant routes blocks away


@pytest.mark.parametrize("length", [1, 100, 128, 129, 257, 385])
def test_fused_prefill_edge_lengths(length):
    shape = synthetic.LayerShape(2, length, 8, 2)
    q, k, v = synthetic.attention_inputs(shape, seed=length, needles=1)
    blocks = oracle.num_blocks(length)
    for method in ("mean_native", "cgf_mean"):
        run_fused_vs_oracle(method, q, k, v, 0.08, list(range(blocks)))


def test_fused_prefill_wide_gqa_c5_shape():
    shape = synthetic.LayerShape(2, 1024, 40, 8)
    q, k, v = synthetic.attention_inputs(shape, seed=3, key_lognormal_sigma=0.5)
    for method in ("cgf_mean", "dispersion_mean"):
        run_fused_vs_oracle(method, q, k, v, 0.08, [0, 3, 7])


def test_backend_forward_on_hf_layout_matches_fused_op():
    shape = synthetic.LayerShape(1, 1024, 28, 4)
    q, k, v = cuda(*synthetic.attention_inputs(shape, seed=11, needles=2))
    backend = AttentionBackend(alpha=0.08)

    class Layer:
        layer_idx = 3

    for method in ("mean_native", "dispersion_mean", "dense"):
        backend.configure(method)
        out, none = backend.forward(Layer(), q.transpose(1, 2), k.transpose(1, 2), v.transpose(1, 2), None, SCALE)
        assert none is None and out.shape == (1, 1024, 28, 128) and out.is_contiguous()
        ref = ops.prefill_attention(q, k, v, method, 0.08, SCALE)
        assert torch.equal(out, ref)
    backend.configure("mean_native")
    backend.start_profile()
    backend.forward(Layer(), q.transpose(1, 2), k.transpose(1, 2), v.transpose(1, 2), None, SCALE)
    rows = backend.finish_profile()
    assert rows[0]["layer"] == 3 and rows[0]["exact_ms"] > 0 and rows[0]["attention_ms"] > 0
    assert 0 < rows[0]["effective_exact_token_pair_ratio"] <= 1


def test_future_keys_do_not_change_past_outputs():
    """check_math.py:322-329: with the routing fixed, later K/V never reach earlier rows."""
    shape = synthetic.LayerShape(1, 385, 8, 2)
    q, k, v = cuda(*synthetic.attention_inputs(shape, seed=2))
    selected = kernels.protected_selection(torch.zeros(1, 4, 4, 8, device=DEV), 0.0, 2, 4, 2)
    selected[:, 2, 0, ::2] = False
    selected[:, 3, 1, :] = False
    idx, cnt = kernels.indices_from_mask(selected)

    def path(kk, vv):
        desc = kernels.block_descriptors(kk, vv)
        eo, el = upstream.exact_attention(q, kk, vv, idx, cnt, SCALE)
        mo, ml = kernels.mean_tail(q, desc, selected, SCALE)
        return kernels.merge_exact_mean(eo, el, mo, ml)[0]

    first = path(k, v)
    k2, v2 = k.clone(), v.clone()
    k2[:, 300:] *= 19
    v2[:, 300:] += 23
    assert torch.equal(path(k2, v2)[:, :300], first[:, :300])


@pytest.mark.parametrize("method", ["mean_native", "cgf_mean", "fp_v1_rescue_v2"])
def test_fused_path_is_causal_bit_for_bit(method):
    """The fused path (routing, tcgen05 exact attention, tails): K/V rows from block 5 on never
    change rows of tiles 0..4, to the bit (each row's softmax is independent of its warp's
    other rows)."""
    shape = synthetic.LayerShape(1, 1000, 8, 2)
    q, k, v = cuda(*synthetic.attention_inputs(shape, seed=4, needles=2, structured_sigma=0.5))
    first = ops.prefill_attention(q, k, v, method, 0.08, SCALE)
    k2, v2 = k.clone(), v.clone()
    k2[:, 640:] *= 19
    v2[:, 640:] += 23
    second = ops.prefill_attention(q, k2, v2, method, 0.08, SCALE)
    assert torch.equal(second[:, :640], first[:, :640])
    assert not torch.equal(second[:, 640:], first[:, 640:])


def test_decode_matches_dense_softmax():
    g = torch.Generator().manual_seed(9)
    for lq, s_len in ((1, 4097), (3, 300)):
        q = torch.randn(2, lq, 28, 128, generator=g).to(torch.bfloat16)
        k = torch.randn(2, s_len, 4, 128, generator=g).to(torch.bfloat16)
        v = torch.randn(2, s_len, 4, 128, generator=g).to(torch.bfloat16)
        out = decode.decode_attention(*cuda(q, k, v), SCALE).cpu().float()
        kf = k.float().repeat_interleave(7, dim=2)
        vf = v.float().repeat_interleave(7, dim=2)
        w = torch.einsum("bqhd,bkhd->bhqk", q.float(), kf).mul(SCALE).softmax(-1)
        ref = torch.einsum("bhqk,bkhd->bqhd", w, vf)
        torch.testing.assert_close(out, ref, atol=O_TOL, rtol=0)


# --------------------------------------------------------------------------- benchmark configurations


def test_config1_4k_mean_native_sampled_tiles():
    q, k, v = synthetic.config_inputs("c1", seed=0)
    sel = run_fused_vs_oracle("mean_native", q, k, v, 0.08, [0, 1, 9, 20, 30, 31])
    assert sel.shape == (1, 32, 32, 28)


@pytest.mark.slow
def test_config2_32k_properties_and_sampled_tiles():
    q, k, v = synthetic.config_inputs("c2", seed=0)
    run_fused_vs_oracle("mean_native", q, k, v, 0.08, [0, 37, 255])
    # Size-independent properties at full size: idempotence (same inputs, same bits) and
    # density reported as selected / causal blocks.
    qd, kd, vd = cuda(q, k, v)
    a = ops.prefill_attention(qd, kd, vd, "mean_native", 0.08, SCALE)
    b = ops.prefill_attention(qd, kd, vd, "mean_native", 0.08, SCALE)
    assert torch.equal(a, b)
    sel, _, cnt = ops.export_routing("mean_native", 1, 32768, 28, 4)
    causal = 28 * 256 * 257 // 2
    assert int(cnt.sum()) == int(sel.sum()) <= causal
    assert math.isfinite(a.float().abs().max().item())


@pytest.mark.slow
def test_config4_128k_sampled_tiles_and_properties():
    """Config 4 (131072 tokens, 1024 blocks): late tiles route over eight 128-block chunks."""
    q, k, v = synthetic.config_inputs("c4", seed=0)
    run_fused_vs_oracle("mean_native", q, k, v, 0.08, [3, 600, 1023])
    qd, kd, vd = cuda(q, k, v)
    a = ops.prefill_attention(qd, kd, vd, "mean_native", 0.08, SCALE)
    sel, idx, cnt = ops.export_routing("mean_native", 1, 131072, 28, 4)
    assert int(cnt.sum()) == int(sel.sum()) <= 28 * 1024 * 1025 // 2
    assert bool((idx.max(dim=2).values <= 1024).all())
    b = ops.prefill_attention(qd, kd, vd, "mean_native", 0.08, SCALE)
    assert torch.equal(a, b)
    assert _capi.device_error() == 0


def test_tcgen05_and_mma_exact_kernels_agree():
    shape = synthetic.LayerShape(1, 2048, 28, 4)
    q, k, v = cuda(*synthetic.attention_inputs(shape, seed=5, needles=3, structured_sigma=0.5))
    results = []
    try:
        for which in ("mma", "tcgen05"):
            _capi.set_exact_kernel(which)
            lse = torch.empty(1, 2048, 28, device=DEV)
            out = ops.prefill_attention(q, k, v, "mean_native", 0.08, SCALE, lse=lse)
            results.append((out, lse))
    finally:
        _capi.set_exact_kernel("tcgen05")
    torch.testing.assert_close(results[0][0].float(), results[1][0].float(), atol=O_TOL, rtol=0)
    torch.testing.assert_close(results[0][1], results[1][1], atol=LSE_TOL, rtol=0)
    assert _capi.device_error() == 0


@pytest.mark.parametrize("kernel", ["tcgen05_single"])
@pytest.mark.parametrize("method", ["mean_native", "fp_v1", "dense", "cgf_mean"])
def test_single_tile_exact_kernel_matches_oracle(method, kernel):
    """The one-tile-per-CTA tcgen05 kernel (double-buffered S) at head dim 128, selected with
    fpx_set_option(1, 2): the fused path against the oracle, ragged last tile, B = 2, heads of an
    odd group (7) included."""
    shape = synthetic.LayerShape(2, 2177, 14, 2)
    q, k, v = synthetic.attention_inputs(shape, seed=12, needles=4, structured_sigma=0.5)
    try:
        _capi.set_exact_kernel(kernel)
        run_fused_vs_oracle(method, q, k, v, 0.08, list(range(oracle.num_blocks(2177))))
    finally:
        _capi.set_exact_kernel("tcgen05")
    assert _capi.device_error() == 0


def test_alternative_exact_kernels_reference_layout_and_agreement():
    data, q, k, v = load("exact_mean_l257.npz")
    qd, kd, vd = cuda(q, k, v)
    idx, cnt = t(data["indices_fixed"]).to(DEV), t(data["counts_fixed"]).to(DEV)
    shape = synthetic.LayerShape(1, 32768, 28, 4)
    q2, k2, v2 = cuda(*synthetic.attention_inputs(shape, seed=8, needles=8, structured_sigma=0.5))
    results = []
    try:
        for which in ("tcgen05_single", "tcgen05"):
            _capi.set_exact_kernel(which)
            out, lse = upstream.exact_attention(qd, kd, vd, idx, cnt, SCALE)
            torch.testing.assert_close(out.cpu().float(), t(data["out_fixed"]), atol=O_TOL, rtol=0)
            torch.testing.assert_close(lse.cpu(), t(data["lse_fixed"]), atol=LSE_TOL, rtol=0)
            lse2 = torch.empty(1, 32768, 28, device=DEV)
            results.append((ops.prefill_attention(q2, k2, v2, "mean_native", 0.08, SCALE, lse=lse2), lse2))
    finally:
        _capi.set_exact_kernel("tcgen05")
    # 32K: the tcgen05 kernels agree (same products, same rounding points)
    torch.testing.assert_close(results[0][0].float(), results[1][0].float(), atol=O_TOL, rtol=0)
    torch.testing.assert_close(results[0][1], results[1][1], atol=LSE_TOL, rtol=0)
    assert _capi.device_error() == 0


@pytest.mark.parametrize("length,heads,kv", [(2049, 14, 2), (32768, 28, 4), (40000, 10, 2), (65600, 4, 2)])
def test_tcgen05_and_mma_route_kernels_agree(length, heads, kv):
    """The tensor-core V1 routing (transposed products in TMEM, persistent CTAs) against the
    mma.sync kernel: scores within fp32 rounding, masks bit-exact outside the threshold band.
    40000 tokens give 313 blocks: items past 256 blocks stream their block means per unit, and
    the last tile is ragged. 65600 tokens give 513 blocks: heads of five chunks, more than a
    warpgroup's two accumulator slots hold."""
    shape = synthetic.LayerShape(1, length, heads, kv)
    q, k, v = cuda(*synthetic.attention_inputs(shape, seed=length, needles=3, structured_sigma=0.5))
    mk = upstream.block_mean_k(k)
    scores, sels = [], []
    try:
        for which in ("mma", "tcgen05"):
            _capi.set_route_kernel(which)
            scores.append(upstream.v1_scores(q, mk, SCALE).cpu())
            ops.prefill_attention(q, k, v, "mean_native", 0.08, SCALE)
            sels.append(ops.export_routing("mean_native", 1, length, heads, kv)[0].cpu())
    finally:
        _capi.set_route_kernel("tcgen05")
    torch.testing.assert_close(scores[1], scores[0], atol=1e-6, rtol=1e-5)
    blocks = oracle.num_blocks(length)
    assert_masks_match("mean_native", sels[1], sels[0], scores[0], 0.08, list(range(blocks)))
    assert _capi.device_error() == 0


@pytest.mark.parametrize("length,heads,kv", [(4096, 28, 4), (40000, 10, 2)])
def test_tcgen05_and_fp32_mean_tails_agree(length, heads, kv):
    """The tensor-core tail (mean K as bf16 high + low halves, chunks of 128 pseudo-keys) against
    the fp32 CUDA-core tail on structured inputs with real tails; 40000 tokens give 313 blocks,
    so late tiles span three chunks."""
    shape = synthetic.LayerShape(1, length, heads, kv)
    q, k, v = cuda(*synthetic.attention_inputs(shape, seed=length + 1, needles=3, structured_sigma=0.5))
    results = []
    try:
        for which in ("fp32", "tcgen05"):
            _capi.set_mean_kernel(which)
            lse = torch.empty(1, length, heads, device=DEV)
            out = ops.prefill_attention(q, k, v, "mean_native", 0.08, SCALE, lse=lse)
            results.append((out, lse))
    finally:
        _capi.set_mean_kernel("tcgen05")
    sel = ops.export_routing("mean_native", 1, length, heads, kv)[0]
    assert int(sel.sum()) < heads * oracle.num_blocks(length) * (oracle.num_blocks(length) + 1) // 2  # tails exist
    torch.testing.assert_close(results[1][0].float(), results[0][0].float(), atol=O_TOL, rtol=0)
    torch.testing.assert_close(results[1][1], results[0][1], atol=LSE_TOL, rtol=0)
    assert _capi.device_error() == 0


@pytest.mark.parametrize("method", ["fp_v1_rescue", "fp_v1_rescue_v2"])
@pytest.mark.parametrize("length,heads,kv", [(4096, 28, 4), (40000, 10, 2)])
def test_tcgen05_and_fp32_rescue_tails_agree(method, length, heads, kv):
    """The tensor-core rescue tail (gathered rescue rows; for _v2 the remainder means as bf16
    high + low halves) against the fp32 CUDA-core tail on structured inputs with real tails;
    40000 tokens give 313 blocks, so late tiles have three chunks of tail keys per pass."""
    shape = synthetic.LayerShape(1, length, heads, kv)
    q, k, v = cuda(*synthetic.attention_inputs(shape, seed=length + 2, needles=3, structured_sigma=0.5))
    results = []
    try:
        for which in ("fp32", "tcgen05"):
            _capi.set_mean_kernel(which)
            lse = torch.empty(1, length, heads, device=DEV)
            out = ops.prefill_attention(q, k, v, method, 0.08, SCALE, lse=lse)
            results.append((out, lse))
    finally:
        _capi.set_mean_kernel("tcgen05")
    sel = ops.export_routing(method, 1, length, heads, kv)[0]
    assert int(sel.sum()) < heads * oracle.num_blocks(length) * (oracle.num_blocks(length) + 1) // 2  # tails exist
    torch.testing.assert_close(results[1][0].float(), results[0][0].float(), atol=O_TOL, rtol=0)
    torch.testing.assert_close(results[1][1], results[0][1], atol=LSE_TOL, rtol=0)
    assert _capi.device_error() == 0


@pytest.mark.parametrize("method", ["mean_balanced", "cgf_mean", "dispersion_mean"])
@pytest.mark.parametrize("length,heads,kv", [(4096, 14, 2), (40000, 10, 2)])
def test_tcgen05_and_fp32_selector_routing_agree(method, length, heads, kv):
    """The tensor-core selector routing (descriptors as bf16 high + low halves, two passes)
    against the fp32 CUDA-core kernel: masks bit-exact outside the threshold band of the fp32
    scores (fpx_selector_scores). 40000 tokens: late tiles span three 128-block chunks."""
    shape = synthetic.LayerShape(1, length, heads, kv)
    q, k, v = cuda(*synthetic.attention_inputs(shape, seed=length + 7, needles=3, structured_sigma=0.5))
    sels = []
    try:
        for which in ("fp32", "tcgen05"):
            _capi.set_selector_kernel(which)
            ops.prefill_attention(q, k, v, method, 0.08, SCALE, stages=_capi.STAGE_ROUTE)
            sels.append(ops.export_routing(method, 1, length, heads, kv)[0].cpu())
    finally:
        _capi.set_selector_kernel("tcgen05")
    desc = kernels.block_descriptors(k, v)
    scores = kernels.selector_scores(q, desc, SCALE, method).cpu()
    blocks = oracle.num_blocks(length)
    assert_masks_match(method, sels[1], sels[0], scores, 0.08, list(range(blocks)))
    assert int(sels[1].sum()) < heads * blocks * (blocks + 1) // 2  # the structured inputs route blocks away
    assert _capi.device_error() == 0


@pytest.mark.slow
def test_fused_prefill_divergent_head_lists_32k():
    """Two query heads of one KV group whose block lists differ a lot (structured routing at 32K):
    the tensor-core kernel streams the union of both lists, so one tile runs far ahead of the other."""
    shape = synthetic.LayerShape(1, 32768, 2, 1)
    q, k, v = synthetic.attention_inputs(shape, seed=13, needles=4, structured_sigma=0.5)
    sel = run_fused_vs_oracle("mean_native", q, k, v, 0.08, [40, 160, 255])
    assert not torch.equal(sel[..., 0], sel[..., 1])  # the heads really route differently
    assert _capi.device_error() == 0
