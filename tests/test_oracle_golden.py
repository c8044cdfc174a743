"""Pins the CPU oracle against the reference's own outputs (tests/golden, made by make_golden.py)."""

import math

import numpy as np
import torch

import oracle
from golden_cases import SCALE, load, t


def test_v1_block_mean_matches_reference_mean():
    data, q, k, v = load("v1_routing_l1089.npz")
    mine = oracle.block_mean_k(k)
    ref = t(data["block_mean_fp32"])
    # The reference's own gate (check_math.py:292-300).
    torch.testing.assert_close(mine.float(), ref, atol=2e-3, rtol=2e-2)
    # The oracle's bf16 mean is the correctly rounded fp32 mean almost everywhere.
    same = (mine == ref.to(torch.bfloat16)).float().mean().item()
    assert same > 0.999, same


def test_v1_scores_match_reference_kernel():
    data, q, k, v = load("v1_routing_l1089.npz")
    mk = t(data["mean_k_bf16_bits"]).view(torch.bfloat16)
    mine = oracle.v1_scores(q, mk, SCALE)
    torch.testing.assert_close(mine, t(data["scores"]), atol=1e-6, rtol=1e-5)
    torch.testing.assert_close(mine, t(data["scores_check_math"]), atol=1e-6, rtol=1e-5)


def test_v1_selection_is_bit_exact():
    data, *_ = load("v1_routing_l1089.npz")
    scores = t(data["scores"])
    idx, cnt = oracle.deal_output_score(scores, 2, 4, 0.08, 2, 0)
    assert torch.equal(idx, t(data["indices_a008"])) and torch.equal(cnt, t(data["counts_a008"]))
    idx, cnt = oracle.deal_output_score(scores.square().square(), 2, 4, 0.8, 2, 0)
    assert torch.equal(idx, t(data["indices_pow4_a08"])) and torch.equal(cnt, t(data["counts_pow4_a08"]))


def test_exact_path_matches_reference_kernel():
    data, q, k, v = load("exact_mean_l257.npz")
    q32, k32, v32 = q.float(), k.float(), v.float()
    out, lse = oracle.exact_attention(q32, k32, v32, t(data["indices_fixed"]), t(data["counts_fixed"]), SCALE)
    torch.testing.assert_close(out, t(data["out_fixed"]), atol=2e-6, rtol=1e-5)
    torch.testing.assert_close(lse, t(data["lse_fixed"]), atol=2e-6, rtol=1e-5)
    every = oracle.protected_selection(torch.zeros(1, 3, 3, 4), 0.0, 2, 4, 2)
    idx, cnt = oracle.indices_from_mask(every)
    _, lse_all = oracle.exact_attention(q32, k32, v32, idx, cnt, SCALE)
    torch.testing.assert_close(lse_all, t(data["lse_all"]), atol=2e-6, rtol=1e-5)
    torch.testing.assert_close(lse_all, t(data["dense_lse"]), atol=2e-6, rtol=1e-5)


def test_descriptors_mean_tail_and_merge_match_reference():
    data, q, k, v = load("exact_mean_l257.npz")
    q32, k32, v32 = q.float(), k.float(), v.float()
    desc = oracle.block_descriptors(k32, v32)
    for name in ("mean_k", "mean_v", "var_k", "sigma_v"):
        torch.testing.assert_close(getattr(desc, name), t(data[f"desc_{name}"]), atol=1e-6, rtol=1e-5)
    assert torch.equal(desc.counts, t(data["desc_counts"]))
    selected = t(data["selected_fixed"])
    out_e, lse_e = oracle.exact_attention(q32, k32, v32, *oracle.indices_from_mask(selected), SCALE)
    out_m, lse_m = oracle.mean_tail(q32, desc, selected, SCALE)
    torch.testing.assert_close(lse_m, t(data["mean_lse"]), atol=2e-6, rtol=1e-5)
    merged, merged_lse = oracle.merge_exact_mean(out_e, lse_e, out_m, lse_m)
    torch.testing.assert_close(merged, t(data["merged"]), atol=2e-6, rtol=1e-5)
    torch.testing.assert_close(merged_lse, t(data["merged_lse"]), atol=2e-6, rtol=1e-5)
    torch.testing.assert_close(merged_lse, t(data["explicit_lse"]), atol=1e-5, rtol=1e-5)
    # Tile-wise whole-path helper gives the same merged result (bf16 exact output path aside).
    outs, _, _ = oracle.prefill_attention_tiles(
        "mean_native", q32, k32, v32, SCALE, 0.08, routing=(selected, None, desc))
    for tile, (o_t, l_t) in outs.items():
        lo, hi = tile * 128, min(257, tile * 128 + 128)
        torch.testing.assert_close(o_t, t(data["merged"])[:, lo:hi], atol=2e-6, rtol=1e-5)


def test_accounting_matches_reference():
    data, *_ = load("exact_mean_l257.npz")
    acc = oracle.selection_accounting(t(data["selected_fixed"]), 257, 64, 64, "mean_native", 64)
    for key, value in zip(data["accounting_keys"], data["accounting_values"]):
        mine = acc[str(key)]
        if math.isnan(value):
            assert mine is None, key
        else:
            assert math.isclose(float(mine), float(value), rel_tol=1e-6), (key, mine, value)  # ratios are fp32 tensors there


def test_selectors_match_reference():
    data, q, k, v = load("selectors_l385.npz")
    desc = oracle.block_descriptors(k, v)
    for selector in oracle.SELECTORS:
        scores = oracle.selector_scores(q, desc, SCALE, selector)
        torch.testing.assert_close(scores, t(data[f"{selector}_scores"]), atol=1e-6, rtol=1e-5)
        selected = oracle.protected_selection(t(data[f"{selector}_scores"]), 0.08, 2, 4, 2)
        assert torch.equal(selected, t(data[f"{selector}_selected"]))
        idx, cnt = oracle.indices_from_mask(selected)
        assert torch.equal(idx, t(data[f"{selector}_indices"]))
        assert torch.equal(cnt, t(data[f"{selector}_counts"]))
        assert torch.equal(oracle.mask_from_indices(idx, cnt), selected)


def test_unknown_selector_raises():
    _, q, k, v = load("selectors_l385.npz")
    try:
        oracle.selector_scores(q, oracle.block_descriptors(k, v), SCALE, "nope")
    except ValueError:
        return
    raise AssertionError("unknown selector accepted")


def test_rescue_tails_match_reference():
    data, q, k, v = load("rescue_l1153.npz")
    selected = t(data["selected"])
    rows = t(data["rows"])
    assert (~selected).any()  # the fixture's tiles have tails
    for name, remainder in (("rescue", False), ("rescue_v2", True)):
        out, lse = oracle.rescue_tail(q, k, v, selected, SCALE, remainder=remainder)
        torch.testing.assert_close(lse, t(data[f"{name}_lse"]), atol=1e-5, rtol=1e-5)
        torch.testing.assert_close(out[:, rows], t(data[f"{name}_out_rows"]), atol=1e-5, rtol=1e-5)


# ---------------------------------------------------------------- head dim 256 (Qwen3.5 shape)


def test_head_dim_256_routing_matches_reference():
    data, q, k, v = load("qwen35_routing_l1025.npz")
    assert q.shape == (1, 1025, 16, 256) and k.shape == (1, 1025, 4, 256)
    mine = oracle.block_mean_k(k)
    ref = t(data["block_mean_fp32"])
    torch.testing.assert_close(mine.float(), ref, atol=2e-3, rtol=2e-2)
    assert (mine == ref.to(torch.bfloat16)).float().mean().item() > 0.999
    mk = t(data["mean_k_bf16_bits"]).view(torch.bfloat16)
    scores = oracle.v1_scores(q, mk, 256 ** -0.5)
    torch.testing.assert_close(scores, t(data["scores"]), atol=1e-6, rtol=1e-5)
    ref_scores = t(data["scores"])
    idx, cnt = oracle.deal_output_score(ref_scores, 2, 4, 0.08, 2, 0)
    assert torch.equal(idx, t(data["indices_a008"])) and torch.equal(cnt, t(data["counts_a008"]))
    idx, cnt = oracle.deal_output_score(ref_scores.square().square(), 2, 4, 0.8, 2, 0)
    assert torch.equal(idx, t(data["indices_pow4_a08"])) and torch.equal(cnt, t(data["counts_pow4_a08"]))


def test_head_dim_256_exact_path_matches_reference():
    data, q, k, v = load("qwen35_exact_l385.npz")
    q32, k32, v32 = q.float(), k.float(), v.float()
    rows, heads = t(data["rows"]), t(data["out_heads"])
    out, lse = oracle.exact_attention(q32, k32, v32, t(data["indices_fixed"]), t(data["counts_fixed"]), 256 ** -0.5)
    torch.testing.assert_close(lse, t(data["lse_fixed"]), atol=2e-6, rtol=1e-5)
    torch.testing.assert_close(out[:, rows][:, :, heads], t(data["out_fixed_rows"]), atol=2e-6, rtol=1e-5)
    every = oracle.protected_selection(torch.zeros(1, 4, 4, 16), 0.0, 2, 4, 2)
    idx, cnt = oracle.indices_from_mask(every)
    out, lse = oracle.exact_attention(q32, k32, v32, idx, cnt, 256 ** -0.5)
    torch.testing.assert_close(lse, t(data["lse_all"]), atol=2e-6, rtol=1e-5)
    torch.testing.assert_close(out[:, rows][:, :, heads], t(data["out_all_rows"]), atol=2e-6, rtol=1e-5)


def test_head_dim_256_tails_and_selectors_match_reference():
    """The oracle's descriptors, block-mean tail, selectors + selection and rescue tails at
    d = 256 against the reference's own kernels.py functions on the same inputs."""
    data, q, k, v = load("qwen35_tails_l1153.npz")
    scale = 256 ** -0.5
    q32, k32, v32 = q.float(), k.float(), v.float()
    rows, heads = t(data["rows"]), t(data["out_heads"])
    desc = oracle.block_descriptors(k32, v32)
    for name in ("mean_k", "mean_v", "var_k", "sigma_v"):
        torch.testing.assert_close(getattr(desc, name), t(data[f"desc_{name}"]), atol=1e-6, rtol=1e-5)
    selected = t(data["selected"])
    out, lse = oracle.mean_tail(q32, desc, selected, scale)
    torch.testing.assert_close(lse, t(data["mean_lse"]), atol=2e-6, rtol=1e-5)
    torch.testing.assert_close(out[:, rows][:, :, heads], t(data["mean_out_rows"]), atol=2e-6, rtol=1e-5)
    for selector in oracle.SELECTORS:
        scores = oracle.selector_scores(q32, desc, scale, selector)
        torch.testing.assert_close(scores, t(data[f"{selector}_scores"]), atol=2e-5, rtol=2e-5)
        sel = oracle.protected_selection(t(data[f"{selector}_scores"]), 0.08, 2, 4, 2)
        assert torch.equal(sel, t(data[f"{selector}_selected"]))
    for name, remainder in (("rescue", False), ("rescue_v2", True)):
        o, l = oracle.rescue_tail(q32, k32, v32, selected, scale, remainder=remainder)
        torch.testing.assert_close(l, t(data[f"{name}_lse"]), atol=2e-6, rtol=1e-5)
        torch.testing.assert_close(o[:, rows][:, :, heads], t(data[f"{name}_out_rows"]), atol=2e-6, rtol=1e-5)


def test_edge_lengths_match_reference():
    """L = 1 and L = 129 (a one-row block): the oracle's V1 block mean, scores, selection, exact
    path, mean tail and merge against the reference run on the same inputs."""
    from exp3_b200 import synthetic
    from golden_cases import GOLDEN
    data = dict(np.load(GOLDEN / "edges_l1_l129.npz", allow_pickle=False))
    for length in (1, 129):
        tag = f"l{length}"
        shape = synthetic.LayerShape(1, length, 4, 2)
        q, k, v = synthetic.attention_inputs(shape, seed=int(data[f"{tag}_seed"]), needles=2, apply_rope=True)
        assert synthetic.tensor_digest(q, k, v) == str(data[f"{tag}_digest"])
        q32, k32, v32 = q.float(), k.float(), v.float()
        mk = oracle.block_mean_k(k)
        torch.testing.assert_close(mk.float(), t(data[f"{tag}_block_mean_fp32"]), atol=2e-3, rtol=2e-2)
        ref_mk = t(data[f"{tag}_block_mean_fp32"]).to(torch.bfloat16)
        scores = oracle.v1_scores(q, ref_mk, SCALE)
        torch.testing.assert_close(scores, t(data[f"{tag}_scores"]), atol=1e-6, rtol=1e-5)
        idx, cnt = oracle.deal_output_score(t(data[f"{tag}_scores"]), 2, 4, 0.08, 2, 0)
        assert torch.equal(idx, t(data[f"{tag}_indices_a008"])) and torch.equal(cnt, t(data[f"{tag}_counts_a008"]))
        blocks = (length + 127) // 128
        every = oracle.protected_selection(torch.zeros(1, blocks, blocks, 4), 0.0, 2, 4, 2)
        a_idx, a_cnt = oracle.indices_from_mask(every)
        out, lse = oracle.exact_attention(q32, k32, v32, a_idx, a_cnt, SCALE)
        torch.testing.assert_close(out, t(data[f"{tag}_out_all"]), atol=2e-6, rtol=1e-5)
        torch.testing.assert_close(lse, t(data[f"{tag}_lse_all"]), atol=2e-6, rtol=1e-5)
        selected = t(data[f"{tag}_selected"])
        f_idx, f_cnt = oracle.indices_from_mask(selected)
        eo, el = oracle.exact_attention(q32, k32, v32, f_idx, f_cnt, SCALE)
        desc = oracle.block_descriptors(k32, v32)
        mo, ml = oracle.mean_tail(q32, desc, selected, SCALE)
        merged, merged_lse = oracle.merge_exact_mean(eo, el, mo, ml)
        torch.testing.assert_close(merged.float(), t(data[f"{tag}_merged"]), atol=2e-6, rtol=1e-5)
        torch.testing.assert_close(merged_lse, t(data[f"{tag}_merged_lse"]), atol=2e-6, rtol=1e-5)
