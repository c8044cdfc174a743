"""Generate the golden vectors in this folder by running the exp3 reference itself.

Run in the build container, where the reference tree is mounted; its path is the
first argument (or ``FPX_REFERENCE_ROOT``). The GPU box never runs this.

    python tests/golden/make_golden.py <path of the reference tree>

What runs, all on the CPU in fp32:
- the reference's torch functions in ``kernels.py`` (descriptors, selectors,
  protected selection, index/mask conversion, mean tail, rescue tails, merge,
  accounting);
- the reference's Triton kernels in ``upstream/flashprefill_native_forward.py``
  under ``TRITON_INTERPRET=1`` (``compute_mean_vector``, ``compute_block_score``,
  ``_flash_forward`` called through ``.fn[grid]`` with fixed tile sizes, which
  bypasses the autotuner), plus the uncompiled bodies of its ``torch.compile``
  helpers (``normalize_scores``, ``_deal_output_score_compiled``);
- the fp32 restatements in ``check_math.py`` (``dense_reference``,
  ``v1_score_reference``, ``v1_selection_reference``,
  ``explicit_mean_reference``, ``selector_reference``);
- for head dim 256 (the Qwen3.5 shape, 16 query heads over 4 KV heads), the same Triton
  kernels with ``D_HEAD=256`` and the restatements in ``check_qwen35_math.py``
  (``mean_reference``, ``score_reference``, ``selection_reference``, ``dense_reference``),
  and the torch functions of ``kernels.py`` (descriptors, mean tail, selectors, rescue tails)
  on d = 256 inputs.

The interpreter cannot run bf16 (it yields NaN), so bf16 inputs are upcast to
fp32 first; values stay bf16-representable. Inputs are not stored: they are
regenerated from the seeds by ``exp3_b200.synthetic`` and pinned by a sha256
digest stored with each case.
"""

from __future__ import annotations

import os
import sys
from pathlib import Path

os.environ["TRITON_INTERPRET"] = "1"

import numpy as np  # noqa: E402
import torch  # noqa: E402

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parents[1]))
from exp3_b200 import synthetic  # noqa: E402

SCALE = 128 ** -0.5


def load_reference(root: str):
    sys.path.insert(0, root)
    import check_math  # noqa: F401  (imports attention, kernels, upstream)
    import kernels
    from upstream import flashprefill_native_forward as upstream
    return check_math, kernels, upstream


def load_qwen35(root: str):
    """check_qwen35_math.py uses package-relative imports: import it as a package module."""
    import importlib
    parent, name = os.path.split(os.path.abspath(root))
    sys.path.insert(0, parent)
    return importlib.import_module(f"{name}.check_qwen35_math")


def inputs(seed, length, heads, kv_heads, head_dim=128):
    shape = synthetic.LayerShape(1, length, heads, kv_heads, head_dim)
    return synthetic.attention_inputs(shape, seed=seed, needles=2, apply_rope=True)


def ref_block_mean(upstream, k32):
    b, length, hkv, d = k32.shape
    blocks = (length + 127) // 128
    mean = torch.empty(b, blocks, hkv, d)
    upstream.compute_mean_vector.fn[(blocks, b * hkv, 1)](
        k32, mean, *k32.stride(), *mean.stride(), hkv, length, BLOCK_SIZE=128, D_HEAD=d)
    return mean


def ref_v1_scores(upstream, q32, mk32, scale=SCALE):
    b, length, h, d = q32.shape
    blocks, hkv = mk32.shape[1], mk32.shape[2]
    score = torch.full((b, blocks, blocks, h), float("-inf"))
    maximum = torch.full_like(score, float("-inf"))
    upstream.compute_block_score.fn[(blocks, b * h, 1)](
        q32, mk32, scale, score, maximum, *q32.stride(), *mk32.stride(), *score.stride(),
        *maximum.stride(), h, hkv, length, blocks, BLOCK_SIZE=128, K_TILE_SIZE=64, K_STRIDE=128, D_HEAD=d)
    return upstream.normalize_scores._torchdynamo_orig_callable(score, maximum)


def ref_exact(upstream, q32, k32, v32, indices, counts, scale=SCALE):
    b, length, h, d = q32.shape
    out = torch.empty_like(q32)
    lse = torch.empty(b, length, h)
    upstream._flash_forward.fn[((length + 63) // 64, b * h, 1)](
        q32, k32, v32, out, lse, indices, counts, scale, *q32.stride(), *k32.stride(), *v32.stride(),
        *out.stride(), *lse.stride(), *indices.stride(), *counts.stride(), length, length, h, k32.shape[2],
        Q_TILE_SIZE=64, K_TILE_SIZE=64, BLOCK_SIZE=128, D_HEAD=d)
    return out, lse


def deal(upstream, score, alpha):
    return upstream._deal_output_score_compiled._torchdynamo_orig_callable(score, 2, 4, alpha, 2, 0)


def main(root=None):
    root = root or os.environ.get("FPX_REFERENCE_ROOT")
    if not root:
        raise SystemExit("usage: make_golden.py <path of the reference tree> (or set FPX_REFERENCE_ROOT)")
    check_math, kernels, upstream = load_reference(root)
    torch.manual_seed(0)

    # Case 1: V1 routing at L=1089 (9 blocks, the last with 65 rows), GQA 2:1.
    seed, length, heads, kv_heads = 101, 1089, 4, 2
    q, k, v = inputs(seed, length, heads, kv_heads)
    q32, k32 = q.float(), k.float()
    mean32 = ref_block_mean(upstream, k32)
    mk = mean32.to(torch.bfloat16)  # bf16 input for the scoring stage
    scores = ref_v1_scores(upstream, q32, mk.float())
    scores_cm = check_math.v1_score_reference(q32, mk.float(), SCALE)
    idx08, cnt08 = deal(upstream, scores, 0.08)
    idx_p4, cnt_p4 = deal(upstream, scores.square().square(), 0.8)
    ref_i, ref_c = check_math.v1_selection_reference(scores.square().square(), 2, 4, 0.8, 2)
    assert torch.equal(idx_p4, ref_i) and torch.equal(cnt_p4, ref_c)
    np.savez_compressed(
        HERE / "v1_routing_l1089.npz",
        seed=seed, length=length, heads=heads, kv_heads=kv_heads,
        digest=synthetic.tensor_digest(q, k, v),
        block_mean_fp32=mean32.numpy(), mean_k_bf16_bits=mk.view(torch.int16).numpy(),
        scores=scores.numpy(), scores_check_math=scores_cm.numpy(),
        indices_a008=idx08.numpy(), counts_a008=cnt08.numpy(),
        indices_pow4_a08=idx_p4.numpy(), counts_pow4_a08=cnt_p4.numpy(),
    )

    # Case 2: exact path (all causal) and exact + mean merge with a fixed mask, L=257.
    seed, length, heads, kv_heads = 17, 257, 4, 2
    q, k, v = inputs(seed, length, heads, kv_heads)
    q32, k32, v32 = q.float(), k.float(), v.float()
    blocks = 3
    all_selected = kernels.protected_selection(torch.zeros(1, blocks, blocks, heads), 0.0, 2, 4, 2)
    a_idx, a_cnt = kernels.indices_from_mask(all_selected)
    out_all, lse_all = ref_exact(upstream, q32, k32, v32, a_idx, a_cnt)
    dense_o, dense_lse = check_math.dense_reference(q32, k32, v32, SCALE)
    selected = all_selected.clone()
    selected[:, 2, 1, ::2] = False
    f_idx, f_cnt = kernels.indices_from_mask(selected)
    out_fixed, lse_fixed = ref_exact(upstream, q32, k32, v32, f_idx, f_cnt)
    desc = kernels.block_descriptors(k32, v32)
    m_out, m_lse = kernels.mean_tail(q32, desc, selected, SCALE)
    merged, merged_lse = kernels.merge_exact_mean(out_fixed, lse_fixed, m_out, m_lse)
    explicit, explicit_lse = check_math.explicit_mean_reference(q32, k32, v32, selected, desc, SCALE)
    accounting = kernels.selection_accounting(selected, length, 64, 64, "mean_native", 64)
    # The reference's own gates (check_math.py:237-250), checked here instead of storing both sides.
    torch.testing.assert_close(out_all, dense_o, atol=1e-5, rtol=1e-5)
    torch.testing.assert_close(merged, explicit, atol=1e-5, rtol=1e-5)
    torch.testing.assert_close(merged_lse, explicit_lse, atol=1e-5, rtol=1e-5)
    np.savez_compressed(
        HERE / "exact_mean_l257.npz",
        seed=seed, length=length, heads=heads, kv_heads=kv_heads,
        digest=synthetic.tensor_digest(q, k, v),
        selected_fixed=selected.numpy(), indices_fixed=f_idx.numpy(), counts_fixed=f_cnt.numpy(),
        lse_all=lse_all.numpy(), dense_lse=dense_lse.numpy(),
        out_fixed=out_fixed.numpy(), lse_fixed=lse_fixed.numpy(),
        mean_lse=m_lse.numpy(),
        merged=merged.numpy(), merged_lse=merged_lse.numpy(),
        explicit_lse=explicit_lse.numpy(),
        desc_mean_k=desc.mean_k.numpy(), desc_mean_v=desc.mean_v.numpy(),
        desc_var_k=desc.var_k.numpy(), desc_sigma_v=desc.sigma_v.numpy(), desc_counts=desc.counts.numpy(),
        accounting_keys=np.array(sorted(accounting)),
        accounting_values=np.array([float(accounting[key]) if accounting[key] is not None else np.nan
                                    for key in sorted(accounting)]),
    )

    # Case 3: the three new selectors and their protected selection, L=385 (last tile 1 row).
    seed, length, heads, kv_heads = 23, 385, 4, 2
    q, k, v = inputs(seed, length, heads, kv_heads)
    q32, k32, v32 = q.float(), k.float(), v.float()
    desc = kernels.block_descriptors(k32, v32)
    record = {"seed": seed, "length": length, "heads": heads, "kv_heads": kv_heads,
              "digest": synthetic.tensor_digest(q, k, v)}
    for selector in ("mean_balanced", "cgf_mean", "dispersion_mean"):
        s = kernels.selector_scores(q32, desc, SCALE, selector, chunk_tiles=2)
        s_ref = check_math.selector_reference(q32, desc, SCALE, selector)
        torch.testing.assert_close(s, s_ref, atol=2e-5, rtol=2e-5)
        sel = kernels.protected_selection(s, 0.08, 2, 4, 2)
        i, c = kernels.indices_from_mask(sel)
        record[f"{selector}_scores"] = s.numpy()
        record[f"{selector}_selected"] = sel.numpy()
        record[f"{selector}_indices"] = i.numpy()
        record[f"{selector}_counts"] = c.numpy()
    np.savez_compressed(HERE / "selectors_l385.npz", **record)
    # Case 4: the rescue tails (kernels.py:233-309) of fp_v1_rescue / _v2, L=1153 (10 blocks, the
    # last with one row), on a random protected selection with narrow protection so tiles have
    # tails. O is stored on every 9th row (fp32 outputs are large), the LSE on all rows.
    seed, length, heads, kv_heads = 29, 1153, 4, 2
    q, k, v = inputs(seed, length, heads, kv_heads)
    q32, k32, v32 = q.float(), k.float(), v.float()
    blocks = 10
    g = torch.Generator().manual_seed(seed)
    selected = kernels.protected_selection(torch.rand(1, blocks, blocks, heads, generator=g), 0.6, 1, 1, 1)
    record = {"seed": seed, "length": length, "heads": heads, "kv_heads": kv_heads,
              "digest": synthetic.tensor_digest(q, k, v), "selected": selected.numpy(),
              "rows": np.arange(0, length, 9)}
    for name, remainder in (("rescue", False), ("rescue_v2", True)):
        o, lse = kernels.rescue_tail(q32, k32, v32, selected, SCALE, chunk_tiles=3, remainder=remainder)
        record[f"{name}_out_rows"] = o[:, ::9].numpy()
        record[f"{name}_lse"] = lse.numpy()
    np.savez_compressed(HERE / "rescue_l1153.npz", **record)

    # Case 5: head dim 256, 16 query heads over 4 KV heads (check_qwen35_math.py:93-185): V1
    # routing at L=1025 (9 blocks, the last with one row) and the exact path at L=385, all
    # causal blocks and a fixed mask. O is stored on every 8th row of heads 0, 5, 10, 15.
    q35 = load_qwen35(root)
    scale256 = 256 ** -0.5
    seed, length, heads, kv_heads = 35, 1025, 16, 4
    q, k, v = inputs(seed, length, heads, kv_heads, 256)
    q32, k32 = q.float(), k.float()
    mean32 = ref_block_mean(upstream, k32)
    torch.testing.assert_close(mean32, q35.mean_reference(k32), atol=1e-6, rtol=1e-6)
    mk = mean32.to(torch.bfloat16)
    scores = ref_v1_scores(upstream, q32, mk.float(), scale256)
    # The reference's own gate (check_qwen35_math.py:117-124).
    torch.testing.assert_close(scores, q35.score_reference(q32, mk.float(), scale256), atol=3e-4, rtol=0.008)
    idx08, cnt08 = deal(upstream, scores, 0.08)
    idx_p4, cnt_p4 = deal(upstream, scores.square().square(), 0.8)
    ref_i, ref_c = q35.selection_reference(scores.square().square(), 0.8)
    assert torch.equal(idx_p4, ref_i) and torch.equal(cnt_p4, ref_c)
    record = {"seed": seed, "length": length, "heads": heads, "kv_heads": kv_heads, "head_dim": 256,
              "digest": synthetic.tensor_digest(q, k, v),
              "block_mean_fp32": mean32.numpy(), "mean_k_bf16_bits": mk.view(torch.int16).numpy(),
              "scores": scores.numpy(), "indices_a008": idx08.numpy(), "counts_a008": cnt08.numpy(),
              "indices_pow4_a08": idx_p4.numpy(), "counts_pow4_a08": cnt_p4.numpy()}
    np.savez_compressed(HERE / "qwen35_routing_l1025.npz", **record)
    seed, length = 36, 385
    q, k, v = inputs(seed, length, heads, kv_heads, 256)
    q32, k32, v32 = q.float(), k.float(), v.float()
    blocks = 4
    all_selected = kernels.protected_selection(torch.zeros(1, blocks, blocks, heads), 0.0, 2, 4, 2)
    a_idx, a_cnt = kernels.indices_from_mask(all_selected)
    out_all, lse_all = ref_exact(upstream, q32, k32, v32, a_idx, a_cnt, scale256)
    dense_o, dense_lse = q35.dense_reference(q32, k32, v32, scale256)
    torch.testing.assert_close(out_all, dense_o, atol=1e-5, rtol=1e-5)
    torch.testing.assert_close(lse_all, dense_lse, atol=1e-5, rtol=1e-5)
    selected = all_selected.clone()
    selected[:, 3, 1, ::2] = False
    selected[:, 3, 0, 1::4] = False
    selected[:, 2, 0, 3::4] = False
    f_idx, f_cnt = kernels.indices_from_mask(selected)
    out_fixed, lse_fixed = ref_exact(upstream, q32, k32, v32, f_idx, f_cnt, scale256)
    keep_heads = [0, 5, 10, 15]
    np.savez_compressed(
        HERE / "qwen35_exact_l385.npz",
        seed=seed, length=length, heads=heads, kv_heads=kv_heads, head_dim=256,
        digest=synthetic.tensor_digest(q, k, v), rows=np.arange(0, length, 8), out_heads=np.array(keep_heads),
        lse_all=lse_all.numpy(), out_all_rows=out_all[:, ::8][:, :, keep_heads].numpy(),
        selected_fixed=selected.numpy(), indices_fixed=f_idx.numpy(), counts_fixed=f_cnt.numpy(),
        lse_fixed=lse_fixed.numpy(), out_fixed_rows=out_fixed[:, ::8][:, :, keep_heads].numpy(),
    )

    # Case 6: head dim 256 for the mean-corrected methods and the rescue tails, L=1153 (10 blocks,
    # the last with one row), 8 query heads over 2 KV heads: the reference's descriptors, mean
    # tail and merge, its three selectors with their protected selection, and both rescue tails.
    seed, length, heads, kv_heads = 49, 1153, 8, 2
    q, k, v = inputs(seed, length, heads, kv_heads, 256)
    q32, k32, v32 = q.float(), k.float(), v.float()
    blocks = 10
    desc = kernels.block_descriptors(k32, v32)
    g = torch.Generator().manual_seed(seed)
    selected = kernels.protected_selection(torch.rand(1, blocks, blocks, heads, generator=g), 0.6, 1, 1, 1)
    m_out, m_lse = kernels.mean_tail(q32, desc, selected, scale256)
    record = {"seed": seed, "length": length, "heads": heads, "kv_heads": kv_heads, "head_dim": 256,
              "digest": synthetic.tensor_digest(q, k, v), "selected": selected.numpy(), "rows": np.arange(0, length, 9),
              "out_heads": np.array([0, 3, 6]),
              "desc_mean_k": desc.mean_k.numpy(), "desc_var_k": desc.var_k.numpy(),
              "desc_mean_v": desc.mean_v.numpy(), "desc_sigma_v": desc.sigma_v.numpy(),
              "mean_lse": m_lse.numpy(), "mean_out_rows": m_out[:, ::9][:, :, [0, 3, 6]].numpy()}
    for selector in ("mean_balanced", "cgf_mean", "dispersion_mean"):
        sc = kernels.selector_scores(q32, desc, scale256, selector, chunk_tiles=2)
        record[f"{selector}_scores"] = sc.numpy()
        record[f"{selector}_selected"] = kernels.protected_selection(sc, 0.08, 2, 4, 2).numpy()
    for name, remainder in (("rescue", False), ("rescue_v2", True)):
        o, lse = kernels.rescue_tail(q32, k32, v32, selected, scale256, chunk_tiles=3, remainder=remainder)
        record[f"{name}_out_rows"] = o[:, ::9][:, :, [0, 3, 6]].numpy()
        record[f"{name}_lse"] = lse.numpy()
    np.savez_compressed(HERE / "qwen35_tails_l1153.npz", **record)

    # Case 7: edge lengths, L = 1 (one block of one row) and L = 129 (two blocks, the last with one
    # row), 4 query heads over 2 KV heads: V1 block mean, scores and selection, the exact path over
    # every causal block, and the mean tail and merge of a selection with one unselected block.
    record = {}
    for length in (1, 129):
        seed = 60 + length
        q, k, v = inputs(seed, length, 4, 2)
        q32, k32, v32 = q.float(), k.float(), v.float()
        blocks = (length + 127) // 128
        mean32 = ref_block_mean(upstream, k32)
        mk = mean32.to(torch.bfloat16)
        scores = ref_v1_scores(upstream, q32, mk.float())
        idx, cnt = deal(upstream, scores, 0.08)
        every = kernels.protected_selection(torch.zeros(1, blocks, blocks, 4), 0.0, 2, 4, 2)
        a_idx, a_cnt = kernels.indices_from_mask(every)
        out_all, lse_all = ref_exact(upstream, q32, k32, v32, a_idx, a_cnt)
        selected = every.clone()
        if blocks > 1:
            selected[:, 1, 0, ::2] = False  # heads 0 and 2 of the last tile lose block 0
        desc = kernels.block_descriptors(k32, v32)
        f_idx, f_cnt = kernels.indices_from_mask(selected)
        out_f, lse_f = ref_exact(upstream, q32, k32, v32, f_idx, f_cnt)
        m_out, m_lse = kernels.mean_tail(q32, desc, selected, SCALE)
        merged, merged_lse = kernels.merge_exact_mean(out_f, lse_f, m_out, m_lse)
        tag = f"l{length}"
        record.update({f"{tag}_seed": seed, f"{tag}_digest": synthetic.tensor_digest(q, k, v),
                       f"{tag}_block_mean_fp32": mean32.numpy(), f"{tag}_scores": scores.numpy(),
                       f"{tag}_indices_a008": idx.numpy(), f"{tag}_counts_a008": cnt.numpy(),
                       f"{tag}_out_all": out_all.numpy(), f"{tag}_lse_all": lse_all.numpy(),
                       f"{tag}_selected": selected.numpy(), f"{tag}_merged": merged.numpy(),
                       f"{tag}_merged_lse": merged_lse.numpy()})
    np.savez_compressed(HERE / "edges_l1_l129.npz", **record)
    for name in ("v1_routing_l1089.npz", "exact_mean_l257.npz", "selectors_l385.npz", "rescue_l1153.npz",
                 "qwen35_routing_l1025.npz", "qwen35_exact_l385.npz", "qwen35_tails_l1153.npz",
                 "edges_l1_l129.npz"):
        print(name, (HERE / name).stat().st_size, "bytes")


if __name__ == "__main__":
    main(*sys.argv[1:])
