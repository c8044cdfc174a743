"""Every tensor op of the boundary is a PyTorch custom op (``torch.ops.fpx.*``).

On the CPU: each op's fake implementation gives the reference's output shapes and dtypes
(``kernels.py`` / ``upstream/…`` layouts) for fake CUDA inputs, so ``torch.compile`` and
fake-tensor tracing can place the op without running it. On a GPU: ``torch.library.opcheck``
runs each op for real against its registration (schema, fake implementation, no aliasing of
inputs).
"""

import pytest
import torch
from torch._subclasses.fake_tensor import FakeTensorMode

import exp3_b200.decode  # noqa: F401  (registers the ops)
import exp3_b200.kernels  # noqa: F401
import exp3_b200.ops  # noqa: F401
import exp3_b200.upstream  # noqa: F401

B, L, H, HKV, D = 1, 300, 4, 2, 128
NB = 3


def _inputs(dev):
    bf = dict(dtype=torch.bfloat16, device=dev)
    q, k, v = torch.randn(B, L, H, D, **bf), torch.randn(B, L, HKV, D, **bf), torch.randn(B, L, HKV, D, **bf)
    return q, k, v


def _calls(q, k, v):
    f = torch.ops.fpx
    dev = q.device
    mean_k = f.block_mean_k(k, 128)
    scores = f.v1_scores(q, mean_k, D ** -0.5, 128)
    idx, cnt = f.deal_output_score(scores, 2, 4, 0.08, 2, 0)
    mk, mv, vk, sv, counts = f.block_descriptors(k, v, 128)
    sel = f.protected_selection(scores, 0.08, 2, 4, 2)
    idx2, cnt2 = f.indices_from_mask(sel)
    sel2 = f.mask_from_indices(idx, cnt)
    o, lse = f.exact_attention(q, k, v, idx, cnt, D ** -0.5, 128)
    mo, ml = f.mean_tail(q, mk, mv, counts, sel, D ** -0.5, 128)
    ro, rl = f.rescue_tail(q, k, v, sel, D ** -0.5, 128, True)
    so = f.selector_scores(q, mk, vk, sv, counts, D ** -0.5, "cgf_mean", 128)
    merged, mlse = f.merge_exact_mean(o, lse, mo, ml)
    acct = f.selection_counters(sel, L, 128)
    dec = f.decode_attention(q[:, :1], k, v, D ** -0.5)
    pre = f.prefill_attention(q, k, v, "mean_native", 0.08, D ** -0.5, 2, 4, 2)
    return dict(mean_k=mean_k, scores=scores, idx=idx, cnt=cnt, mk=mk, sv=sv, counts=counts, sel=sel, idx2=idx2,
                cnt2=cnt2, sel2=sel2, o=o, lse=lse, mo=mo, ml=ml, ro=ro, so=so, merged=merged, mlse=mlse,
                acct=acct, dec=dec, pre=pre, dev=dev)


def test_fake_implementations_give_the_reference_layouts():
    with FakeTensorMode():
        r = _calls(*_inputs("cuda"))
    expect = {
        "mean_k": ((B, NB, HKV, D), torch.bfloat16), "scores": ((B, NB, NB, H), torch.float32),
        "idx": ((B, NB, NB, H), torch.int64), "cnt": ((B, NB, H), torch.int32),
        "mk": ((B, NB, HKV, D), torch.float32), "sv": ((B, NB, HKV), torch.float32),
        "counts": ((NB,), torch.int32), "sel": ((B, NB, NB, H), torch.bool),
        "idx2": ((B, NB, NB, H), torch.int64), "cnt2": ((B, NB, H), torch.int32),
        "sel2": ((B, NB, NB, H), torch.bool), "o": ((B, L, H, D), torch.bfloat16),
        "lse": ((B, L, H), torch.float32), "mo": ((B, L, H, D), torch.float32), "ml": ((B, L, H), torch.float32),
        "ro": ((B, L, H, D), torch.float32), "so": ((B, NB, NB, H), torch.float32),
        "merged": ((B, L, H, D), torch.bfloat16), "mlse": ((B, L, H), torch.float32),
        "acct": ((3,), torch.int64), "dec": ((B, 1, H, D), torch.bfloat16), "pre": ((B, L, H, D), torch.bfloat16),
    }
    for name, (shape, dtype) in expect.items():
        assert tuple(r[name].shape) == shape, name
        assert r[name].dtype == dtype, name
        assert r[name].device.type == "cuda", name


@pytest.mark.gpu
def test_opcheck_on_the_device():
    q, k, v = _inputs("cuda")
    f = torch.ops.fpx
    mean_k = f.block_mean_k(k, 128)
    scores = f.v1_scores(q, mean_k, D ** -0.5, 128)
    idx, cnt = f.deal_output_score(scores, 2, 4, 0.08, 2, 0)
    mk, mv, vk, sv, counts = f.block_descriptors(k, v, 128)
    sel = f.protected_selection(scores, 0.08, 2, 4, 2)
    o, lse = f.exact_attention(q, k, v, idx, cnt, D ** -0.5, 128)
    mo, ml = f.mean_tail(q, mk, mv, counts, sel, D ** -0.5, 128)
    cases = [
        (f.block_mean_k, (k, 128)), (f.v1_scores, (q, mean_k, D ** -0.5, 128)),
        (f.deal_output_score, (scores, 2, 4, 0.08, 2, 0)), (f.block_descriptors, (k, v, 128)),
        (f.protected_selection, (scores, 0.08, 2, 4, 2)), (f.indices_from_mask, (sel,)),
        (f.mask_from_indices, (idx, cnt)), (f.exact_attention, (q, k, v, idx, cnt, D ** -0.5, 128)),
        (f.mean_tail, (q, mk, mv, counts, sel, D ** -0.5, 128)),
        (f.rescue_tail, (q, k, v, sel, D ** -0.5, 128, False)),
        (f.selector_scores, (q, mk, vk, sv, counts, D ** -0.5, "dispersion_mean", 128)),
        (f.merge_exact_mean, (o, lse, mo, ml)), (f.selection_counters, (sel, L, 128)),
        (f.decode_attention, (q[:, :1].contiguous(), k, v, D ** -0.5)),
        (f.prefill_attention, (q, k, v, "mean_native", 0.08, D ** -0.5, 2, 4, 2)),
    ]
    for op, args in cases:
        torch.library.opcheck(op, args, test_utils=("test_schema", "test_faketensor"))
