"""The full-model path against HF transformers' Qwen2ForCausalLM built from the same weights.

The reference times HF Qwen2 (evaluate.py:323-345) with its backend registered as the sdpa
attention (attention.py:57). Here a small Qwen2 (head_dim 128, GQA 2:1) is run (a) by the
HF modules with torch's own sdpa for method "dense", and (b) by the HF modules with this
package's AttentionBackend for "mean_native", and compared with exp3_b200.model on the last
token's logits and on a short greedy decode.
"""

import pytest
import torch

from exp3_b200.attention import AttentionBackend
from exp3_b200.model import AttentionSettings, Qwen2Config, Qwen2Model

pytestmark = pytest.mark.gpu
CFG = Qwen2Config(vocab_size=512, hidden_size=512, intermediate_size=1024, num_hidden_layers=2,
                  num_attention_heads=4, num_key_value_heads=2)


def hf_model(mine: Qwen2Model):
    from transformers import Qwen2Config as HFConfig, Qwen2ForCausalLM
    cfg = HFConfig(vocab_size=CFG.vocab_size, hidden_size=CFG.hidden_size, intermediate_size=CFG.intermediate_size,
                   num_hidden_layers=CFG.num_hidden_layers, num_attention_heads=CFG.num_attention_heads,
                   num_key_value_heads=CFG.num_key_value_heads, max_position_embeddings=8192,
                   rope_theta=CFG.rope_theta, rms_norm_eps=CFG.rms_norm_eps, tie_word_embeddings=False,
                   attn_implementation="sdpa")
    hf = Qwen2ForCausalLM(cfg).to(torch.bfloat16).cuda().eval()
    with torch.no_grad():
        hf.model.embed_tokens.weight.copy_(mine.embed)
        hf.lm_head.weight.copy_(mine.lm_head)
        for lw, layer in zip(mine.layers, hf.model.layers):
            f = lw.full
            a, m = layer.self_attn, layer.mlp
            a.q_proj.weight.copy_(f["wq"]), a.q_proj.bias.copy_(f["bq"])
            a.k_proj.weight.copy_(f["wk"]), a.k_proj.bias.copy_(f["bk"])
            a.v_proj.weight.copy_(f["wv"]), a.v_proj.bias.copy_(f["bv"])
            a.o_proj.weight.copy_(f["wo"])
            m.gate_proj.weight.copy_(f["wg"]), m.up_proj.weight.copy_(f["wu"]), m.down_proj.weight.copy_(f["wd"])
    return hf


def close(a, b, rel=3e-2):
    err = (a - b).abs().max().item()
    scale = b.abs().max().item()
    cos = torch.nn.functional.cosine_similarity(a.flatten(), b.flatten(), dim=0).item()
    assert err <= rel * scale + 1e-3 and cos > 0.999, (err, scale, cos)


def test_prefill_and_decode_match_hf_dense():
    from transformers.integrations.sdpa_attention import sdpa_attention_forward
    from transformers.modeling_utils import ALL_ATTENTION_FUNCTIONS
    ALL_ATTENTION_FUNCTIONS["sdpa"] = sdpa_attention_forward  # torch's own attention in the HF model
    mine = Qwen2Model(CFG, seed=3, keep_full=True, attention=AttentionSettings("dense"))
    hf = hf_model(mine)
    ids = torch.randint(0, CFG.vocab_size, (777,), generator=torch.Generator().manual_seed(4)).cuda()
    with torch.inference_mode():
        ref = hf(input_ids=ids[None], use_cache=True, logits_to_keep=1).logits[0, -1].float()
        mine.prefill(ids, max_new_tokens=4)
        mine_logits = mine._forward(ids, 0, decoding=False)
        close(mine_logits, ref)
        # greedy decode steps on the cache (evaluate.py:384-400), each against HF over the same prefix
        seq = ids.tolist()
        token = int(mine_logits.argmax())
        for _ in range(3):
            step = mine._forward(torch.tensor([token], device="cuda"), mine.length, decoding=True)
            mine.length += 1
            seq.append(token)
            ref_step = hf(input_ids=torch.tensor([seq], device="cuda"), logits_to_keep=1).logits[0, -1].float()
            close(step, ref_step)
            token = int(step.argmax())


def test_prefill_matches_hf_with_backend_mean_native():
    backend = AttentionBackend(alpha=0.08)  # registers itself as HF's sdpa, like attention.py:57
    backend.configure("mean_native")
    mine = Qwen2Model(CFG, seed=5, keep_full=True, attention=AttentionSettings("mean_native", 0.08))
    hf = hf_model(mine)
    ids = torch.randint(0, CFG.vocab_size, (1500,), generator=torch.Generator().manual_seed(6)).cuda()
    with torch.inference_mode():
        ref = hf(input_ids=ids[None], use_cache=True, logits_to_keep=1).logits[0, -1].float()
        mine.prefill(ids)
        out = mine._forward(ids, 0, decoding=False)
    close(out, ref)


def test_graph_decode_matches_eager_decode():
    """decode_graph (each step one CUDA-graph replay, position and key count on the device)
    yields the same greedy tokens as decode_step."""
    ids = torch.randint(0, CFG.vocab_size, (600,), generator=torch.Generator().manual_seed(9)).cuda()
    settings = AttentionSettings("mean_native", 0.08)
    eager_model = Qwen2Model(CFG, seed=11, attention=settings)
    graph_model = Qwen2Model(CFG, seed=11, attention=settings)
    with torch.inference_mode():
        tokens = [eager_model.prefill(ids, max_new_tokens=8)]
        for _ in range(7):
            tokens.append(eager_model.decode_step(tokens[-1]))
        first = graph_model.prefill(ids, max_new_tokens=8)
        graph = graph_model.decode_graph(first, 8)
    assert torch.equal(torch.stack(tokens), graph)
    assert graph_model.length == eager_model.length == 607
