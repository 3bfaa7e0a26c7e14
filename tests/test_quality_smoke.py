"""Quality-smoke comparison (reference scripts/quality_smoke.py:223-262): KL over the
overlapping top-k tokens, overlap, top-1 and greedy agreement.  CPU: the arithmetic on
hand-made distributions.  GPU: one small random-init model, stock vs compressed."""
import math

import pytest
import torch

from butterfly_b200.integrations.quality_smoke import compare, kl_over_overlap, prompt_ids


def _dist(pairs):
    return [{"token_id": t, "logit": 0.0, "log_prob": math.log(p)} for t, p in pairs]


def test_kl_and_agreement_arithmetic():
    p = {1: math.log(0.5), 2: math.log(0.3), 3: math.log(0.2)}
    q = {1: math.log(0.4), 2: math.log(0.4), 4: math.log(0.2)}
    want = 0.5 * math.log(0.5 / 0.4) + 0.3 * math.log(0.3 / 0.4)
    assert abs(kl_over_overlap(p, q) - want) < 1e-12
    assert math.isnan(kl_over_overlap({5: 0.0}, {6: 0.0}))
    stock = {"final_log_softmax_top_k": _dist([(1, 0.5), (2, 0.3), (3, 0.2)]), "decoded_ids": [1, 7, 8, 9]}
    comp = {"final_log_softmax_top_k": _dist([(1, 0.4), (2, 0.4), (4, 0.2)]), "decoded_ids": [1, 7, 0, 9]}
    m = compare(stock, comp)
    assert m["top_k_overlap"] == 2 and m["top_k_total"] == 3 and m["top1_agree"]
    assert not m["greedy_exact_match"] and m["greedy_token_agreement"] == 0.75


def test_prompt_is_deterministic_and_repeats():
    a, b = prompt_ids(1000, 1500), prompt_ids(1000, 1500)
    assert torch.equal(a, b) and a.shape == (1, 1500)
    assert torch.equal(a[0, :512], a[0, 512:1024])


@pytest.mark.gpu
def test_quality_smoke_runs_stock_and_compressed():
    from transformers import Qwen3_5TextConfig
    from transformers.models.qwen3_5.modeling_qwen3_5 import Qwen3_5ForCausalLM

    from butterfly_b200.integrations import qwen_torch as qt
    from butterfly_b200.integrations.quality_smoke import quality_smoke
    cfg = Qwen3_5TextConfig(hidden_size=512, num_attention_heads=8, num_key_value_heads=2, head_dim=128,
                            num_hidden_layers=3, layer_types=["full_attention"] * 3, intermediate_size=1024,
                            vocab_size=1000)
    torch.manual_seed(3)
    m = Qwen3_5ForCausalLM(cfg).eval().to(torch.bfloat16).cuda()
    res = quality_smoke(m, prompt_ids(1000, 4096).cuda(), decode_len=8, top_k=50)
    met = res["metrics"]
    assert met["top_k_total"] == 50 and 0 <= met["top_k_overlap"] <= 50
    assert math.isfinite(met["kl_stock_compressed"]) and math.isfinite(met["kl_compressed_stock"])
    assert len(res["stock"]["decoded_ids"]) == 8 and len(res["compressed"]["decoded_ids"]) == 8
    assert not list(qt.iter_qwen_butterfly_layers(m))  # stock attention restored
