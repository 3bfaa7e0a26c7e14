"""Layer swap on a tiny random-init Qwen3.5 (all full-attention layers, head_dim 128) on the
GPU: prefill and greedy decode through the swapped model match the same model whose
attention runs the reference's algorithm (oracle/torch_port.py, fp32)."""
import contextlib
import copy

import numpy as np
import pytest
import torch

pytest.importorskip("transformers")
from transformers import DynamicCache, Qwen3_5TextConfig  # noqa: E402
from transformers.models.qwen3_5.modeling_qwen3_5 import Qwen3_5ForCausalLM  # noqa: E402

from butterfly_b200.integrations import qwen_torch as qt  # noqa: E402
from oracle import torch_port  # noqa: E402

pytestmark = pytest.mark.gpu


class _ReferenceAttention:
    """Stand-in for butterfly_b200.attention running the reference algorithm in fp32."""

    @staticmethod
    def butterfly_compressed_attention(q, k, v, *, layout, local_window_tokens, scale=None, **_):
        y = torch_port.prefill(q.float(), k.float(), v.float(), layout.block_neighbors[0].tolist(),
                               block_size=layout.block_size, window=local_window_tokens)
        return y.to(q.dtype)

    @staticmethod
    def butterfly_compressed_attention_active(q, k, v, *, layout, query_positions, local_window_tokens,
                                              scale=None, **_):
        y = torch_port.active(q.float(), k.float(), v.float(), layout.block_neighbors[0].tolist(),
                              query_positions.tolist(), block_size=layout.block_size, window=local_window_tokens)
        return y.to(q.dtype)


@contextlib.contextmanager
def _reference_attention():
    saved = qt._attn
    qt._attn = _ReferenceAttention
    try:
        yield
    finally:
        qt._attn = saved


def _model():
    qt.patch_qwen35_full_attention_decode()
    cfg = Qwen3_5TextConfig(hidden_size=512, num_attention_heads=8, num_key_value_heads=2, head_dim=128,
                            num_hidden_layers=3, layer_types=["full_attention"] * 3, intermediate_size=768,
                            vocab_size=1000, partial_rotary_factor=0.25)
    torch.manual_seed(1)
    m = Qwen3_5ForCausalLM(cfg).eval().to(torch.bfloat16).cuda()
    qt.swap_qwen_attention_with_butterfly_cuda(m, qt.compressed_config())
    return m


def _run(m, ids, steps, cache):
    out = m(input_ids=ids, past_key_values=cache, use_cache=True)
    logits = [out.logits[:, -1].float()]
    cache = out.past_key_values
    tok = out.logits[:, -1].argmax(-1, keepdim=True)
    toks = []
    for _ in range(steps):
        toks.append(int(tok))
        out = m(input_ids=tok, past_key_values=cache, use_cache=True)
        cache = out.past_key_values
        logits.append(out.logits[:, -1].float())
        tok = out.logits[:, -1].argmax(-1, keepdim=True)
    return torch.stack(logits), toks


@torch.no_grad()
def test_prefill_and_decode_match_reference_algorithm():
    m = _model()
    ids = torch.randint(0, 1000, (1, 700), generator=torch.Generator().manual_seed(3)).cuda()
    ours_hf, toks_hf = _run(m, ids, 6, DynamicCache(config=m.config))
    for layer in qt.iter_qwen_butterfly_layers(m):
        assert layer.last_profile["block_sparse_backend"] == "compressed_butterfly_active"
    ours_cc, toks_cc = _run(m, ids, 6, qt.make_compressed_cache(m, DynamicCache(config=m.config)))
    for layer in qt.iter_qwen_butterfly_layers(m):
        assert layer.last_profile["block_sparse_backend"] == "compressed_cache_decode_step"
    with _reference_attention():
        ref, toks_ref = _run(m, ids, 6, DynamicCache(config=m.config))
    scale = float(ref.abs().max())
    e_hf = float((ours_hf - ref).abs().max()) / scale
    e_cc = float((ours_cc - ref).abs().max()) / scale
    assert e_hf < 3e-2 and e_cc < 3e-2, (e_hf, e_cc)
    assert toks_hf[:3] == toks_ref[:3] and toks_cc[:3] == toks_ref[:3]
