"""Layer-swap surface (no GPU needed): config validation, swap / iterate / restore,
fallback policy, and that the compressed path has no CPU execution."""
import pytest
import torch

pytest.importorskip("transformers")
from transformers import Qwen3_5TextConfig  # noqa: E402
from transformers.models.qwen3_5.modeling_qwen3_5 import Qwen3_5ForCausalLM  # noqa: E402

from butterfly_b200.integrations import qwen_torch as qt  # noqa: E402


def _tiny(layer_types=("full_attention", "full_attention")):
    qt.patch_qwen35_full_attention_decode()
    cfg = Qwen3_5TextConfig(hidden_size=256, num_attention_heads=4, num_key_value_heads=1, head_dim=128,
                            num_hidden_layers=len(layer_types), layer_types=list(layer_types),
                            intermediate_size=256, vocab_size=500, partial_rotary_factor=0.25)
    torch.manual_seed(0)
    return Qwen3_5ForCausalLM(cfg).eval()


@pytest.mark.parametrize("kw", [dict(path="nope"), dict(block_size=0), dict(block_partner_rule="zig"),
                                dict(block_compression="max"), dict(compressed_local_window_tokens=0),
                                dict(max_graph_cache_entries=0), dict(path="block_sparse", strategy="greedy")])
def test_config_validation_matches_reference(kw):
    with pytest.raises(ValueError):
        qt.QwenCUDAButterflyConfig(**kw)


def test_swap_iterate_restore():
    m = _tiny(("full_attention", "linear_attention", "full_attention"))
    assert qt.swap_qwen_attention_with_butterfly_cuda(m, qt.compressed_config()) == [0, 2]
    assert [l.layer_idx for l in qt.iter_qwen_butterfly_layers(m)] == [0, 2]
    assert qt.swap_qwen_attention_with_butterfly_cuda(m, qt.compressed_config()) == [0, 2]  # idempotent
    lay = next(qt.iter_qwen_butterfly_layers(m))
    assert (lay.num_heads, lay.num_key_value_heads, lay.head_dim) == (4, 1, 128)
    assert qt.restore_qwen_dense_attention(m) == [0, 2]
    assert list(qt.iter_qwen_butterfly_layers(m)) == []


def test_only_compressed_path_is_swappable():
    m = _tiny()
    with pytest.raises(ValueError):
        qt.swap_qwen_attention_with_butterfly_cuda(m, qt.QwenCUDAButterflyConfig(path="block_sparse"))
    with pytest.raises(ValueError):
        qt.swap_qwen_attention_with_butterfly_cuda(m)  # reference default path="permute"


def test_training_falls_back_to_stock_attention():
    m = _tiny()
    qt.swap_qwen_attention_with_butterfly_cuda(m, qt.compressed_config())
    m.train()
    ids = torch.randint(0, 500, (1, 40))
    m(input_ids=ids)
    assert all(l.last_profile["reason"] == "training" for l in qt.iter_qwen_butterfly_layers(m))


def test_compressed_path_has_no_cpu_execution():
    m = _tiny()
    qt.swap_qwen_attention_with_butterfly_cuda(m, qt.compressed_config())
    with torch.no_grad(), pytest.raises(ValueError, match="CUDA"):
        m(input_ids=torch.randint(0, 500, (1, 40)))


def test_layout_cache_is_bounded():
    m = _tiny()
    qt.swap_qwen_attention_with_butterfly_cuda(m, qt.compressed_config(max_graph_cache_entries=2))
    lay = next(qt.iter_qwen_butterfly_layers(m))
    for T in (100, 200, 300, 200):
        lay._layout(T)
    assert list(lay._layouts) == [300, 200]


def test_fused_layer_state_folds_norms_and_tracks_weight_loads():
    """fuse_qwen_decoder_layers on CPU: the folded-norm weights are round(W * (1 + g)) and are
    recomputed after an in-place weight load (version counters), not served stale."""
    from butterfly_b200.integrations.qwen_fused import fuse_qwen_decoder_layers, unfuse_qwen_decoder_layers
    m = _tiny()
    m = m.to(torch.bfloat16)
    qt.swap_qwen_attention_with_butterfly_cuda(m, qt.compressed_config())
    assert fuse_qwen_decoder_layers(m) == [0, 1]
    layer = m.model.layers[0]
    st = layer._bna_fused
    assert st.fold_norms  # hidden 256, head_dim 128, intermediate 256: every GEMM epilogue applies
    g = layer.input_layernorm.weight
    with torch.no_grad():
        g.copy_(torch.randn_like(g) * 0.1)
    f1 = st.folded("qkv", g, st.w_qkv)
    assert torch.equal(f1, (st.w_qkv.float() * (1 + g.float())[None]).to(st.w_qkv.dtype))
    assert st.folded("qkv", g, st.w_qkv) is f1  # cached
    with torch.no_grad():  # a weight load into the module (a view of the merged buffer)
        layer.self_attn.fallback.q_proj.weight.mul_(2)
    f2 = st.folded("qkv", g, st.w_qkv)
    assert f2 is not f1
    assert torch.equal(f2, (st.w_qkv.float() * (1 + g.float())[None]).to(st.w_qkv.dtype))
    with torch.no_grad():
        g.zero_()
    assert torch.equal(st.folded("qkv", g, st.w_qkv), st.w_qkv)  # (1 + 0) folds to the weights
    assert unfuse_qwen_decoder_layers(m) == [0, 1]


def test_row_statistics_reused_only_for_the_same_storage_and_version():
    from butterfly_b200.integrations.qwen_fused import _row_stats
    x = torch.randn(2, 3, 256).bfloat16()
    ss = torch.zeros(6, 4)
    x._bna_row_ss = (ss, x.data_ptr(), x._version)
    assert _row_stats(x, 6) is ss
    x.add_(1)  # modified in place after the statistics were written: recomputed (needs the GPU)
    with pytest.raises(ValueError):
        _row_stats(x, 6)
