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
