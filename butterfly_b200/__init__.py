"""B200-native compressed Butterfly attention (sm_100a CUDA behind a C ABI).

Drop-in for the reference's ``bna.torch`` compressed-attention functions and its Qwen
layer-swap API; see ``butterfly_b200.attention``, ``butterfly_b200.cache`` and
``butterfly_b200.integrations.qwen_torch``.
"""
from .topology import (BlockHamiltonianLayout, build_block_butterfly_layout, build_block_wayfinder_layout,
                       butterfly_stage_meta, butterfly_width, num_blocks_for_seq_len)
from .attention import (block_mean_summaries, butterfly_compressed_attention,
                        butterfly_compressed_attention_active)

__all__ = [
    "BlockHamiltonianLayout", "build_block_butterfly_layout", "build_block_wayfinder_layout",
    "butterfly_stage_meta", "butterfly_width", "num_blocks_for_seq_len", "block_mean_summaries",
    "butterfly_compressed_attention", "butterfly_compressed_attention_active",
]
