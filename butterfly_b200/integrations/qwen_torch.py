"""Qwen3.5 layer swap onto the B200 compressed Butterfly kernels.

Mirrors the reference's ``bna/integrations/qwen_torch.py`` surface for the compressed
path (``path="block_sparse"``, ``block_compression="mean"``):
  QwenCUDAButterflyConfig                     :253-351  (same fields, defaults, validation)
  extract_qkv_from_qwen_attention             :535-573
  QwenCUDAButterflyAttention                  :576-1621 (fallback policy :1187-1219,
                                                         prefill :1461-1470, decode :1417-1427,
                                                         output gate + o_proj :1585-1591)
  swap_qwen_attention_with_butterfly_cuda     :1652-1691
  restore_qwen_dense_attention                :1624-1641
  iter_qwen_butterfly_layers                  :1644-1649
The other reference paths (permute / sparse / flex / Triton) are not part of this package;
a config selecting them is rejected when layers are swapped.

Decode has two modes.  With an ordinary HF cache the module follows the reference exactly:
the full K/V history is kept by HF and every step runs the active-row kernel over it
(O(T) summary recompute per step, as the reference).  With a ``CompressedButterflyCache``
(see ``make_compressed_cache``) each swapped layer keeps the two-pool cache instead and a
decode step is one fused append + block-close + attention launch.
"""
from __future__ import annotations

import contextlib
import copy
import importlib
import math
import time
from collections import OrderedDict
from dataclasses import dataclass
from functools import lru_cache
from typing import Any, Dict, Iterable, Literal, Optional, Sequence

import torch
import torch.nn as nn

from .. import attention as _attn
from .. import glue
from ..cache import CompressedKVCache
from ..topology import build_block_butterfly_layout


@dataclass
class QwenCUDAButterflyConfig:
    """Configuration of the Butterfly overlay (field names and defaults as the reference)."""

    path: str = "permute"
    strategy: str = "random"
    window: int = 64
    landmark_stride: Optional[int] = 64
    num_cycles: int = 1
    edge_disjoint: bool = True
    enforce_hamiltonian: bool = True
    regular_num_clusters: int = 8
    seed: int = 0
    routing_dim: Optional[int] = None
    edge_bias: bool = False
    window_drop: float = 0.0
    compiled_graph_dir: Optional[str] = None
    engine: str = "auto"
    dense_fallback_q_len: int = 1
    fallback_on_output_attentions: bool = True
    fallback_on_mask: bool = True
    compute_graph_metrics: bool = False
    max_graph_cache_entries: int = 1
    sparse_query_chunk_size: int = 0
    sparse_kv_head_chunk_size: int = 0
    sparse_degree_chunk_size: int = 0
    sparse_chunk_temp_budget_mib: float = 160.0
    sparse_compute_dtype: str = "auto"
    sparse_precomputed_backend: str = "auto"
    sparse_trace_dir: Optional[str] = None
    sparse_trace_max_per_layer: int = 0
    sparse_trace_layer_indices: Optional[tuple[int, ...]] = None
    block_size: int = 128
    block_local_window_blocks: int = 1
    block_partner_count: int = 1
    block_sink_blocks: int = 1
    block_partner_rule: str = "xor"
    block_chunk_size: int = 0
    block_compression: Literal["none", "mean"] = "none"
    compressed_local_window_tokens: int = 128

    def __post_init__(self) -> None:
        if self.path not in {"permute", "sparse", "block_sparse"}:
            raise ValueError(f"Unsupported Butterfly path: {self.path!r}")
        if self.strategy not in {"random", "regular_partition", "greedy", "online_insertion"}:
            raise ValueError(f"Unsupported Butterfly strategy: {self.strategy!r}")
        if self.path == "block_sparse" and self.strategy in {"greedy", "online_insertion"}:
            raise ValueError("block_sparse currently supports only static strategies ('random', 'regular_partition')")
        if int(self.window) < 0:
            raise ValueError("window must be >= 0")
        if int(self.num_cycles) <= 0:
            raise ValueError("num_cycles must be > 0")
        if int(self.block_size) <= 0:
            raise ValueError("block_size must be > 0")
        if int(self.block_local_window_blocks) < 0:
            raise ValueError("block_local_window_blocks must be >= 0")
        if int(self.block_partner_count) < 0:
            raise ValueError("block_partner_count must be >= 0")
        if int(self.block_sink_blocks) < 0:
            raise ValueError("block_sink_blocks must be >= 0")
        if self.block_partner_rule not in {"xor", "bit_reversal", "benes", "causal_shift"}:
            raise ValueError(f"Unsupported block_partner_rule: {self.block_partner_rule!r}")
        if self.block_compression not in {"none", "mean"}:
            raise ValueError(f"Unsupported block_compression: {self.block_compression!r}")
        if int(self.compressed_local_window_tokens) <= 0:
            raise ValueError("compressed_local_window_tokens must be > 0")
        if int(self.dense_fallback_q_len) < 0:
            raise ValueError("dense_fallback_q_len must be >= 0")
        if int(self.max_graph_cache_entries) <= 0:
            raise ValueError("max_graph_cache_entries must be > 0")
        if self.sparse_trace_layer_indices is not None:
            self.sparse_trace_layer_indices = tuple(sorted({int(i) for i in self.sparse_trace_layer_indices}))

    def is_compressed_path(self) -> bool:
        return self.path == "block_sparse" and self.block_compression == "mean"


def compressed_config(**overrides) -> QwenCUDAButterflyConfig:
    """The configuration of the reference's compressed-Butterfly runs (bench ``--path
    compressed_butterfly``: block_sparse, mean compression, causal_shift, window 64)."""
    base = dict(path="block_sparse", strategy="random", block_compression="mean",
                block_partner_rule="causal_shift", compressed_local_window_tokens=64, block_size=128,
                block_local_window_blocks=1, block_partner_count=1, block_sink_blocks=1, engine="auto")
    base.update(overrides)
    return QwenCUDAButterflyConfig(**base)


# ----------------------------------------------------------------------------- helpers
def _has_required_qwen_attention_attrs(module: nn.Module) -> bool:
    return all(hasattr(module, n) for n in ("q_proj", "k_proj", "v_proj", "o_proj", "head_dim"))


_ROTARY_MODULES = (
    "transformers.models.qwen3_5_moe.modeling_qwen3_5_moe",
    "transformers.models.qwen3_5.modeling_qwen3_5",
)


@lru_cache(maxsize=None)
def _load_rotary(module_name: str):
    fn = getattr(importlib.import_module(module_name), "apply_rotary_pos_emb", None)
    if fn is None:
        raise AttributeError(f"`apply_rotary_pos_emb` not found in {module_name}")
    return fn


def _resolve_rotary(attn: nn.Module):
    errors = []
    for name in (attn.__class__.__module__,) + _ROTARY_MODULES:
        try:
            return _load_rotary(name)
        except Exception as exc:  # noqa: BLE001 - collect and report every candidate
            errors.append(f"{name}: {exc}")
    raise ImportError("Could not resolve a Qwen rotary helper: " + "; ".join(errors))


def _get_decoder_with_layers(model: nn.Module) -> nn.Module:
    if hasattr(model, "get_decoder"):
        dec = model.get_decoder()
        if hasattr(dec, "layers"):
            return dec
    for path in (("model", "language_model"), ("model",), ("language_model",), ()):
        obj = model
        for p in path:
            obj = getattr(obj, p, None)
            if obj is None:
                break
        if obj is not None and hasattr(obj, "layers"):
            return obj
    raise ValueError("Could not find a decoder with `.layers` on the supplied model.")


def _cache_seq_len(past_key_values: Optional[Any], layer_idx: Optional[int]) -> int:
    if past_key_values is None or layer_idx is None:
        return 0
    getter = getattr(past_key_values, "get_seq_length", None)
    if getter is None:
        return 0
    try:
        return int(getter(layer_idx))
    except TypeError:
        try:
            return int(getter())
        except Exception:
            return 0
    except Exception:
        return 0


def _is_standard_causal_mask(attention_mask: Optional[torch.Tensor], *, q_len: int, k_len: int) -> bool:
    """Same acceptance test as the reference (qwen_torch.py:495-532)."""
    if attention_mask is None:
        return True
    if attention_mask.dim() == 2:
        return bool(torch.all(attention_mask == 1))
    if attention_mask.dim() != 4:
        return False
    if int(attention_mask.shape[-2]) != q_len or int(attention_mask.shape[-1]) != k_len:
        return False
    if int(attention_mask.shape[1]) != 1 or q_len != k_len or not attention_mask.is_floating_point():
        return False
    min_dtype = torch.finfo(attention_mask.dtype).min
    m = attention_mask
    if q_len > 1:
        if float(m[0, 0, 0, 1]) != min_dtype or float(m[0, 0, 1, 0]) != 0.0:
            return False
        if float(m[0, 0, q_len - 1, 0]) != 0.0 or float(m[0, 0, 0, q_len - 1]) != min_dtype:
            return False
    return bool(torch.all(torch.diagonal(m[0, 0]) == 0))


def extract_qkv_from_qwen_attention(attn: nn.Module, hidden_states: torch.Tensor,
                                    position_embeddings: tuple[torch.Tensor, torch.Tensor], *,
                                    past_key_values: Optional[Any] = None,
                                    cache_position: Optional[torch.LongTensor] = None):
    """(query, key, value, gate) of a Qwen3.5 attention module, as the reference (:535-573):
    gated q_proj split, q/k RMSNorm, RoPE, HF cache update when a cache is given.
    Returns [B, H, T, dh] transposed views of token-major storage."""
    input_shape = hidden_states.shape[:-1]
    hidden_shape = (*input_shape, -1, attn.head_dim)
    rope = _resolve_rotary(attn)
    q, gate = torch.chunk(attn.q_proj(hidden_states).view(*input_shape, -1, attn.head_dim * 2), 2, dim=-1)
    gate = gate.reshape(*input_shape, -1)
    q = attn.q_norm(q.view(hidden_shape)).transpose(1, 2)
    k = attn.k_norm(attn.k_proj(hidden_states).view(hidden_shape)).transpose(1, 2)
    v = attn.v_proj(hidden_states).view(hidden_shape).transpose(1, 2)
    cos, sin = position_embeddings
    q, k = rope(q, k, cos, sin)
    if past_key_values is not None:
        layer_idx = getattr(attn, "layer_idx", None)
        if layer_idx is None:
            raise ValueError("Attention module missing `layer_idx`; cannot update cache.")
        k, v = past_key_values.update(k, v, layer_idx)
    return q, k, v, gate


# ----------------------------------------------------------------------------- cache adapter
class CompressedButterflyCache:
    """Per-layer two-pool caches for the swapped layers, wrapped around the model's own cache.

    Swapped full-attention layers keep their K/V in a ``CompressedKVCache`` (tail ring +
    block-summary pool); every other call (linear-attention layers, mask helpers) goes to
    the wrapped HF cache unchanged.  ``get_seq_length(layer_idx)`` answers for swapped
    layers from their own offset.
    """

    def __init__(self, base: Any, layer_indices: Iterable[int], *, block_size: int, local_window_tokens: int,
                 max_kv_size: Optional[int] = None, max_chunk_size: int = 512):
        object.__setattr__(self, "_base", base)
        object.__setattr__(self, "compressed", {
            int(i): CompressedKVCache(block_size=block_size, local_window_tokens=local_window_tokens,
                                      max_kv_size=max_kv_size, max_chunk_size=max_chunk_size)
            for i in layer_indices})

    def __getattr__(self, name):
        return getattr(object.__getattribute__(self, "_base"), name)

    def __setattr__(self, name, value):
        setattr(object.__getattribute__(self, "_base"), name, value)

    def get_seq_length(self, layer_idx: int = 0, *args, **kwargs) -> int:
        comp = object.__getattribute__(self, "compressed")
        if int(layer_idx) in comp:
            return comp[int(layer_idx)].size()
        base = object.__getattribute__(self, "_base")
        if base is None:
            return 0
        return int(base.get_seq_length(layer_idx, *args, **kwargs))

    @property
    def nbytes(self) -> int:
        """Retained bytes of the swapped layers' two-pool caches (valid slices)."""
        return sum(c.nbytes for c in object.__getattribute__(self, "compressed").values())


def make_compressed_cache(model: nn.Module, base_cache: Any = None, *, max_kv_size: Optional[int] = None,
                          max_chunk_size: int = 512) -> CompressedButterflyCache:
    """Two-pool caches for every swapped layer of ``model`` (call after the swap)."""
    layers = list(iter_qwen_butterfly_layers(model))
    if not layers:
        raise ValueError("model has no swapped Butterfly layers")
    cfg = layers[0].cfg
    return CompressedButterflyCache(base_cache, [l.layer_idx for l in layers], block_size=cfg.block_size,
                                    local_window_tokens=cfg.compressed_local_window_tokens,
                                    max_kv_size=max_kv_size, max_chunk_size=max_chunk_size)


class GraphedGreedyDecode:
    """A fixed number of greedy decode steps of a swapped model, captured once in a CUDA graph.

    Every swapped layer's decode step is one fused append + block-close + attention launch
    with host-side cache counters, so a run of ``steps`` tokens from a given cache state is
    a static sequence of launches: it is recorded once and replayed.  Construction runs the
    steps once eagerly on the capture stream (library warm-up; ``eager_tokens`` keeps the
    tokens it produced), puts the two-pool counters back, and captures the same steps.
    ``replay()`` re-runs them from the post-prefill state: each replay rewrites the same
    ring slots and summary slots with the same values, so replays are repeatable.  After
    construction the cache counters stand at the end of the captured steps.

    ``first_token`` [B,1] (device, int64) seeds step 0; ``tokens`` [B,steps] receives the
    greedy tokens of each replay and ``logits`` [steps,B,vocab] their logits.
    """

    @torch.no_grad()
    def __init__(self, model: nn.Module, cache: "CompressedButterflyCache", first_token: torch.Tensor, steps: int):
        comp = cache.compressed
        self.steps = int(steps)
        self.input = first_token.detach().clone()
        B = int(self.input.shape[0])
        dev = self.input.device
        self.tokens = torch.empty((B, self.steps), dtype=torch.int64, device=dev)
        saved = {i: (c.offset, c.summary_offset, c.summary_count, c.tail_size) for i, c in comp.items()}
        logits = []

        def run():
            logits.clear()
            tok = self.input
            for i in range(self.steps):
                out = model(input_ids=tok, past_key_values=cache, use_cache=True)
                lg = out.logits[:, -1]
                tok = lg.argmax(-1, keepdim=True)
                self.tokens[:, i:i + 1].copy_(tok)
                logits.append(lg)

        def restore():
            for i, c in comp.items():
                c.offset, c.summary_offset, c.summary_count, c.tail_size = saved[i]

        stream = torch.cuda.Stream(device=dev)
        stream.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(stream):
            run()
        torch.cuda.current_stream(dev).wait_stream(stream)
        torch.cuda.synchronize(dev)
        self.eager_tokens = self.tokens.clone()
        self.eager_logits = torch.stack(logits).clone()
        restore()
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph, stream=stream, capture_error_mode="thread_local"):
            run()
            self.logits = torch.stack(logits)
        torch.cuda.synchronize(dev)

    def replay(self) -> None:
        self.graph.replay()


# ----------------------------------------------------------------------------- attention module
class QwenCUDAButterflyAttention(nn.Module):
    """Wrap a stock Qwen3.5 full-attention layer with compressed Butterfly attention."""

    def __init__(self, fallback_attention: nn.Module, cfg: QwenCUDAButterflyConfig):
        super().__init__()
        if not _has_required_qwen_attention_attrs(fallback_attention):
            raise TypeError("fallback_attention does not look like a Qwen3.5 attention module. "
                            "Expected q_proj/k_proj/v_proj/o_proj and head_dim.")
        self.fallback = fallback_attention
        self.cfg = copy.deepcopy(cfg)
        self.config = getattr(fallback_attention, "config", None)
        self.layer_idx = getattr(fallback_attention, "layer_idx", None)
        self.head_dim = int(getattr(fallback_attention, "head_dim"))
        self.num_key_value_groups = int(getattr(fallback_attention, "num_key_value_groups", 1))
        self.scaling = float(getattr(fallback_attention, "scaling", self.head_dim ** -0.5))
        self.is_causal = getattr(fallback_attention, "is_causal", True)
        # q_proj emits query and gate: divide by 2 * head_dim
        self.num_heads = fallback_attention.q_proj.out_features // (self.head_dim * 2)
        self.num_key_value_heads = fallback_attention.k_proj.out_features // self.head_dim
        self.hidden_size = fallback_attention.q_proj.in_features
        self._layouts: "OrderedDict[int, Any]" = OrderedDict()
        self.last_profile: Dict[str, Any] = {}
        self._shard: Optional["SequenceShard"] = None

    # -- layouts (reference _get_or_build_cache :1039-1058, keyed by sequence length) --
    def _layout(self, seq_len: int):
        lay = self._layouts.get(int(seq_len))
        if lay is not None:
            self._layouts.move_to_end(int(seq_len))
            return lay, True
        lay = build_block_butterfly_layout(
            seq_len=int(seq_len), block_size=int(self.cfg.block_size),
            num_key_value_heads=int(self.num_key_value_heads), num_key_value_groups=int(self.num_key_value_groups),
            layer_idx=0 if self.layer_idx is None else int(self.layer_idx),
            local_window_blocks=int(self.cfg.block_local_window_blocks), sink_count=int(self.cfg.block_sink_blocks),
            partner_count=int(self.cfg.block_partner_count), partner_rule=self.cfg.block_partner_rule)
        self._layouts[int(seq_len)] = lay
        while len(self._layouts) > int(self.cfg.max_graph_cache_entries):
            self._layouts.popitem(last=False)
        return lay, False

    def _fallback_reason(self, *, attention_mask, q_len: int, k_len_after: int, output_attentions: bool,
                         compressed_cache: bool) -> Optional[str]:
        """Reference policy (:1187-1219) for the compressed path."""
        if self.training:
            return "training"
        cached = k_len_after > q_len
        if self.layer_idx is None:
            return "missing_layer_idx"
        if self.cfg.fallback_on_output_attentions and output_attentions:
            return "output_attentions"
        if q_len <= int(self.cfg.dense_fallback_q_len) and not cached and not compressed_cache:
            return "short_query"
        if self.cfg.fallback_on_mask and not compressed_cache and not cached and not _is_standard_causal_mask(
                attention_mask, q_len=q_len, k_len=k_len_after):
            return "attention_mask"
        return None

    def plan(self, q_len: int, attention_mask, past_key_values, output_attentions: bool = False):
        """(fallback reason or None, this layer's two-pool cache or None, cached length,
        key length after this call) — the routing decision of ``forward``."""
        if self._shard is not None:
            if _cache_seq_len(past_key_values, self.layer_idx) or isinstance(past_key_values, CompressedButterflyCache):
                raise RuntimeError("a sequence-sharded forward is a prefill without a cache (pass use_cache=False)")
            if self.training or (output_attentions and self.cfg.fallback_on_output_attentions):
                raise RuntimeError("a sequence-sharded forward runs only the compressed kernels (eval, no attentions)")
            return None, None, 0, self._shard.total_len
        comp_cache = None
        if isinstance(past_key_values, CompressedButterflyCache):
            comp_cache = past_key_values.compressed.get(int(self.layer_idx)) if self.layer_idx is not None else None
        cache_len = comp_cache.size() if comp_cache is not None else _cache_seq_len(past_key_values, self.layer_idx)
        k_len_after = q_len + cache_len
        reason = self._fallback_reason(attention_mask=attention_mask, q_len=q_len, k_len_after=k_len_after,
                                       output_attentions=output_attentions, compressed_cache=comp_cache is not None)
        if reason is not None and comp_cache is not None:
            raise RuntimeError(f"compressed cache layer {self.layer_idx} cannot fall back to dense attention "
                               f"({reason}): its K/V history lives in the two-pool cache")
        if reason is None and self.head_dim != 128:
            raise ValueError(f"compressed Butterfly kernels need head_dim 128, layer has {self.head_dim}")
        return reason, comp_cache, cache_len, k_len_after

    def attend(self, q, k, v, comp_cache, cache_len: int, k_len_after: int, cache_position=None, qk_prep=None,
               gate=None):
        """Compressed attention of q [B,Hq,Tq,dh] over k/v [B,Hkv,Tk,dh] (HF-cache history
        included, or the new tokens only when ``comp_cache`` holds the history).  Returns
        ([B,Hq,Tq,dh] view of [B,Tq,Hq,dh] storage, backend name, layout-cache hit).
        ``qk_prep`` (a decode step into ``comp_cache`` only): q / k are raw projection rows and
        the step applies the q/k norm and rotary embedding itself (see decode_step).
        ``gate`` [B,Hq,Tq,dh]: return ``out * sigmoid(gate)`` (Qwen3.5's output gate), fused
        into the prefill kernel's store on whole-prompt prefills, a separate launch otherwise."""
        gated = False
        q_len = int(q.shape[2])
        W = int(self.cfg.compressed_local_window_tokens)
        scale = 1.0 / math.sqrt(self.head_dim)  # SDPA's default, as the reference (the module scaling is not passed)
        lay, hit = self._layout(k_len_after)
        if comp_cache is not None:
            if q_len == 1 and cache_len > 0:
                out = comp_cache.decode_step(q, k, v, lay, scale=scale, qk_prep=qk_prep)
                backend = "compressed_cache_decode_step"
            elif cache_len == 0:
                # The prefill's block means are written straight into the cache's summary
                # slots; the cache then takes over the prompt as if fed in max_chunk_size
                # chunks, keeping only its tail rows (no whole-prompt copy, no re-close).
                comp_cache.reserve(k.shape[0], k.shape[1], k.shape[3], k.dtype, k.device)
                slots = comp_cache.summary_slots(lay.num_blocks)
                ks_out, vs_out = slots if slots is not None else (None, None)
                out, _, ks, vs = _attn.prefill_with_summaries(q, k, v, lay, W, scale, False, ks_out, vs_out, gate=gate)
                gated = True
                comp_cache.adopt_prefill(k, v, ks, vs)
                backend = "compressed_prefill+cache_handoff"
            else:
                comp_cache.append(k, v)
                out = comp_cache.attend(q, lay, scale=scale)
                backend = "compressed_cache_chunk"
        elif k_len_after > q_len:
            pos = (cache_position.view(-1) if cache_position is not None
                   else torch.arange(cache_len, cache_len + q_len, device=q.device))
            out = _attn.butterfly_compressed_attention_active(q, k, v, layout=lay, query_positions=pos,
                                                             local_window_tokens=W, scale=scale)
            backend = "compressed_butterfly_active"
        elif gate is not None:
            out = _attn.prefill_with_summaries(q, k, v, lay, W, scale, gate=gate)[0]
            gated = True
            backend = "compressed_butterfly"
        else:
            out = _attn.butterfly_compressed_attention(q, k, v, layout=lay, local_window_tokens=W, scale=scale)
            backend = "compressed_butterfly"
        if gate is not None and not gated:
            B, Hq, Tq, dh = out.shape
            out = glue.gate_sigmoid_mul(out.transpose(1, 2).contiguous(), gate.transpose(1, 2)).view(
                B, Tq, Hq, dh).transpose(1, 2)
        return out, backend, hit

    def attend_sharded(self, q, k_ext, v_ext, halo: int):
        """Sequence-sharded prefill of this rank's queries q [B,Hq,T_local,dh]: k_ext / v_ext
        [B,Hkv,halo+T_local,dh] hold the local keys / values at rows [halo, ...); the block
        means and the previous rank's last ``halo`` rows are exchanged over the shard's
        process group (NCCL all-gathers) and the kernel runs on global positions."""
        from .. import seqshard
        sh = self._shard
        W = int(self.cfg.compressed_local_window_tokens)
        Tl = int(q.shape[2])
        lay, hit = self._layout(sh.total_len)
        seqshard.check_shard(Tl, int(lay.block_size), W, sh.world, lay)
        ops = seqshard.cuda_ops(lay, W, 1.0 / math.sqrt(self.head_dim))
        ks, vs, ka, va, kv_pos0 = seqshard.shard_exchange(k_ext, v_ext, halo, int(lay.block_size), ops, sh.group)
        out = ops.attend(q, ka, va, ks, vs, sh.rank * Tl, kv_pos0, sh.total_len)
        return out, "compressed_sequence_shard", hit

    def _profile(self, q_len, k_len_after, backend, hit, t0, fused=False):
        self.last_profile = {
            "mode": "butterfly", "reason": None, "layer_idx": self.layer_idx, "seq_len": q_len,
            "kv_len": k_len_after, "path": self.cfg.path, "engine": "bna_b200", "strategy": self.cfg.strategy,
            "graph_cache_hit": bool(hit), "block_sparse_backend": backend, "fused_glue": bool(fused),
            "elapsed_ms": float((time.perf_counter() - t0) * 1000.0),
        }

    def forward(self, hidden_states: torch.Tensor, position_embeddings: tuple[torch.Tensor, torch.Tensor],
                attention_mask: Optional[torch.Tensor] = None, past_key_values: Optional[Any] = None,
                cache_position: Optional[torch.LongTensor] = None, **kwargs: Any):
        q_len = int(hidden_states.shape[1])
        reason, comp_cache, cache_len, k_len_after = self.plan(
            q_len, attention_mask, past_key_values, bool(kwargs.get("output_attentions", False)))
        if reason is not None:
            self.last_profile = {"mode": "fallback", "reason": reason, "layer_idx": self.layer_idx,
                                 "seq_len": q_len, "kv_len": k_len_after, "path": self.cfg.path}
            return self.fallback(hidden_states, position_embeddings=position_embeddings,
                                 attention_mask=attention_mask, past_key_values=past_key_values,
                                 cache_position=cache_position, **kwargs)
        t0 = time.perf_counter()
        hf_cache = None if comp_cache is not None or self._shard is not None else past_key_values
        q, k, v, gate = extract_qkv_from_qwen_attention(self.fallback, hidden_states, position_embeddings,
                                                        past_key_values=hf_cache, cache_position=cache_position)
        if self._shard is not None:
            h = int(self.cfg.compressed_local_window_tokens) - 1
            B, Hkv, Tl, dh = k.shape
            k_ext = torch.empty((B, h + Tl, Hkv, dh), device=k.device, dtype=k.dtype).transpose(1, 2)
            v_ext = torch.empty_like(k_ext.transpose(1, 2)).transpose(1, 2)
            k_ext[:, :, h:].copy_(k)
            v_ext[:, :, h:].copy_(v)
            out, backend, hit = self.attend_sharded(q, k_ext, v_ext, h)
        else:
            out, backend, hit = self.attend(q, k, v, comp_cache, cache_len, k_len_after, cache_position)
        input_shape = hidden_states.shape[:-1]
        attn_output = out.transpose(1, 2).reshape(*input_shape, -1)  # storage is already [B, T, Hq, dh]
        attn_output = attn_output * torch.sigmoid(gate)
        attn_output = self.fallback.o_proj(attn_output)
        self._profile(q_len, k_len_after, backend, hit, t0)
        return attn_output, None


@dataclass
class SequenceShard:
    """This process's part of a sequence-sharded prefill: contiguous whole blocks of a
    ``total_len``-token sequence, rank ``rank`` of ``world`` in process group ``group``."""

    group: Any
    rank: int
    world: int
    total_len: int


@contextlib.contextmanager
def sequence_sharded(model: nn.Module, total_len: int, group=None):
    """Run the swapped layers' prefill sequence-sharded across the ranks of ``group``.

    Inside the context every rank calls the model on its own contiguous token shard
    ``input_ids[:, rank*T_local:(rank+1)*T_local]`` with global ``position_ids`` and
    ``use_cache=False``; each swapped layer exchanges only its block means and a W-1-token
    halo of K/V with the other ranks (NCCL all-gathers) and computes exactly the unsharded
    result for its queries.  The last rank holds the next-token logits."""
    import torch.distributed as dist
    world = dist.get_world_size(group) if dist.is_initialized() else 1
    rank = dist.get_rank(group) if dist.is_initialized() else 0
    sh = SequenceShard(group=group, rank=rank, world=world, total_len=int(total_len))
    layers = list(iter_qwen_butterfly_layers(model))
    for l in layers:
        l._shard = sh
    try:
        yield sh
    finally:
        for l in layers:
            l._shard = None


# ----------------------------------------------------------------------------- swap API
def restore_qwen_dense_attention(model: nn.Module) -> list[int]:
    """Remove Butterfly wrappers and restore stock attention in place; returns layer indices."""
    decoder = _get_decoder_with_layers(model)
    restored = []
    for idx, layer in enumerate(decoder.layers):
        attn = getattr(layer, "self_attn", None)
        if isinstance(attn, QwenCUDAButterflyAttention):
            attn._layouts.clear()
            layer.self_attn = attn.fallback
            restored.append(idx)
    return restored


def iter_qwen_butterfly_layers(model: nn.Module) -> Iterable[QwenCUDAButterflyAttention]:
    for layer in _get_decoder_with_layers(model).layers:
        attn = getattr(layer, "self_attn", None)
        if isinstance(attn, QwenCUDAButterflyAttention):
            yield attn


def swap_qwen_attention_with_butterfly_cuda(model: nn.Module, cfg: Optional[QwenCUDAButterflyConfig] = None, *,
                                            layer_indices: Optional[Sequence[int]] = None) -> list[int]:
    """Replace Qwen3.5 full-attention layers with compressed Butterfly wrappers in place."""
    config = copy.deepcopy(cfg) if cfg is not None else QwenCUDAButterflyConfig()
    if not config.is_compressed_path():
        raise ValueError("butterfly_b200 implements the compressed path only: path='block_sparse' with "
                         "block_compression='mean' (see compressed_config())")
    decoder = _get_decoder_with_layers(model)
    selected = None if layer_indices is None else {int(i) for i in layer_indices}
    replaced = []
    for idx, layer in enumerate(decoder.layers):
        if selected is not None and idx not in selected:
            continue
        if getattr(layer, "layer_type", None) != "full_attention":
            continue
        attn = getattr(layer, "self_attn", None)
        if attn is None:
            continue
        if isinstance(attn, QwenCUDAButterflyAttention):
            replaced.append(idx)
            continue
        if not _has_required_qwen_attention_attrs(attn):
            continue
        if getattr(attn, "layer_idx", None) is None:
            setattr(attn, "layer_idx", idx)
        wrapped = QwenCUDAButterflyAttention(attn, config)
        wrapped.train(attn.training)
        layer.self_attn = wrapped
        replaced.append(idx)
    return replaced


swap_qwen_attention_with_wayfinder_cuda = swap_qwen_attention_with_butterfly_cuda

__all__ = [
    "QwenCUDAButterflyConfig", "QwenCUDAButterflyAttention", "CompressedButterflyCache", "GraphedGreedyDecode",
    "SequenceShard", "compressed_config", "sequence_sharded",
    "extract_qkv_from_qwen_attention", "iter_qwen_butterfly_layers", "make_compressed_cache",
    "restore_qwen_dense_attention", "swap_qwen_attention_with_butterfly_cuda",
]


def patch_qwen35_full_attention_decode() -> None:
    """Work around transformers 5.x Qwen3.5 models whose layers are all full attention:
    ``Qwen3_5TextModel._update_linear_attn_mask`` queries ``has_previous_state`` on a cache
    that holds no linear-attention layer and raises.  With no linear-attention layer the
    mask is unused, so the patched method returns the incoming mask in that case and
    defers to the original otherwise.  Idempotent."""
    from transformers.models.qwen3_5 import modeling_qwen3_5 as mq
    cls = mq.Qwen3_5TextModel
    if getattr(cls, "_bna_full_attention_patch", False):
        return
    original = cls._update_linear_attn_mask

    def _patched(self, attention_mask, past_key_values, *args, **kwargs):
        types = getattr(self.config, "layer_types", None) or []
        if types and all(t == "full_attention" for t in types):
            return attention_mask
        return original(self, attention_mask, past_key_values, *args, **kwargs)

    cls._update_linear_attn_mask = _patched
    cls._bna_full_attention_patch = True
