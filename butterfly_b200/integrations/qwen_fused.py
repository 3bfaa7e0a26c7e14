"""Fused decoder-layer glue for Qwen3.5 layers already swapped onto compressed Butterfly.

``swap_qwen_attention_with_butterfly_cuda`` replaces only the attention, as the reference
does; the rest of each decoder layer still runs as transformers' eager ops, which at long
prompts cost several times the GEMMs and the attention together (fp32 RMSNorm chains,
rotary-embedding concatenations, separate sigmoid / SiLU / multiply / residual passes).
``fuse_qwen_decoder_layers`` replaces that glue, per swapped layer, with:

    h   = rmsnorm(x)                                  one kernel   (input_layernorm)
    qkv = h @ [Wq; Wk; Wv]^T, q/k norm + RoPE         one tcgen05 GEMM (q/k/v merged; q_norm/k_norm
                                                      and the partial RoPE in its epilogue)
    y   = attention(q,k,v) * sigmoid(gate)            the path's kernels (whole-prompt prefill: the
                                                      gate is applied in the attention kernel's store;
                                                      otherwise one more kernel)
    a   = y @ Wo^T                                    one GEMM
    x2, h2 = x + a, rmsnorm(x + a)                    one kernel   (residual + post_attention_layernorm)
    act = silu(h2 @ Wg^T) * (h2 @ Wu^T)               one tcgen05 GEMM, SwiGLU in its epilogue
    x2 += act @ Wd^T                                  one GEMM accumulating into x2

For a decode step (one token per sequence, up to 8 sequences) the projections are instead
weight-streaming GEMV kernels with the neighbouring steps fused in: rmsnorm+qkv,
gate+o_proj+residual, rmsnorm+gate/up+SwiGLU, down_proj+residual, and (into a two-pool
cache) the decode step with the q/k norm + RoPE of the new token fused in: five launches
per layer, each overlapping the previous one's tail through programmatic dependent launch.

The projection weights are moved into one buffer per layer ([Wq; Wk; Wv] and [Wg; Wu]) and
the modules' ``weight`` parameters become views of it, so the model's parameters, its
``state_dict`` and the unfused path are unchanged.  Numerics follow the eager layer op by
op except that the MLP's down projection is accumulated onto the residual in fp32 inside
the GEMM (one rounding where the eager layer rounds twice).  A layer whose attention would
fall back to dense attention (training, masks, ``output_attentions``) runs its original
forward.  ``unfuse_qwen_decoder_layers`` restores the original forwards.
"""
from __future__ import annotations

import time
import types
from typing import Any, Optional

import torch
import torch.nn as nn
import torch.nn.functional as F

from .. import glue
from .qwen_torch import QwenCUDAButterflyAttention, _get_decoder_with_layers


def _is_qwen35_norm(mod: nn.Module) -> bool:
    return type(mod).__name__ in ("Qwen3_5RMSNorm", "Qwen3_5MoeRMSNorm") and hasattr(mod, "weight")


def _merge_weights(mods: list[nn.Linear]) -> torch.Tensor:
    """Move the weights of ``mods`` into one [sum(out), in] buffer; each module's weight
    becomes a view (Parameter) of its rows.  Returns the buffer."""
    ws = [m.weight for m in mods]
    buf = torch.cat([w.detach() for w in ws], 0)
    r = 0
    for m, w in zip(mods, ws):
        n = w.shape[0]
        m.weight = nn.Parameter(buf[r:r + n], requires_grad=w.requires_grad)
        r += n
    return buf


class _FusedState:
    def __init__(self, layer: nn.Module):
        attn: QwenCUDAButterflyAttention = layer.self_attn
        src = attn.fallback
        mlp = layer.mlp
        for lin in (src.q_proj, src.k_proj, src.v_proj, src.o_proj, mlp.gate_proj, mlp.up_proj, mlp.down_proj):
            if getattr(lin, "bias", None) is not None:
                raise ValueError("fused glue needs bias-free projections")
        self.attn = attn
        self.w_qkv = _merge_weights([src.q_proj, src.k_proj, src.v_proj])
        self.w_gu = _merge_weights([mlp.gate_proj, mlp.up_proj])
        self.hq, self.hkv, self.dh = attn.num_heads, attn.num_key_value_heads, attn.head_dim
        self.inter = mlp.gate_proj.out_features
        # the tcgen05 gate/up GEMM tiles K by 64 and the intermediate size by 128
        self.gemm_swiglu = mlp.gate_proj.in_features % 64 == 0 and self.inter % 128 == 0
        # and the q/k/v GEMM with the q/k norm + RoPE epilogue: 128-wide heads, N by 256
        self.gemm_qkv = (src.q_proj.in_features % 64 == 0 and self.dh == 128 and
                         int(self.w_qkv.shape[0]) % 256 == 0)
        # and o_proj / down_proj with the residual add in the epilogue: N (hidden) by 256
        hidden = src.o_proj.out_features
        self.gemm_resid = (hidden % 256 == 0 and src.o_proj.in_features % 64 == 0 and self.inter % 64 == 0
                           and mlp.down_proj.out_features == hidden)
        # with all three, the two RMSNorms fold into the GEMMs after them (weights with the norm
        # weight folded in, cached against both tensors' version counters)
        self.fold_norms = self.gemm_qkv and self.gemm_swiglu and self.gemm_resid
        self._folded: dict = {}

    def folded(self, key: str, norm_weight: torch.Tensor, w: torch.Tensor) -> torch.Tensor:
        """w with the Qwen3.5 RMSNorm weight folded into its columns: round(w[:, k] * (1 + g[k])).
        Recomputed whenever either tensor changes in place (a weight load)."""
        ver = (norm_weight.data_ptr(), norm_weight._version, w.data_ptr(), w._version)
        hit = self._folded.get(key)
        if hit is None or hit[0] != ver:
            f = (w.float() * (1.0 + norm_weight.float())[None, :]).to(w.dtype)
            self._folded[key] = (ver, f)
            return f
        return hit[1]


def _row_stats(x: torch.Tensor, rows: int) -> torch.Tensor:
    """Per-row partial sums of squares of the residual stream x: the ones the previous layer's
    down projection wrote (still valid for this storage and version), else computed."""
    t = getattr(x, "_bna_row_ss", None)
    if t is not None and t[1] == x.data_ptr() and t[2] == x._version and int(t[0].shape[0]) == rows:
        return t[0]
    return glue.row_sumsq(x)


def _fused_layer_forward(self, hidden_states: torch.Tensor, position_embeddings=None, attention_mask=None,
                         position_ids=None, past_key_values=None, **kwargs: Any):
    st: _FusedState = self._bna_fused
    attn = st.attn
    B, T, H = hidden_states.shape
    reason, comp_cache, cache_len, k_len_after = attn.plan(
        T, attention_mask, past_key_values, bool(kwargs.get("output_attentions", False)))
    if reason is not None or self.training or hidden_states.dtype not in (torch.bfloat16, torch.float16):
        return type(self).forward(self, hidden_states, position_embeddings=position_embeddings,
                                  attention_mask=attention_mask, position_ids=position_ids,
                                  past_key_values=past_key_values, **kwargs)
    t0 = time.perf_counter()
    src = attn.fallback
    hq, hkv, dh = st.hq, st.hkv, st.dh
    x = hidden_states
    decode = T == 1 and B <= 8 and H % 256 == 0 and st.inter % 256 == 0 and attn._shard is None
    if decode:  # weight-streaming projections with the norms, gate and residual adds fused in
        qkv = glue.gemv_rmsnorm(x.view(B, H), self.input_layernorm.weight, self.input_layernorm.eps,
                                st.w_qkv).view(B, 1, -1)
    cos, sin = position_embeddings
    # whole-prompt / chunk prefill: q/k norm + RoPE in the q/k/v GEMM's epilogue
    prepped = (not decode and attn._shard is None and st.gemm_qkv and int(cos.shape[-1]) % 32 == 0)
    fold = prepped and st.fold_norms
    if fold:  # the input RMSNorm folded into the q/k/v GEMM (row statistics, folded weights)
        qkv = glue.gemm_qkv_norm_rope(x, st.folded("qkv", self.input_layernorm.weight, st.w_qkv), hq, hkv,
                                      src.q_norm.weight, src.k_norm.weight, cos, sin, src.q_norm.eps,
                                      row_ss=_row_stats(x, B * T), norm_eps=self.input_layernorm.eps)
    elif not decode:
        h = glue.rmsnorm(x, self.input_layernorm.weight, self.input_layernorm.eps)
        if prepped:
            qkv = glue.gemm_qkv_norm_rope(h, st.w_qkv, hq, hkv, src.q_norm.weight, src.k_norm.weight, cos, sin,
                                          src.q_norm.eps)
        else:
            qkv = F.linear(h, st.w_qkv)                           # [B,T,2*hq*dh + 2*hkv*dh]
    nq = 2 * hq * dh
    qg = qkv[..., :nq].view(B, T, hq, 2 * dh)                     # per head: query, then gate
    k_raw = qkv[..., nq:nq + hkv * dh].view(B, T, hkv, dh)
    v = qkv[..., nq + hkv * dh:].view(B, T, hkv, dh)
    gated = None  # the gated attention output [B,T,hq*dh] when the gate rode along with attention
    if attn._shard is not None:
        # sequence shard: K and V go straight into buffers whose first W-1 rows receive the
        # previous rank's halo
        hl = int(attn.cfg.compressed_local_window_tokens) - 1
        k_ext = torch.empty((B, hl + T, hkv, dh), device=x.device, dtype=x.dtype)
        v_ext = torch.empty_like(k_ext)
        q, _ = glue.qk_norm_rope(qg[..., :dh], k_raw, src.q_norm.weight, src.k_norm.weight, cos, sin,
                                 src.q_norm.eps, k_out=k_ext[:, hl:], v=v, v_out=v_ext[:, hl:])
        out, backend, hit = attn.attend_sharded(q.transpose(1, 2), k_ext.transpose(1, 2), v_ext.transpose(1, 2), hl)
    elif decode and comp_cache is not None and cache_len > 0:
        # one launch: q/k norm + RoPE of the new token, append, block close and attention
        prep = (src.q_norm.weight, src.k_norm.weight, cos, sin, src.q_norm.eps)
        out, backend, hit = attn.attend(qg[..., :dh].transpose(1, 2), k_raw.transpose(1, 2), v.transpose(1, 2),
                                        comp_cache, cache_len, k_len_after, qk_prep=prep)
    else:
        if prepped:
            q, k = qg[..., :dh], k_raw
        else:
            q, k = glue.qk_norm_rope(qg[..., :dh], k_raw, src.q_norm.weight, src.k_norm.weight, cos, sin,
                                     src.q_norm.eps)
        qt, kt, vt = q.transpose(1, 2), k.transpose(1, 2), v.transpose(1, 2)
        if comp_cache is None and past_key_values is not None:
            kt, vt = past_key_values.update(kt, vt, attn.layer_idx)
        if decode:  # the gate rides along with the o_proj GEMV
            out, backend, hit = attn.attend(qt, kt, vt, comp_cache, cache_len, k_len_after,
                                            kwargs.get("cache_position"))
        else:
            out, backend, hit = attn.attend(qt, kt, vt, comp_cache, cache_len, k_len_after,
                                            kwargs.get("cache_position"), gate=qg[..., dh:].transpose(1, 2))
            gated = out.transpose(1, 2).reshape(B, T, hq * dh)
    if decode:
        x2 = glue.gemv_gated(out.transpose(1, 2).reshape(B, hq, dh), qg[:, 0, :, dh:], src.o_proj.weight,
                             residual=x.view(B, H))
        act = glue.gemv_rmsnorm(x2, self.post_attention_layernorm.weight, self.post_attention_layernorm.eps,
                                st.w_gu, swiglu=True)
        x3 = glue.gemv(act, self.mlp.down_proj.weight, residual=x2)
        attn._profile(T, k_len_after, backend, hit, t0, fused=True)
        return x3.view(B, 1, H)
    if gated is None:
        y = glue.gate_sigmoid_mul(out.transpose(1, 2), qg[..., dh:])  # out storage is [B,T,hq,dh]
    else:
        y = gated
    if st.fold_norms:
        # o_proj + residual (writing the row statistics), gate/up with the post-attention norm
        # folded in, down_proj accumulated in place (writing the next layer's statistics; a
        # sequence shard's next layer, which keeps its input norm kernel, ignores them)
        rs2 = torch.empty((B * T, 4 * (H // 256)), device=x.device, dtype=torch.float32)
        x2 = glue.gemm_residual(y, src.o_proj.weight, x, ss_out=rs2)
        act = glue.gemm_swiglu(x2, st.folded("gu", self.post_attention_layernorm.weight, st.w_gu), st.inter,
                               row_ss=rs2, norm_eps=self.post_attention_layernorm.eps)
        rs3 = torch.empty_like(rs2)
        glue.gemm_residual(act, self.mlp.down_proj.weight, x2, out=x2, ss_out=rs3)
        x2._bna_row_ss = (rs3, x2.data_ptr(), x2._version)
        attn._profile(T, k_len_after, backend, hit, t0, fused=True)
        return x2
    if st.gemm_resid:  # o_proj with the residual add in the epilogue, then the norm
        x2 = glue.gemm_residual(y, src.o_proj.weight, x)
        h2 = glue.rmsnorm(x2, self.post_attention_layernorm.weight, self.post_attention_layernorm.eps)
    else:
        a = F.linear(y, src.o_proj.weight)
        h2, x2 = glue.rmsnorm(a, self.post_attention_layernorm.weight, self.post_attention_layernorm.eps,
                              residual=x, want_sum=True)
    if st.gemm_swiglu:  # gate/up GEMM with SwiGLU in the epilogue (no [T, 2*inter] product in HBM)
        act = glue.gemm_swiglu(h2, st.w_gu, st.inter)
    else:
        act = glue.swiglu(F.linear(h2, st.w_gu), st.inter)
    if st.gemm_resid:  # down_proj accumulated onto the residual in place
        glue.gemm_residual(act, self.mlp.down_proj.weight, x2, out=x2)
    else:
        x2.view(-1, H).addmm_(act.view(-1, st.inter), self.mlp.down_proj.weight.t())
    attn._profile(T, k_len_after, backend, hit, t0, fused=True)
    return x2


def _fused_lm_head_forward(self, x: torch.Tensor):
    """The output projection for up to 8 rows (decode, or the kept position of a prefill)
    as a weight-streaming GEMV (it streams the whole [vocab, hidden] matrix once)."""
    K = int(x.shape[-1])
    rows = x.numel() // K if K else 0
    w = self.weight
    if (x.is_cuda and x.dtype in (torch.bfloat16, torch.float16) and self.bias is None and 0 < rows <= 8
            and K % 256 == 0 and K <= 8192 and w.dtype == x.dtype and w.is_contiguous()):
        return glue.gemv(x.reshape(rows, K), w).view(*x.shape[:-1], int(w.shape[0]))
    return type(self).forward(self, x)


def _fused_norm_forward(self, x: torch.Tensor):
    if x.dtype not in (torch.bfloat16, torch.float16) or not x.is_cuda:
        return type(self).forward(self, x)
    return glue.rmsnorm(x, self.weight, self.eps)


def fuse_qwen_decoder_layers(model: nn.Module) -> list[int]:
    """Run every swapped decoder layer (and the final norm, and the output projection for up
    to 8 rows) through the fused glue kernels.
    Call after ``swap_qwen_attention_with_butterfly_cuda``; returns the fused layer indices."""
    decoder = _get_decoder_with_layers(model)
    fused = []
    for idx, layer in enumerate(decoder.layers):
        attn = getattr(layer, "self_attn", None)
        if not isinstance(attn, QwenCUDAButterflyAttention) or hasattr(layer, "_bna_fused"):
            if hasattr(layer, "_bna_fused"):
                fused.append(idx)
            continue
        if not (_is_qwen35_norm(layer.input_layernorm) and _is_qwen35_norm(layer.post_attention_layernorm)
                and _is_qwen35_norm(attn.fallback.q_norm) and _is_qwen35_norm(attn.fallback.k_norm)):
            continue
        if getattr(getattr(layer.mlp, "act_fn", None), "__class__", type(None)).__name__ not in ("SiLU", "SiLUActivation"):
            continue
        layer._bna_fused = _FusedState(layer)
        layer.forward = types.MethodType(_fused_layer_forward, layer)
        fused.append(idx)
    norm = getattr(decoder, "norm", None)
    if fused and norm is not None and _is_qwen35_norm(norm) and "forward" not in norm.__dict__:
        norm.forward = types.MethodType(_fused_norm_forward, norm)
    head = getattr(model, "lm_head", None)
    if fused and isinstance(head, nn.Linear) and "forward" not in head.__dict__:
        head.forward = types.MethodType(_fused_lm_head_forward, head)
    return fused


def unfuse_qwen_decoder_layers(model: nn.Module) -> list[int]:
    """Put back the original forwards (the merged weight buffers stay; modules see views)."""
    decoder = _get_decoder_with_layers(model)
    out = []
    for idx, layer in enumerate(decoder.layers):
        if hasattr(layer, "_bna_fused"):
            del layer._bna_fused
            layer.__dict__.pop("forward", None)
            out.append(idx)
    norm = getattr(decoder, "norm", None)
    if norm is not None:
        norm.__dict__.pop("forward", None)
    head = getattr(model, "lm_head", None)
    if isinstance(head, nn.Module):
        head.__dict__.pop("forward", None)
    return out


__all__ = ["fuse_qwen_decoder_layers", "unfuse_qwen_decoder_layers"]
