"""Compressed Butterfly attention — drop-in for the reference's bna.torch functions.

Replaces, with the same signatures, argument meaning and ValueError behaviour:
  butterfly_compressed_attention          (bna/torch/attention_wayfinder_permute.py:1046-1122)
  butterfly_compressed_attention_active   (:1125-1197)
  _block_mean_summaries_torch             (:1022-1043)  -> block_mean_summaries
Every call goes through libbna_b200.so (C ABI, include/bna_b200.h) into sm_100a kernels:
the mean-pool compressor, the tcgen05 prefill kernel and the active-row kernel.
There is no CPU path: CPU tensors raise ValueError.
"""
from __future__ import annotations

import ctypes
import math
from typing import Optional

import numpy as np
import torch

from . import _lib
from .topology import BlockHamiltonianLayout

# Device copies of neighbour tables for layouts built outside this package.
_table_cache: dict = {}


def route_for(layout, device: torch.device) -> tuple[_lib.Route, Optional[torch.Tensor]]:
    """C-ABI route for a layout.  Layouts built here carry a closed-form route; any other
    BlockHamiltonianLayout-like object is routed by its block_neighbors[0] table."""
    r = getattr(layout, "route", None)
    if r is not None:
        return r, None
    nb = layout.block_neighbors[0]
    key = (id(layout), nb.data_ptr(), str(device))
    hit = _table_cache.get(key)
    if hit is None:
        table = nb.to(device=device, dtype=torch.int32).contiguous()
        rr = _lib.Route()
        rr.block_size = int(layout.block_size)
        rr.num_blocks = int(layout.num_blocks)
        rr.max_degree = int(nb.shape[-1])
        rr.rule = 0
        rr.width = max(1, int(getattr(layout, "stage_count", 1)))
        rr.stage_idx = int(getattr(layout, "stage_idx", 0))
        rr.stage_count = max(1, int(getattr(layout, "stage_count", 1)))
        rr.partner_count = 0
        rr.local_window_blocks = 0
        rr.sink_count = 0
        rr.neighbors = table.data_ptr()
        if len(_table_cache) > 64:
            _table_cache.clear()
        hit = (rr, table, layout)
        _table_cache[key] = hit
    return hit[0], hit[1]


def block_mean_summaries(x: torch.Tensor, *, seq_len: int, block_size: int, num_blocks: int,
                         out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Mean of each block's valid tokens: [B,H,T,dh] -> [B,H,N,dh] in x's dtype."""
    B, H, T, dh = x.shape
    if int(T) != int(seq_len):
        raise ValueError(f"summary seq_len mismatch: x has T={T}, expected {seq_len}")
    _lib.require_cuda(x)
    if out is None:
        out = torch.empty((B, H, int(num_blocks), dh), device=x.device, dtype=x.dtype)
    xs, os_ = _lib.t4(x), _lib.t4(out)
    _lib.check(_lib.lib().bna_compress_blocks(
        ctypes.byref(xs), ctypes.byref(os_), _lib.dtype_code(x.dtype), int(block_size), 0, int(num_blocks),
        int(seq_len), 0, 0, _lib.stream_ptr(x.device)))
    return out


def block_mean_summaries_kv(k: torch.Tensor, v: torch.Tensor, *, seq_len: int, block_size: int, num_blocks: int,
                            k_out: Optional[torch.Tensor] = None, v_out: Optional[torch.Tensor] = None):
    """Block means of K and V in one launch: two [B,H,T,dh] -> two [B,H,N,dh]."""
    B, H, T, dh = k.shape
    if int(T) != int(seq_len) or tuple(v.shape) != tuple(k.shape):
        raise ValueError(f"summary seq_len mismatch: k/v have shapes {tuple(k.shape)}/{tuple(v.shape)}, T={seq_len}")
    _lib.require_cuda(k, v)
    if k_out is None:
        k_out = torch.empty((B, H, int(num_blocks), dh), device=k.device, dtype=k.dtype)
    if v_out is None:
        v_out = torch.empty_like(k_out)
    tk, tv, tko, tvo = (_lib.t4(x) for x in (k, v, k_out, v_out))
    _lib.check(_lib.lib().bna_compress_kv_blocks(
        ctypes.byref(tk), ctypes.byref(tv), ctypes.byref(tko), ctypes.byref(tvo), _lib.dtype_code(k.dtype),
        int(block_size), 0, int(num_blocks), int(seq_len), 0, 0, _lib.stream_ptr(k.device)))
    return k_out, v_out


def _lse_args(lse: Optional[torch.Tensor]):
    if lse is None:
        return None, 0, 0
    return lse.data_ptr(), int(lse.stride(0)), int(lse.stride(1))


def butterfly_compressed_attention(
    q: torch.Tensor,
    k: torch.Tensor,
    v: torch.Tensor,
    *,
    layout: BlockHamiltonianLayout,
    local_window_tokens: int,
    block_chunk_size: int = 0,
    return_lse: bool = False,
    scale: Optional[float] = None,
):
    """Compressed Butterfly prefill: exact local token window plus routed block summaries.

    q [B,Hq,T,dh], k/v [B,Hkv,T,dh] (any strides with dh contiguous).  Returns
    [B,Hq,T,dh] in q's dtype (a view whose storage is [B,T,Hq,dh], so the caller's
    ``transpose(1, 2).contiguous()`` is free); with ``return_lse`` also the fp32
    natural-log LSE [B,Hq,T] of the union softmax.  ``block_chunk_size`` is accepted for
    signature compatibility; the kernel streams tiles and needs no chunking.
    """
    batch, H_q, T, dh = q.shape
    H_kv = int(k.shape[1])
    if int(k.shape[0]) != batch or int(v.shape[0]) != batch:
        raise ValueError("q, k, v batch size mismatch")
    if int(k.shape[2]) != T or int(v.shape[2]) != T:
        raise ValueError("Compressed Butterfly prefill requires matching q/k/v lengths")
    if int(k.shape[-1]) != dh or int(v.shape[-1]) != dh:
        raise ValueError("q, k, v head_dim mismatch")
    if int(T) <= 0:
        raise ValueError("T must be positive")
    if int(local_window_tokens) <= 0:
        raise ValueError("local_window_tokens must be positive")
    _lib.require_cuda(q, k, v)
    if q.dtype != k.dtype or q.dtype != v.dtype:
        raise ValueError("q, k, v dtype mismatch")
    dt = _lib.dtype_code(q.dtype)
    BS, N = int(layout.block_size), int(layout.num_blocks)
    if N != -(-int(T) // BS):
        raise ValueError(f"layout has {N} blocks but T={T} needs {-(-int(T) // BS)}")
    out, lse, _, _ = prefill_with_summaries(q, k, v, layout, int(local_window_tokens), scale, return_lse)
    return (out, lse) if return_lse else out


def prefill_with_summaries(q, k, v, layout, window: int, scale: Optional[float] = None, return_lse: bool = False,
                           k_sum_out: Optional[torch.Tensor] = None, v_sum_out: Optional[torch.Tensor] = None,
                           gate: Optional[torch.Tensor] = None):
    """Compressor + prefill kernel; returns (out, lse or None, k_sum, v_sum).

    The block means land in ``k_sum_out``/``v_sum_out`` [B,Hkv,N,dh] when given (for
    instance a two-pool cache's summary slots, so that a prefill hands its closed blocks
    to the cache without a copy).  With ``gate`` [B,Hq,T,dh] the output is
    ``out * sigmoid(gate)`` (Qwen3.5's gated attention), applied in the kernel's store;
    the lse stays that of the ungated attention.  Shapes are checked by the caller."""
    batch, H_q, T, dh = q.shape
    BS, N = int(layout.block_size), int(layout.num_blocks)
    route, _keep = route_for(layout, q.device)
    if tuple(k.shape) == tuple(v.shape):
        ks, vs = block_mean_summaries_kv(k, v, seq_len=T, block_size=BS, num_blocks=N, k_out=k_sum_out,
                                         v_out=v_sum_out)
    else:
        ks = block_mean_summaries(k, seq_len=T, block_size=BS, num_blocks=N, out=k_sum_out)
        vs = block_mean_summaries(v, seq_len=T, block_size=BS, num_blocks=N, out=v_sum_out)
    out = torch.empty((batch, T, H_q, dh), device=q.device, dtype=q.dtype).transpose(1, 2)
    lse = torch.empty((batch, H_q, T), device=q.device, dtype=torch.float32) if return_lse else None
    sc = float(scale) if scale is not None else 1.0 / math.sqrt(dh)
    if gate is not None and not prefill_attention_into(q, k, v, ks, vs, out, lse, route, int(window), sc, gate=gate):
        from . import glue  # window beyond the fused kernel's ring: gate in a separate launch
        out = glue.gate_sigmoid_mul(out.transpose(1, 2), gate.transpose(1, 2)).view(
            batch, T, H_q, dh).transpose(1, 2)
    elif gate is None:
        prefill_attention_into(q, k, v, ks, vs, out, lse, route, int(window), sc)
    return out, lse, ks, vs


def prefill_attention_into(q, k, v, k_sum, v_sum, out, lse, route, window: int, scale: float, *,
                           q_pos0: int = 0, kv_pos0: int = 0, total_len: Optional[int] = None,
                           gate: Optional[torch.Tensor] = None) -> bool:
    """Launch the tcgen05 prefill kernel on pre-computed summaries (no allocation).

    Query row i is at global position q_pos0 + i and key row j at kv_pos0 + j; the
    routing covers a sequence of ``total_len`` tokens (default: q_pos0 + Tq).  With
    ``gate`` [B,Hq,Tq,dh] the store writes ``out * sigmoid(gate)``; when the window is
    too large for the gated kernel the ungated output is written and False is returned
    (the caller gates it), else True."""
    T = int(q.shape[2])
    tot = q_pos0 + T if total_len is None else int(total_len)
    lp, lb, lh = _lse_args(lse)
    tq, tk, tv, tks, tvs, to = (_lib.t4(x) for x in (q, k, v, k_sum, v_sum, out))
    L = _lib.lib()
    args_tail = (ctypes.byref(to), lp, lb, lh, _lib.dtype_code(q.dtype), ctypes.byref(route), int(window),
                 int(q_pos0), int(kv_pos0), tot, float(scale), _lib.stream_ptr(q.device))
    if gate is not None:
        if gate.dtype != q.dtype or tuple(gate.shape) != tuple(out.shape):
            raise ValueError("gate must match the output's shape and dtype")
        tg = _lib.t4(gate)
        st = L.bna_prefill_attention_gated(ctypes.byref(tq), ctypes.byref(tk), ctypes.byref(tv), ctypes.byref(tks),
                                           ctypes.byref(tvs), ctypes.byref(tg), *args_tail)
        if st != _lib.UNSUPPORTED:
            _lib.check(st)
            return True
    _lib.check(L.bna_prefill_attention(ctypes.byref(tq), ctypes.byref(tk), ctypes.byref(tv), ctypes.byref(tks),
                                       ctypes.byref(tvs), *args_tail))
    return gate is None


def butterfly_compressed_attention_active(
    q: torch.Tensor,
    k: torch.Tensor,
    v: torch.Tensor,
    *,
    layout: BlockHamiltonianLayout,
    query_positions: torch.Tensor,
    local_window_tokens: int,
    return_lse: bool = False,
    scale: Optional[float] = None,
):
    """Compressed Butterfly for active (cached) query rows over a full K/V history."""
    batch, H_q, Tq, dh = q.shape
    H_kv = int(k.shape[1])
    Tk = int(k.shape[2])
    if int(k.shape[0]) != batch or int(v.shape[0]) != batch:
        raise ValueError("q, k, v batch size mismatch")
    if int(v.shape[2]) != Tk:
        raise ValueError("k and v sequence length mismatch")
    if int(k.shape[-1]) != dh or int(v.shape[-1]) != dh:
        raise ValueError("q, k, v head_dim mismatch")
    if Tk <= 0:
        raise ValueError("kv_len must be positive")
    if int(local_window_tokens) <= 0:
        raise ValueError("local_window_tokens must be positive")
    _lib.require_cuda(q, k, v)
    dt = _lib.dtype_code(q.dtype)
    BS, N = int(layout.block_size), int(layout.num_blocks)
    if N != -(-Tk // BS):
        raise ValueError(f"layout has {N} blocks but kv_len={Tk} needs {-(-Tk // BS)}")
    pos = query_positions.to(device=q.device, dtype=torch.int64).reshape(-1).contiguous()
    if int(pos.numel()) != Tq:
        raise ValueError("query_positions must have one entry per query row")
    route, _keep = route_for(layout, q.device)
    ks = block_mean_summaries(k, seq_len=Tk, block_size=BS, num_blocks=N)
    vs = block_mean_summaries(v, seq_len=Tk, block_size=BS, num_blocks=N)
    out = torch.empty((batch, Tq, H_q, dh), device=q.device, dtype=q.dtype).transpose(1, 2)
    lse = torch.empty((batch, H_q, Tq), device=q.device, dtype=torch.float32) if return_lse else None
    lp, lb, lh = _lse_args(lse)
    sc = float(scale) if scale is not None else 1.0 / math.sqrt(dh)
    tq, tk, tv, tks, tvs, to = (_lib.t4(x) for x in (q, k, v, ks, vs, out))
    _lib.check(_lib.lib().bna_active_attention(
        ctypes.byref(tq), ctypes.byref(tk), ctypes.byref(tv), ctypes.byref(tks), ctypes.byref(tvs),
        ctypes.byref(to), lp, lb, lh, dt, ctypes.byref(route), int(local_window_tokens), pos.data_ptr(),
        0, 0, 0, N, sc, _lib.stream_ptr(q.device)))
    return (out, lse) if return_lse else out


def prefill_selection(layout, T: int, local_window_tokens: int):
    """Host dump (same C++ code as the kernels) of per-block raw-window start and summary slots."""
    r, _ = route_for(layout, torch.device("cpu")) if getattr(layout, "route", None) is not None else (None, None)
    if r is None:
        raise ValueError("prefill_selection needs a layout built by butterfly_b200")
    N, K = int(r.num_blocks), int(r.max_degree)
    ls = np.empty(N, np.int32)
    idx = np.empty((N, K), np.int32)
    cnt = np.empty(N, np.int32)
    P = ctypes.POINTER(ctypes.c_int32)
    _lib.check(_lib.lib().bna_prefill_selection_host(ctypes.byref(r), int(T), int(local_window_tokens),
                                                     ls.ctypes.data_as(P), idx.ctypes.data_as(P), cnt.ctypes.data_as(P)))
    return ls, idx, cnt


def active_selection(layout, query_positions, local_window_tokens: int, num_summary_limit: Optional[int] = None):
    r = getattr(layout, "route", None)
    if r is None:
        raise ValueError("active_selection needs a layout built by butterfly_b200")
    pos = np.ascontiguousarray(np.asarray(query_positions, np.int64).reshape(-1))
    n, K = len(pos), int(r.max_degree)
    blk, ls, cnt = (np.empty(n, np.int32) for _ in range(3))
    idx = np.empty((n, K), np.int32)
    P = ctypes.POINTER(ctypes.c_int32)
    lim = int(r.num_blocks) if num_summary_limit is None else int(num_summary_limit)
    _lib.check(_lib.lib().bna_active_selection_host(
        ctypes.byref(r), int(local_window_tokens), pos.ctypes.data_as(ctypes.POINTER(ctypes.c_int64)), n, lim,
        blk.ctypes.data_as(P), ls.ctypes.data_as(P), idx.ctypes.data_as(P), cnt.ctypes.data_as(P)))
    return blk, ls, idx, cnt
