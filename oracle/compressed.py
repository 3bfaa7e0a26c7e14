"""Oracle restatement of compressed Butterfly attention (test infrastructure only).

Follows ``bna/torch/attention_wayfinder_permute.py`` of the reference:
  _compressed_butterfly_block_index_tensors   :912-966   -> prefill_selection / prefill_index_tensors
  _compressed_butterfly_active_index_tensors  :969-1019  -> active_selection / active_index_tensors
  _block_mean_summaries_torch                 :1022-1043 -> block_means
  butterfly_compressed_attention              :1046-1122 -> prefill_attention
  butterfly_compressed_attention_active       :1125-1197 -> active_attention
The union softmax the reference delegates to ``F.scaled_dot_product_attention`` with a
boolean mask (scale 1/sqrt(dh), GQA by head groups) is restated directly, and its
log-sum-exp (which SDPA does not return) is produced alongside it.
All arithmetic is fp32 numpy, as the reference runs on CPU.
"""
from __future__ import annotations

import math

import numpy as np


def round_bf16(x: np.ndarray) -> np.ndarray:
    """Round fp32 values to the nearest bf16 (ties to even), returned as fp32."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    u = x.view(np.uint32).astype(np.uint64)
    nan = np.isnan(x)
    rounded = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16) << 16
    out = rounded.astype(np.uint32).view(np.float32).copy()
    out[nan] = np.nan
    return out


def _summary_slots_for(row: list[int], block_idx: int, cutoff: int, block_size: int,
                       slots: int, num_summary_blocks: int | None = None) -> list[int]:
    """Cursor-packed routed summaries (reference :952-964 / :1005-1017)."""
    out = []
    for n in row:
        if n < 0 or n >= block_idx:
            continue
        if (n + 1) * block_size > cutoff:
            continue
        if num_summary_blocks is not None and n >= num_summary_blocks:
            continue
        out.append(n)
        if len(out) >= slots:
            break
    return out


def prefill_selection(neighbors, T: int, block_size: int, window: int):
    """Per block: (local_start, [valid summary blocks in slot order])."""
    N = len(neighbors)
    slots = len(neighbors[0]) if N else 0
    sel = []
    for b in range(N):
        local_start = max(0, b * block_size - window + 1)
        sel.append((local_start, _summary_slots_for(neighbors[b], b, local_start, block_size, slots)))
    return sel


def active_selection(neighbors, query_positions, block_size: int, window: int):
    """Per query: (block, raw_start, [valid summary blocks in slot order])."""
    N = len(neighbors)
    slots = len(neighbors[0]) if N else 0
    sel = []
    for p in [int(x) for x in query_positions]:
        b = min(max(0, p // max(1, block_size)), max(0, N - 1))
        local_start = max(0, p - window + 1)
        sel.append((b, local_start, _summary_slots_for(neighbors[b], b, local_start, block_size, slots)))
    return sel


def prefill_index_tensors(neighbors, T: int, block_size: int, window: int):
    """Exact restatement of the reference's four prefill index tensors (:912-966)."""
    N = len(neighbors)
    BS = block_size
    raw_slots = window + BS - 1
    S = len(neighbors[0])
    raw_idx = np.zeros((N, raw_slots), np.int64)
    raw_mask = np.zeros((N, BS, raw_slots), bool)
    summary_idx = np.zeros((N, S), np.int64)
    summary_mask = np.zeros((N, BS, S), bool)
    offs = np.arange(raw_slots)
    boffs = np.arange(BS)
    for b, (ls, summ) in enumerate(prefill_selection(neighbors, T, BS, window)):
        qpos = b * BS + boffs
        qv = qpos < T
        rp = ls + offs
        raw_idx[b] = np.clip(rp, 0, max(0, T - 1))
        raw_mask[b] = (qv[:, None] & (rp < T)[None, :] & (rp[None, :] <= qpos[:, None])
                       & (rp[None, :] >= qpos[:, None] - window + 1))
        for c, n in enumerate(summ):
            summary_idx[b, c] = n
            summary_mask[b, :, c] = qv
    return raw_idx, raw_mask, summary_idx, summary_mask


def active_index_tensors(neighbors, kv_len: int, query_positions, block_size: int, window: int):
    """Exact restatement of the reference's four active index tensors (:969-1019)."""
    qp = [int(x) for x in query_positions]
    S = len(neighbors[0])
    raw_idx = np.zeros((len(qp), window), np.int64)
    raw_mask = np.zeros((len(qp), window), bool)
    summary_idx = np.zeros((len(qp), S), np.int64)
    summary_mask = np.zeros((len(qp), S), bool)
    offs = np.arange(window)
    for i, (b, ls, summ) in enumerate(active_selection(neighbors, qp, block_size, window)):
        rp = ls + offs
        raw_idx[i] = np.clip(rp, 0, max(0, kv_len - 1))
        raw_mask[i] = (rp <= qp[i]) & (rp < kv_len)
        for c, n in enumerate(summ):
            summary_idx[i, c] = n
            summary_mask[i, c] = True
    return raw_idx, raw_mask, summary_idx, summary_mask


def block_means(x: np.ndarray, block_size: int, num_blocks: int | None = None) -> np.ndarray:
    """fp32 mean of each block's valid tokens; [B,H,T,dh] -> [B,H,N,dh] (:1022-1043)."""
    B, H, T, dh = x.shape
    N = num_blocks if num_blocks is not None else -(-T // block_size)
    pad = N * block_size - T
    xf = x.astype(np.float32)
    if pad:
        xf = np.concatenate([xf, np.zeros((B, H, pad, dh), np.float32)], axis=2)
    s = xf.reshape(B, H, N, block_size, dh).sum(axis=3, dtype=np.float32)
    cnt = np.clip(np.minimum(block_size, T - np.arange(N) * block_size), 1, None).astype(np.float32)
    return s / cnt[None, None, :, None]


def _softmax_rows(scores: np.ndarray, mask: np.ndarray):
    s = np.where(mask, scores, -np.inf)
    m = s.max(axis=-1, keepdims=True)
    m_safe = np.where(np.isfinite(m), m, 0.0)
    e = np.where(mask, np.exp(s - m_safe), 0.0).astype(np.float32)
    l = e.sum(axis=-1, keepdims=True)
    w = e / np.maximum(l, 1e-30)
    with np.errstate(divide="ignore"):
        lse = (m_safe + np.log(l))[..., 0]
    return w, lse


def prefill_attention(q, k, v, neighbors, *, block_size: int, window: int,
                      summary_round=None, scale: float | None = None, block_chunk: int = 16):
    """Union softmax over the raw window and routed summaries for every query.

    q [B,Hq,T,dh], k/v [B,Hkv,T,dh] (fp32 arrays holding the kernel's input values).
    ``summary_round`` rounds the fp32 block means to the storage dtype (the reference
    casts them to the input dtype, :1043).  Returns (out fp32 [B,Hq,T,dh], lse fp32 [B,Hq,T]).
    """
    B, Hq, T, dh = q.shape
    Hkv = k.shape[1]
    G = Hq // Hkv
    BS = block_size
    N = len(neighbors)
    scale = 1.0 / math.sqrt(dh) if scale is None else scale
    ks = block_means(k, BS, N)
    vs = block_means(v, BS, N)
    if summary_round is not None:
        ks, vs = summary_round(ks), summary_round(vs)
    raw_idx, raw_mask, summary_idx, summary_mask = prefill_index_tensors(neighbors, T, BS, window)
    R = raw_idx.shape[1]
    S = summary_idx.shape[1]
    pad = N * BS - T
    qf = q.astype(np.float32)
    if pad:
        qf = np.concatenate([qf, np.zeros((B, Hq, pad, dh), np.float32)], axis=2)
    qb = qf.reshape(B, Hkv, G, N, BS, dh)
    out = np.zeros((B, Hkv, G, N, BS, dh), np.float32)
    lse = np.zeros((B, Hkv, G, N, BS), np.float32)
    kf = k.astype(np.float32)
    vf = v.astype(np.float32)
    for c0 in range(0, N, block_chunk):
        c1 = min(N, c0 + block_chunk)
        kr = kf[:, :, raw_idx[c0:c1]]                 # [B,Hkv,n,R,dh]
        vr = vf[:, :, raw_idx[c0:c1]]
        ksum = ks[:, :, summary_idx[c0:c1]]           # [B,Hkv,n,S,dh]
        vsum = vs[:, :, summary_idx[c0:c1]]
        kc = np.concatenate([kr, ksum], axis=3)       # [B,Hkv,n,R+S,dh]
        vc = np.concatenate([vr, vsum], axis=3)
        mask = np.concatenate([raw_mask[c0:c1], summary_mask[c0:c1]], axis=2)  # [n,BS,R+S]
        qc = qb[:, :, :, c0:c1]                       # [B,Hkv,G,n,BS,dh]
        sc = np.einsum("bhgnqd,bhnkd->bhgnqk", qc, kc, optimize=True).astype(np.float32) * scale
        w, l = _softmax_rows(sc, mask[None, None, None])
        out[:, :, :, c0:c1] = np.einsum("bhgnqk,bhnkd->bhgnqd", w, vc, optimize=True)
        lse[:, :, :, c0:c1] = l
    out = out.reshape(B, Hq, N * BS, dh)[:, :, :T]
    lse = lse.reshape(B, Hq, N * BS)[:, :, :T]
    return out, lse


def prefill_attention_blocks(q_blocks, k, v, neighbors, blocks, *, block_size: int, window: int,
                             summary_round=None, scale: float | None = None):
    """``prefill_attention`` evaluated only for the query blocks in ``blocks`` (sampled
    rows of a long sequence).  ``q_blocks`` [B,Hq,len(blocks),BS,dh] holds those blocks'
    query rows (rows past T zero); block means and selection are those of the whole
    sequence given by k/v [B,Hkv,T,dh].  Returns (out fp32 [B,Hq,len(blocks),BS,dh],
    lse fp32 [B,Hq,len(blocks),BS]); rows past T are meaningless."""
    B, Hq, nsel, BS, dh = q_blocks.shape
    Hkv, T = k.shape[1], k.shape[2]
    G = Hq // Hkv
    assert BS == block_size and nsel == len(blocks)
    N = len(neighbors)
    scale = 1.0 / math.sqrt(dh) if scale is None else scale
    ks = block_means(k, BS, N)
    vs = block_means(v, BS, N)
    if summary_round is not None:
        ks, vs = summary_round(ks), summary_round(vs)
    raw_idx, raw_mask, summary_idx, summary_mask = prefill_index_tensors(neighbors, T, BS, window)
    out = np.zeros((B, Hq, nsel, BS, dh), np.float32)
    lse = np.zeros((B, Hq, nsel, BS), np.float32)
    for i, b in enumerate(blocks):
        kc = np.concatenate([k[:, :, raw_idx[b]].astype(np.float32), ks[:, :, summary_idx[b]]], axis=2)
        vc = np.concatenate([v[:, :, raw_idx[b]].astype(np.float32), vs[:, :, summary_idx[b]]], axis=2)
        mask = np.concatenate([raw_mask[b], summary_mask[b]], axis=1)                    # [BS,R+S]
        qg = q_blocks[:, :, i].astype(np.float32).reshape(B, Hkv, G, BS, dh)
        sc = np.einsum("bhgqd,bhkd->bhgqk", qg, kc).astype(np.float32) * scale
        w, l = _softmax_rows(sc, mask[None, None, None])
        out[:, :, i] = np.einsum("bhgqk,bhkd->bhgqd", w, vc).reshape(B, Hq, BS, dh)
        lse[:, :, i] = l.reshape(B, Hq, BS)
    return out, lse


def active_attention(q, k, v, neighbors, query_positions, *, block_size: int, window: int,
                     summary_round=None, scale: float | None = None):
    """Active/decode rows over a full K/V history (:1125-1197).  Returns (out, lse)."""
    B, Hq, Tq, dh = q.shape
    Hkv, Tk = k.shape[1], k.shape[2]
    G = Hq // Hkv
    N = len(neighbors)
    scale = 1.0 / math.sqrt(dh) if scale is None else scale
    ks = block_means(k, block_size, N)
    vs = block_means(v, block_size, N)
    if summary_round is not None:
        ks, vs = summary_round(ks), summary_round(vs)
    raw_idx, raw_mask, summary_idx, summary_mask = active_index_tensors(
        neighbors, Tk, query_positions, block_size, window)
    kf, vf = k.astype(np.float32), v.astype(np.float32)
    kc = np.concatenate([kf[:, :, raw_idx], ks[:, :, summary_idx]], axis=3)  # [B,Hkv,Tq,R+S,dh]
    vc = np.concatenate([vf[:, :, raw_idx], vs[:, :, summary_idx]], axis=3)
    mask = np.concatenate([raw_mask, summary_mask], axis=1)                   # [Tq,R+S]
    qg = q.astype(np.float32).reshape(B, Hkv, G, Tq, dh)
    sc = np.einsum("bhgtd,bhtkd->bhgtk", qg, kc).astype(np.float32) * scale
    w, l = _softmax_rows(sc, mask[None, None, None])
    out = np.einsum("bhgtk,bhtkd->bhgtd", w, vc).reshape(B, Hq, Tq, dh)
    return out.astype(np.float32), l.reshape(B, Hq, Tq).astype(np.float32)
