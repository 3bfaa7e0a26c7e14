"""Oracle restatement of the two-pool compressed KV cache (test infrastructure only).

Follows the reference's MLX cache ``bna/mlx/compressed_cache.py``:
  _allocate          :69-92   (tail_capacity = W + 2*max_chunk + 2*BS; summary_capacity)
  update_and_fetch   :94-172  (append :104-118, block close :123-149, tail trim :153-164)
  get_compressed_state :198-209, nbytes :231-244, state / meta_state :246-302
and the cache-aware decode of ``bna/mlx/attention.py``:
  _swa_stream_from_cache        :1669-1710
  _compressed_stream_from_cache :1713-1813
  _online_softmax_merge         :519-548
  compressed_butterfly_attention_from_cache :1816-1876
The tail is kept as a plain array that is shifted on trim, exactly as the reference does;
the CUDA implementation stores it as a ring instead and must expose the same logical view.
"""
from __future__ import annotations

import math

import numpy as np

NEG = -1e30
EPS = 1e-9


class CompressedKVCacheRef:
    def __init__(self, *, block_size=128, local_window_tokens=128, max_kv_size=None,
                 max_chunk_size=512, summary_round=None):
        self.block_size = int(block_size)
        self.local_window_tokens = int(local_window_tokens)
        self.max_kv_size = int(max_kv_size) if max_kv_size else None
        self.max_chunk_size = int(max_chunk_size)
        self.summary_round = summary_round
        self.tail_k = self.tail_v = self.sum_k = self.sum_v = None
        self.tail_capacity = self.summary_capacity = 0
        self.tail_size = self.summary_count = self.offset = self.summary_offset = 0

    def _allocate(self, B, H, dh):
        self.tail_capacity = self.local_window_tokens + 2 * self.max_chunk_size + 2 * self.block_size
        self.summary_capacity = (self.max_kv_size // self.block_size + 4) if self.max_kv_size else 2048
        self.tail_k = np.zeros((B, H, self.tail_capacity, dh), np.float32)
        self.tail_v = np.zeros_like(self.tail_k)
        self.sum_k = np.zeros((B, H, self.summary_capacity, dh), np.float32)
        self.sum_v = np.zeros_like(self.sum_k)

    def update(self, keys: np.ndarray, values: np.ndarray):
        B, H, step, dh = keys.shape
        if self.tail_k is None:
            self._allocate(B, H, dh)
        bs, lw = self.block_size, self.local_window_tokens
        if self.tail_size + step > self.tail_capacity:
            raise RuntimeError("tail capacity exceeded")
        self.tail_k[:, :, self.tail_size:self.tail_size + step] = keys
        self.tail_v[:, :, self.tail_size:self.tail_size + step] = values
        self.tail_size += step
        self.offset += step
        closed = []
        while self.summary_offset + bs <= self.offset - lw:
            tail_start = self.offset - self.tail_size
            bstart = self.summary_offset - tail_start
            if bstart < 0 or bstart + bs > self.tail_size:
                break
            if self.summary_count >= self.summary_capacity:
                raise RuntimeError("summary capacity exhausted")
            mk = self.tail_k[:, :, bstart:bstart + bs].astype(np.float32).mean(axis=2)
            mv = self.tail_v[:, :, bstart:bstart + bs].astype(np.float32).mean(axis=2)
            if self.summary_round is not None:
                mk, mv = self.summary_round(mk), self.summary_round(mv)
            self.sum_k[:, :, self.summary_count] = mk
            self.sum_v[:, :, self.summary_count] = mv
            closed.append(self.summary_offset // bs)
            self.summary_count += 1
            self.summary_offset += bs
        target = max(lw, step + lw - 1)
        while self.tail_size - bs >= target:
            keep = self.tail_size - bs
            self.tail_k[:, :, :keep] = self.tail_k[:, :, bs:bs + keep].copy()
            self.tail_v[:, :, :keep] = self.tail_v[:, :, bs:bs + keep].copy()
            self.tail_size = keep
        return closed

    @property
    def tail_start(self):
        return self.offset - self.tail_size

    def counters(self):
        return dict(offset=self.offset, summary_offset=self.summary_offset,
                    summary_count=self.summary_count, tail_start=self.tail_start,
                    tail_size=self.tail_size)

    def state(self):
        return (self.tail_k[:, :, :self.tail_size], self.tail_v[:, :, :self.tail_size],
                self.sum_k[:, :, :self.summary_count], self.sum_v[:, :, :self.summary_count])

    def meta_state(self):
        return tuple(map(str, (self.block_size, self.local_window_tokens, self.offset, self.summary_offset)))

    def nbytes(self, elem_size=2):
        if self.tail_k is None:
            return 0
        B, H, _, dh = self.tail_k.shape
        return 2 * B * H * dh * elem_size * (self.tail_size + self.summary_count)


def attention_from_cache(q, cache: CompressedKVCacheRef, neighbors, query_positions, *,
                         scale=None, return_lse=False):
    """Two streams (raw tail window, routed summaries) merged by online softmax."""
    B, Hq, Tq, dh = q.shape
    tail_k, tail_v, sk, sv = cache.state()
    Hkv = tail_k.shape[1]
    G = Hq // Hkv
    BS, W = cache.block_size, cache.local_window_tokens
    scale = 1.0 / math.sqrt(dh) if scale is None else scale
    qg = q.astype(np.float32).reshape(B, Hkv, G, Tq, dh)
    qp = np.asarray(query_positions, np.int64).reshape(Tq, 1)
    kabs = (cache.tail_start + np.arange(tail_k.shape[2])).reshape(1, -1)
    mask = (kabs <= qp) & (kabs > qp - W)
    sc = np.einsum("bhgtd,bhkd->bhgtk", qg, tail_k) * scale
    sc = np.where(mask, sc, NEG)
    m1 = sc.max(-1, keepdims=True)
    e = np.where(mask, np.exp(sc - m1), 0.0)
    l1 = e.sum(-1, keepdims=True)
    o1 = np.einsum("bhgtk,bhkd->bhgtd", e, tail_v) / np.maximum(l1, EPS)
    anyv = mask.any(-1).reshape(1, 1, 1, Tq, 1)
    o1, l1, m1 = np.where(anyv, o1, 0), np.where(anyv, l1, 0), np.where(anyv, m1, NEG)
    # routed summary stream
    nsum = sk.shape[2]
    S = len(neighbors[0])
    routed = np.full((Tq, S), -1, np.int64)
    for i, p in enumerate(qp[:, 0].tolist()):
        b = p // BS
        ls = max(0, p - W + 1)
        if b < 0 or b >= len(neighbors):
            continue
        c = 0
        for n in neighbors[b]:
            if n < 0 or n >= b or (n + 1) * BS > ls or n >= nsum:
                continue
            routed[i, c] = n
            c += 1
            if c >= S:
                break
    valid = routed >= 0
    idx = np.where(valid, routed, 0)
    if nsum == 0:
        kg = np.zeros((B, Hkv, Tq, S, dh), np.float32)
        vg = kg
    else:
        kg, vg = sk[:, :, idx], sv[:, :, idx]
    sc2 = np.einsum("bhgtd,bhtsd->bhgts", qg, kg) * scale
    sc2 = np.where(valid, sc2, NEG)
    m2 = sc2.max(-1, keepdims=True)
    e2 = np.where(valid, np.exp(sc2 - m2), 0.0)
    l2 = e2.sum(-1, keepdims=True)
    o2 = np.einsum("bhgts,bhtsd->bhgtd", e2, vg) / np.maximum(l2, EPS)
    anyv2 = valid.any(-1).reshape(1, 1, 1, Tq, 1)
    o2, l2, m2 = np.where(anyv2, o2, 0), np.where(anyv2, l2, 0), np.where(anyv2, m2, NEG)
    m = np.maximum(m1, m2)
    c1, c2 = np.exp(m1 - m), np.exp(m2 - m)
    lt = c1 * l1 + c2 * l2
    out = ((c1 * l1 * o1 + c2 * l2 * o2) / np.maximum(lt, EPS)).reshape(B, Hq, Tq, dh)
    if return_lse:
        return out.astype(np.float32), (m + np.log(lt)).reshape(B, Hq, Tq).astype(np.float32)
    return out.astype(np.float32)
