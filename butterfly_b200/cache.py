"""Two-pool compressed KV cache on the device (tail ring + summary pool).

Semantics follow the reference's ``CompressedKVCache`` (bna/mlx/compressed_cache.py):
capacities (:69-92), append (:104-118), block close (:123-149), tail trim (:153-164),
state / meta_state / nbytes (:198-302).  The counters (offset, summary_offset,
summary_count, tail_size) evolve exactly as there.  The storage differs: the tail is a
ring of ``tail_capacity`` slots where position p lives at slot ``p % tail_capacity``, so
a trim only moves ``tail_start`` and never copies data.  ``state`` materialises the
logical tail in position order, so serialised state is identical to the reference's.

Data movement goes through libbna_b200.so: ``bna_cache_append`` (chunk append),
``bna_compress_blocks`` over the ring (block close) and ``bna_decode_step`` (fused
append + close + attention for one-token decode).
"""
from __future__ import annotations

import ctypes
import math
from typing import Optional

import torch

from . import _lib
from .attention import _lse_args, route_for


class CompressedKVCache:
    def __init__(self, *, block_size: int = 128, local_window_tokens: int = 128,
                 max_kv_size: Optional[int] = None, max_chunk_size: int = 512) -> None:
        self.block_size = int(block_size)
        self.local_window_tokens = int(local_window_tokens)
        self.max_kv_size = int(max_kv_size) if max_kv_size else None
        self.max_chunk_size = int(max_chunk_size)
        self._tail_k: Optional[torch.Tensor] = None
        self._tail_v: Optional[torch.Tensor] = None
        self._sum_k: Optional[torch.Tensor] = None
        self._sum_v: Optional[torch.Tensor] = None
        self.tail_capacity = 0
        self.summary_capacity = 0
        self.tail_size = 0
        self.summary_count = 0
        self.offset = 0
        self.summary_offset = 0

    # ------------------------------------------------------------------ storage
    def _allocate(self, B: int, H: int, dh: int, dtype: torch.dtype, device: torch.device) -> None:
        self.tail_capacity = self.local_window_tokens + 2 * self.max_chunk_size + 2 * self.block_size
        self.summary_capacity = (self.max_kv_size // self.block_size + 4) if self.max_kv_size else 2048
        # every kernel reads only ring slots and summary slots it wrote before (the window of
        # appended positions, closed blocks), so the pools need no clearing
        self._tail_k = torch.empty((B, H, self.tail_capacity, dh), dtype=dtype, device=device)
        self._tail_v = torch.empty_like(self._tail_k)
        self._sum_k = torch.empty((B, H, self.summary_capacity, dh), dtype=dtype, device=device)
        self._sum_v = torch.empty_like(self._sum_k)

    @property
    def ring(self) -> int:
        return self.tail_capacity

    @property
    def tail_start(self) -> int:
        return self.offset - self.tail_size

    # ------------------------------------------------------------------ counter logic
    def _plan_closes(self) -> list[int]:
        """Blocks the reference's close loop (:123-149) closes at the current counters."""
        bs, lw = self.block_size, self.local_window_tokens
        closes = []
        so = self.summary_offset
        while so + bs <= self.offset - lw:
            tail_start = self.offset - self.tail_size
            bstart = so - tail_start
            if bstart < 0 or bstart + bs > self.tail_size:
                break
            if self.summary_count + len(closes) >= self.summary_capacity:
                raise RuntimeError(
                    f"CompressedKVCache.summary_capacity={self.summary_capacity} exhausted "
                    f"at offset={self.offset}; raise max_kv_size at construction time.")
            closes.append(so // bs)
            so += bs
        return closes

    def _trim(self, step: int) -> None:
        target = max(self.local_window_tokens, step + self.local_window_tokens - 1)
        while self.tail_size - self.block_size >= target:
            self.tail_size -= self.block_size

    def _check_room(self, step: int) -> None:
        if self.tail_size + step > self.tail_capacity:
            raise RuntimeError(
                f"CompressedKVCache.tail_capacity={self.tail_capacity} too small to fit "
                f"tail_size={self.tail_size} + step={step}; raise max_chunk_size or "
                f"local_window_tokens to make room.")

    def _close(self, blocks: list[int]) -> None:
        if not blocks:
            return
        first = blocks[0]
        assert blocks == list(range(first, first + len(blocks)))
        dev = self._tail_k.device
        dt = _lib.dtype_code(self._tail_k.dtype)
        tk, tv, sk, sv = (_lib.t4(x) for x in (self._tail_k, self._tail_v, self._sum_k, self._sum_v))
        _lib.check(_lib.lib().bna_compress_kv_blocks(
            ctypes.byref(tk), ctypes.byref(tv), ctypes.byref(sk), ctypes.byref(sv), dt, self.block_size,
            first * self.block_size, len(blocks), len(blocks) * self.block_size, self.ring, self.summary_count,
            _lib.stream_ptr(dev)))
        self.summary_count += len(blocks)
        self.summary_offset += len(blocks) * self.block_size

    # ------------------------------------------------------------------ public API
    def append(self, keys: torch.Tensor, values: torch.Tensor) -> list[int]:
        """Append a chunk [B,H,step,dh]; close and trim as the reference.  Returns closed blocks."""
        _lib.require_cuda(keys, values)
        B, H, step, dh = keys.shape
        if self._tail_k is None:
            self._allocate(B, H, dh, keys.dtype, keys.device)
        self._check_room(step)
        tk, tv, sk, sv = (_lib.t4(x) for x in (self._tail_k, self._tail_v, keys, values))
        _lib.check(_lib.lib().bna_cache_append(ctypes.byref(tk), ctypes.byref(tv), ctypes.byref(sk), ctypes.byref(sv),
                                               _lib.dtype_code(keys.dtype), self.offset, self.ring,
                                               _lib.stream_ptr(keys.device)))
        self.tail_size += step
        self.offset += step
        closes = self._plan_closes()
        self._close(closes)
        self._trim(step)
        return closes

    # ------------------------------------------------------------------ prefill hand-off
    def reserve(self, batch: int, heads: int, head_dim: int, dtype: torch.dtype, device: torch.device) -> None:
        """Allocate the pools now (normally done by the first append)."""
        if self._tail_k is None:
            self._allocate(int(batch), int(heads), int(head_dim), dtype, device)

    def summary_slots(self, num_blocks: int):
        """Views [B,H,num_blocks,dh] of the first summary slots, or None if the pool is
        smaller.  A prefill can write its block means here directly: the closed blocks
        become the cache's summaries and the slots past ``summary_count`` stay unused
        until their block closes (which rewrites them)."""
        if self._sum_k is None or int(num_blocks) > self.summary_capacity:
            return None
        return self._sum_k[:, :, : int(num_blocks)], self._sum_v[:, :, : int(num_blocks)]

    def _advance_counters_chunked(self, total: int, step: int) -> None:
        """Counter evolution of ``append`` over consecutive chunks of ``step`` tokens."""
        if step <= 0:
            raise ValueError("chunk_size must be positive")
        for s in range(0, total, step):
            n = min(step, total - s)
            self._check_room(n)
            self.tail_size += n
            self.offset += n
            closes = self._plan_closes()
            self.summary_count += len(closes)
            self.summary_offset += len(closes) * self.block_size
            self._trim(n)

    def adopt_prefill(self, keys: torch.Tensor, values: torch.Tensor, k_sum: torch.Tensor, v_sum: torch.Tensor,
                      *, chunk_size: Optional[int] = None) -> None:
        """Take over a one-shot prefill of T tokens as if it had been appended in chunks.

        The counters become exactly those of ``append`` called on consecutive chunks of
        ``chunk_size`` tokens (default ``max_chunk_size``; the reference harness feeds its
        MLX cache ``kv_step`` chunks, bench_qwen_consumer_mlx.py:494-522), so the cache
        keeps only its tail and the closed blocks' means instead of the whole prompt.
        The closed summaries are the prefill's block means ``k_sum``/``v_sum``
        [B,H,>=summary_count,dh] (the same fp32 means, summed in the same order, as a
        close computes); they are copied unless they already are this cache's
        ``summary_slots``.  Only the last ``tail_size`` rows of keys/values are copied
        into the ring."""
        _lib.require_cuda(keys, values, k_sum, v_sum)
        if self.offset != 0:
            raise RuntimeError("adopt_prefill needs an empty cache")
        B, H, T, dh = keys.shape
        if tuple(values.shape) != tuple(keys.shape):
            raise ValueError("keys and values must have the same shape")
        self.reserve(B, H, dh, keys.dtype, keys.device)
        self._advance_counters_chunked(int(T), int(chunk_size) if chunk_size else self.max_chunk_size)
        S = self.summary_count
        if S > int(k_sum.shape[2]):
            raise ValueError(f"prefill summaries hold {int(k_sum.shape[2])} blocks, the cache closed {S}")
        if S and k_sum.data_ptr() != self._sum_k.data_ptr():
            self._sum_k[:, :, :S].copy_(k_sum[:, :, :S])
            self._sum_v[:, :, :S].copy_(v_sum[:, :, :S])
        t0 = self.tail_start
        if self.tail_size:
            tk, tv, sk, sv = (_lib.t4(x) for x in (self._tail_k, self._tail_v, keys[:, :, t0:], values[:, :, t0:]))
            _lib.check(_lib.lib().bna_cache_append(ctypes.byref(tk), ctypes.byref(tv), ctypes.byref(sk),
                                                   ctypes.byref(sv), _lib.dtype_code(keys.dtype), t0, self.ring,
                                                   _lib.stream_ptr(keys.device)))

    def update_and_fetch(self, keys: torch.Tensor, values: torch.Tensor):
        self.append(keys, values)
        return self.keys, self.values

    def attend(self, q: torch.Tensor, layout, query_positions: Optional[torch.Tensor] = None, *,
               scale: Optional[float] = None, return_lse: bool = False):
        """Queries [B,Hq,Tq,dh] at absolute positions (default: the last Tq appended tokens)
        over the raw tail window and the routed summaries (MLX from_cache, :1816-1876)."""
        _lib.require_cuda(q)
        B, Hq, Tq, dh = q.shape
        route, _keep = route_for(layout, q.device)
        out = torch.empty((B, Tq, Hq, dh), device=q.device, dtype=q.dtype).transpose(1, 2)
        lse = torch.empty((B, Hq, Tq), device=q.device, dtype=torch.float32) if return_lse else None
        lp, lb, lh = _lse_args(lse)
        pos_ptr = None
        pos0 = self.offset - Tq
        if query_positions is not None:
            pos = query_positions.to(device=q.device, dtype=torch.int64).reshape(-1).contiguous()
            pos_ptr = pos.data_ptr()
        sc = float(scale) if scale is not None else 1.0 / math.sqrt(dh)
        tq, tk, tv, tks, tvs, to = (_lib.t4(x) for x in (q, self._tail_k, self._tail_v, self._sum_k, self._sum_v, out))
        _lib.check(_lib.lib().bna_active_attention(
            ctypes.byref(tq), ctypes.byref(tk), ctypes.byref(tv), ctypes.byref(tks), ctypes.byref(tvs),
            ctypes.byref(to), lp, lb, lh, _lib.dtype_code(q.dtype), ctypes.byref(route), self.local_window_tokens,
            pos_ptr, pos0, 0, self.ring, self.summary_count, sc, _lib.stream_ptr(q.device)))
        return (out, lse) if return_lse else out

    def decode_step(self, q: torch.Tensor, k_new: torch.Tensor, v_new: torch.Tensor, layout, *,
                    scale: Optional[float] = None, return_lse: bool = False, qk_prep=None):
        """One fused launch: append one token per sequence, close a block if one completes,
        trim, and attend q [B,Hq,1,dh] at the new position.

        With ``qk_prep = (q_norm_weight, k_norm_weight, cos, sin, eps)`` q and k_new are the
        raw projection rows: the launch also applies the Qwen3.5 q/k RMSNorm and the rotary
        embedding (cos / sin [B,1,rot]) before appending and attending."""
        _lib.require_cuda(q, k_new, v_new)
        B, Hq, Tq, dh = q.shape
        if Tq != 1 or k_new.shape[2] != 1:
            raise ValueError("decode_step takes exactly one new token per sequence")
        if self._tail_k is None:
            self._allocate(B, k_new.shape[1], dh, k_new.dtype, k_new.device)
        self._check_room(1)
        pos = self.offset
        self.tail_size += 1
        self.offset += 1
        closes = self._plan_closes()
        if len(closes) > 1:  # lagging closes (only after unusual chunk patterns): do all but the last
            self._close(closes[:-1])
            closes = closes[-1:]
        close_block = closes[0] if closes else -1
        close_slot = self.summary_count if closes else -1
        limit = self.summary_count + (1 if closes else 0)
        route, _keep = route_for(layout, q.device)
        out = torch.empty((B, 1, Hq, dh), device=q.device, dtype=q.dtype).transpose(1, 2)
        lse = torch.empty((B, Hq, 1), device=q.device, dtype=torch.float32) if return_lse else None
        lp, lb, lh = _lse_args(lse)
        sc = float(scale) if scale is not None else 1.0 / math.sqrt(dh)
        ts = [_lib.t4(x) for x in (q, k_new, v_new, self._tail_k, self._tail_v, self._sum_k, self._sum_v, out)]
        if qk_prep is None:
            _lib.check(_lib.lib().bna_decode_step(
                *(ctypes.byref(t) for t in ts), lp, lb, lh, _lib.dtype_code(q.dtype), ctypes.byref(route),
                self.local_window_tokens, pos, self.ring, close_block, close_slot, limit, sc,
                _lib.stream_ptr(q.device)))
        else:
            qw, kw, cos, sin, eps = qk_prep
            rot = int(cos.shape[-1])
            if cos.stride(-1) != 1 or sin.stride() != cos.stride() or int(cos.shape[0]) not in (1, B):
                raise ValueError("cos / sin must be [B or 1, 1, rot] with contiguous rows and equal strides")
            if qw.dtype != q.dtype or kw.dtype != q.dtype or not qw.is_contiguous() or not kw.is_contiguous():
                raise ValueError("q / k norm weights must be contiguous and of q's dtype")
            cs_b = int(cos.stride(0)) if int(cos.shape[0]) > 1 else 0
            _lib.check(_lib.lib().bna_decode_step_qk(
                *(ctypes.byref(t) for t in ts), lp, lb, lh, _lib.dtype_code(q.dtype), ctypes.byref(route),
                self.local_window_tokens, pos, self.ring, close_block, close_slot, limit, sc, qw.data_ptr(),
                kw.data_ptr(), cos.data_ptr(), sin.data_ptr(), cs_b, rot, float(eps), _lib.stream_ptr(q.device)))
        if closes:
            self.summary_count += 1
            self.summary_offset += self.block_size
        self._trim(1)
        return (out, lse) if return_lse else out

    # ------------------------------------------------------------------ views / state
    def _tail_view(self, buf: Optional[torch.Tensor]) -> Optional[torch.Tensor]:
        if buf is None:
            return None
        idx = torch.arange(self.tail_start, self.offset, device=buf.device) % self.ring
        return buf.index_select(2, idx)

    @property
    def keys(self):
        return self._tail_view(self._tail_k)

    @property
    def values(self):
        return self._tail_view(self._tail_v)

    @property
    def k_summary(self):
        return None if self._sum_k is None else self._sum_k[:, :, : self.summary_count]

    @property
    def v_summary(self):
        return None if self._sum_v is None else self._sum_v[:, :, : self.summary_count]

    def get_compressed_state(self):
        if self._tail_k is None:
            raise ValueError("CompressedKVCache is empty")
        return self.keys, self.values, self.k_summary, self.v_summary, int(self.tail_start), int(self.offset)

    def size(self) -> int:
        return int(self.offset)

    def empty(self) -> bool:
        return self._tail_k is None or self.tail_size == 0

    @property
    def nbytes(self) -> int:
        """Valid-slice bytes (tail + summaries, K and V), as the reference reports (:231-244)."""
        if self._tail_k is None:
            return 0
        B, H, _, dh = self._tail_k.shape
        e = self._tail_k.element_size()
        return 2 * B * H * dh * e * (self.tail_size + self.summary_count)

    @property
    def state(self):
        return self.keys, self.values, self.k_summary, self.v_summary

    @state.setter
    def state(self, v) -> None:
        keys, values, k_summary, v_summary = v
        if keys is None or values is None:
            self._tail_k = self._tail_v = None
            self.tail_size = 0
        else:
            B, H, T, dh = keys.shape
            if self._tail_k is None or self._tail_k.shape[2] < T:
                self._allocate(B, H, dh, keys.dtype, keys.device)
            # logical tail restored at its positions; offset is set by meta_state, so stage
            # the rows at slots 0..T-1 and re-home them when meta_state arrives
            self._staged_tail = (keys, values)
            self.tail_size = int(T)
        if k_summary is None or v_summary is None:
            self.summary_count = 0
        else:
            B, H, S, dh = k_summary.shape
            if self._sum_k is None or self._sum_k.shape[2] < S:
                self.summary_capacity = max(S, self.summary_capacity)
                self._sum_k = torch.zeros((B, H, self.summary_capacity, dh), dtype=k_summary.dtype,
                                          device=k_summary.device)
                self._sum_v = torch.zeros_like(self._sum_k)
            self._sum_k[:, :, :S] = k_summary
            self._sum_v[:, :, :S] = v_summary
            self.summary_count = int(S)
        self._rehome()

    @property
    def meta_state(self):
        return tuple(map(str, (self.block_size, self.local_window_tokens, self.offset, self.summary_offset)))

    @meta_state.setter
    def meta_state(self, v) -> None:
        self.block_size, self.local_window_tokens, self.offset, self.summary_offset = map(int, v)
        self._rehome()

    def _rehome(self) -> None:
        staged = getattr(self, "_staged_tail", None)
        if staged is None or self._tail_k is None:
            return
        keys, values = staged
        T = keys.shape[2]
        idx = (torch.arange(self.offset - T, self.offset, device=keys.device) % self.ring)
        self._tail_k.index_copy_(2, idx, keys)
        self._tail_v.index_copy_(2, idx, values)
