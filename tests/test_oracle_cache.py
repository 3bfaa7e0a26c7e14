"""Two-pool cache restatement: counters, summary numerics, and decode == active rows.

Mirrors the reference's MLX cache tests (tests/mlx/test_compressed_kv_cache.py:12-53,
tests/mlx/test_compressed_butterfly_from_cache.py:16-82), which cannot run without MLX;
the decode equality is anchored on the reference-pinned torch active-row oracle.
"""
import numpy as np
import pytest

from oracle import compressed as oc
from oracle import topology as ot
from oracle.cache import CompressedKVCacheRef, attention_from_cache


def _nb(kv_len, BS, layer):
    N = ot.num_blocks_for_seq_len(kv_len, BS)
    return ot.block_neighbors_table(N, layer, local_window_blocks=1, sink_count=1, partner_count=1,
                                    partner_rule="causal_shift")


def test_summary_numerics_and_tail_bounds():
    rng = np.random.default_rng(101)
    xk = rng.standard_normal((1, 2, 24, 8), dtype=np.float32)
    xv = rng.standard_normal((1, 2, 24, 8), dtype=np.float32)
    c = CompressedKVCacheRef(block_size=4, local_window_tokens=4)
    for s in range(0, 24, 3):
        c.update(xk[:, :, s:s + 3], xv[:, :, s:s + 3])
    tk, tv, sk, sv = c.state()
    assert c.offset == 24 and c.tail_start % 4 == 0
    assert 4 <= tk.shape[2] < 4 + 3 + 4
    n = sk.shape[2]
    np.testing.assert_allclose(sk, oc.block_means(xk[:, :, :n * 4], 4), atol=1e-6)
    np.testing.assert_allclose(sv, oc.block_means(xv[:, :, :n * 4], 4), atol=1e-6)
    np.testing.assert_array_equal(tk, xk[:, :, c.tail_start:24])


@pytest.mark.parametrize("chunks,BS,W,layer", [
    ([3] * 8, 4, 4, 3),
    ([37, 1, 1, 1, 5, 1, 64, 1, 1], 8, 6, 2),
    ([100] + [1] * 40, 16, 16, 5),
])
def test_decode_from_cache_equals_active_rows(chunks, BS, W, layer):
    rng = np.random.default_rng(202)
    T = sum(chunks)
    B, Hq, Hkv, dh = 2, 4, 2, 8
    k = rng.standard_normal((B, Hkv, T, dh), dtype=np.float32)
    v = rng.standard_normal((B, Hkv, T, dh), dtype=np.float32)
    c = CompressedKVCacheRef(block_size=BS, local_window_tokens=W, max_chunk_size=max(chunks))
    pos = 0
    for n in chunks:
        c.update(k[:, :, pos:pos + n], v[:, :, pos:pos + n])
        pos += n
        qp = np.arange(pos - n, pos)
        q = rng.standard_normal((B, Hq, n, dh), dtype=np.float32)
        nb = _nb(pos, BS, layer)
        ref, ref_lse = oc.active_attention(q, k[:, :, :pos], v[:, :, :pos], nb, qp, block_size=BS, window=W)
        got, got_lse = attention_from_cache(q, c, nb, qp, return_lse=True)
        np.testing.assert_allclose(got, ref, atol=3e-4, rtol=3e-4)
        np.testing.assert_allclose(got_lse, ref_lse, atol=1e-4)
        assert c.tail_start % BS == 0 and c.tail_size >= min(W, c.offset)


def test_capacity_errors():
    c = CompressedKVCacheRef(block_size=4, local_window_tokens=4, max_chunk_size=4)
    x = np.zeros((1, 1, 30, 2), np.float32)
    with pytest.raises(RuntimeError):
        c.update(x, x)
    c = CompressedKVCacheRef(block_size=4, local_window_tokens=4, max_kv_size=8, max_chunk_size=4)
    with pytest.raises(RuntimeError):
        for _ in range(40):
            c.update(x[:, :, :1], x[:, :, :1])


def test_sampled_block_prefill_equals_full_prefill():
    """The sampled-row prefill oracle (used at 128k / 262k) equals the full oracle's rows."""
    rng = np.random.default_rng(5)
    B, Hq, Hkv, T, dh, BS, W = 1, 4, 2, 1000, 16, 64, 24
    q = rng.standard_normal((B, Hq, T, dh), dtype=np.float32)
    k = rng.standard_normal((B, Hkv, T, dh), dtype=np.float32)
    v = rng.standard_normal((B, Hkv, T, dh), dtype=np.float32)
    nb = _nb(T, BS, 3)
    full, full_lse = oc.prefill_attention(q, k, v, nb, block_size=BS, window=W)
    blocks = [0, 1, 5, 8, 15]
    qb = np.zeros((B, Hq, len(blocks), BS, dh), np.float32)
    for i, b in enumerate(blocks):
        n = min(BS, T - b * BS)
        qb[:, :, i, :n] = q[:, :, b * BS:b * BS + n]
    got, got_lse = oc.prefill_attention_blocks(qb, k, v, nb, blocks, block_size=BS, window=W)
    for i, b in enumerate(blocks):
        n = min(BS, T - b * BS)
        np.testing.assert_allclose(got[:, :, i, :n], full[:, :, b * BS:b * BS + n], atol=1e-5)
        np.testing.assert_allclose(got_lse[:, :, i, :n], full_lse[:, :, b * BS:b * BS + n], atol=1e-5)


def test_handoff_counters_equal_chunked_appends():
    """A one-shot prefill handed to the cache ends with the counters of chunked appends
    (the counter arithmetic alone; the device copy is checked in the GPU tests)."""
    from butterfly_b200.cache import CompressedKVCache
    for T, chunk, BS, W in [(10000, 1024, 128, 64), (131072, 4096, 128, 64), (777, 100, 16, 8), (64, 512, 128, 64)]:
        ref = CompressedKVCacheRef(block_size=BS, local_window_tokens=W, max_chunk_size=chunk, max_kv_size=T + 64)
        ref._allocate(1, 1, 1)
        c = CompressedKVCache(block_size=BS, local_window_tokens=W, max_chunk_size=chunk, max_kv_size=T + 64)
        c.tail_capacity = ref.tail_capacity
        c.summary_capacity = ref.summary_capacity
        for s in range(0, T, chunk):
            n = min(chunk, T - s)
            ref.update(np.zeros((1, 1, n, 1), np.float32), np.zeros((1, 1, n, 1), np.float32))
        c._advance_counters_chunked(T, chunk)
        assert (c.offset, c.summary_offset, c.summary_count, c.tail_start, c.tail_size) == tuple(
            ref.counters()[x] for x in ("offset", "summary_offset", "summary_count", "tail_start", "tail_size"))
