"""GPU parity: every kernel through the C ABI against the CPU oracle.

Bars (from the path's contract): selection indices and cache counters bit-exact; bf16
outputs within max-abs 2e-2 of the fp32 oracle evaluated on the same bf16 inputs; LSE
within 1e-3; block means within one bf16 ulp.
"""
import math

import numpy as np
import pytest
import torch

import butterfly_b200 as bb
from butterfly_b200 import _lib
from butterfly_b200.attention import prefill_selection
from butterfly_b200.cache import CompressedKVCache
from oracle import compressed as oc
from oracle import topology as ot
from oracle.cache import CompressedKVCacheRef, attention_from_cache

pytestmark = pytest.mark.gpu

OUT_TOL = 2e-2
LSE_TOL = 1e-3


def _to_np(x: torch.Tensor) -> np.ndarray:
    return x.detach().float().cpu().numpy()


def _inputs(B, Hq, Hkv, T, dh, seed, dtype=torch.bfloat16, layout="bhtd", q_scale=1.0):
    g = torch.Generator().manual_seed(seed)
    if layout == "bhtd":
        q = torch.randn(B, Hq, T, dh, generator=g) * q_scale
        k = torch.randn(B, Hkv, T, dh, generator=g)
        v = torch.randn(B, Hkv, T, dh, generator=g)
    else:  # HF storage [B, T, H, dh] seen through transpose(1, 2)
        q = (torch.randn(B, T, Hq, dh, generator=g) * q_scale).transpose(1, 2)
        k = torch.randn(B, T, Hkv, dh, generator=g).transpose(1, 2)
        v = torch.randn(B, T, Hkv, dh, generator=g).transpose(1, 2)
    return [x.to(dtype).cuda() for x in (q, k, v)]


def _round(dtype):
    if dtype == torch.bfloat16:
        return oc.round_bf16
    return lambda a: a.astype(np.float16).astype(np.float32)


def _layout(T, BS, Hkv, G, layer, rule="causal_shift", lwb=1, sink=1, pc=1):
    return bb.build_block_butterfly_layout(seq_len=T, block_size=BS, num_key_value_heads=Hkv,
                                           num_key_value_groups=G, layer_idx=layer, local_window_blocks=lwb,
                                           sink_count=sink, partner_count=pc, partner_rule=rule)


def _check_prefill(B, Hq, Hkv, T, BS, W, layer, *, dtype=torch.bfloat16, layout="bhtd", rule="causal_shift",
                   lwb=1, sink=1, pc=1, seed=0, q_scale=1.0, foreign_table=False):
    q, k, v = _inputs(B, Hq, Hkv, T, 128, seed, dtype, layout, q_scale)
    lay = _layout(T, BS, Hkv, Hq // Hkv, layer, rule, lwb, sink, pc)
    if foreign_table:  # a layout object without a closed-form route: table-driven path
        import dataclasses
        lay = dataclasses.replace(lay, route=None)
    out, lse = bb.butterfly_compressed_attention(q, k, v, layout=lay, local_window_tokens=W, return_lse=True)
    torch.cuda.synchronize()
    nb = lay.block_neighbors[0].tolist()
    ref, ref_lse = oc.prefill_attention(_to_np(q), _to_np(k), _to_np(v), nb, block_size=BS, window=W,
                                        summary_round=_round(dtype))
    got = _to_np(out)
    err = np.abs(got - ref).max()
    lerr = np.abs(_to_np(lse) - ref_lse).max()
    assert np.isfinite(got).all()
    assert err <= OUT_TOL, f"max-abs {err}"
    assert lerr <= LSE_TOL, f"lse max-abs {lerr}"
    return err, lerr


def test_config1_shapes_bf16():
    # config 1 shapes (B1, 8/2 heads, T4096, BS128, W64, layer 3) in bf16, q scaled by 1/sqrt(128)
    _check_prefill(1, 8, 2, 4096, 128, 64, 3, q_scale=1 / math.sqrt(128))


@pytest.mark.parametrize("layer", range(8))
def test_config2_stages_small(layer):
    # every causal_shift stage 0..7 (partner offsets 1..128) on a 256-block sequence
    _check_prefill(1, 8, 2, 32768, 128, 64, layer)


@pytest.mark.parametrize("case", [
    dict(B=2, Hq=8, Hkv=2, T=1000, BS=128, W=64, layer=2),          # ragged T
    dict(B=1, Hq=8, Hkv=8, T=700, BS=128, W=64, layer=1),           # G = 1
    dict(B=1, Hq=4, Hkv=2, T=513, BS=128, W=64, layer=4),           # G = 2
    dict(B=1, Hq=16, Hkv=2, T=777, BS=128, W=64, layer=5),          # G = 8
    dict(B=1, Hq=8, Hkv=2, T=2048, BS=128, W=128, layer=3),         # W = 128 (reference default)
    dict(B=1, Hq=8, Hkv=2, T=1500, BS=64, W=16, layer=6),           # small blocks / window
    dict(B=1, Hq=8, Hkv=2, T=3000, BS=128, W=64, layer=2, lwb=3, sink=2, pc=2),
    dict(B=1, Hq=8, Hkv=2, T=2000, BS=128, W=64, layer=1, rule="xor"),
    dict(B=1, Hq=8, Hkv=2, T=2000, BS=128, W=64, layer=2, rule="bit_reversal"),
    dict(B=1, Hq=8, Hkv=2, T=2000, BS=128, W=64, layer=7, rule="benes"),
    dict(B=1, Hq=8, Hkv=2, T=1, BS=128, W=64, layer=0),             # single token
    dict(B=1, Hq=8, Hkv=2, T=65, BS=128, W=64, layer=0),
])
def test_prefill_shapes(case):
    _check_prefill(case.pop("B"), case.pop("Hq"), case.pop("Hkv"), case.pop("T"), case.pop("BS"), case.pop("W"),
                   case.pop("layer"), **case)


def test_prefill_hf_transposed_views_fp16_and_table():
    _check_prefill(2, 8, 2, 1200, 128, 64, 3, layout="bthd")
    _check_prefill(1, 8, 2, 1200, 128, 64, 3, dtype=torch.float16)
    _check_prefill(1, 8, 2, 1200, 128, 64, 3, foreign_table=True)


def test_prefill_output_store_paths_agree_bitwise():
    # an output view whose rows are 16- but not 32-byte aligned takes the 128-bit store path;
    # it must write exactly what the 256-bit path writes into a contiguous output
    from butterfly_b200.attention import block_mean_summaries, prefill_attention_into, route_for
    B, Hq, Hkv, T, BS, W = 1, 8, 2, 4096, 128, 64
    q, k, v = _inputs(B, Hq, Hkv, T, 128, 7)
    lay = _layout(T, BS, Hkv, Hq // Hkv, 4)
    route, _keep = route_for(lay, q.device)
    N = lay.num_blocks
    ks = block_mean_summaries(k, seq_len=T, block_size=BS, num_blocks=N)
    vs = block_mean_summaries(v, seq_len=T, block_size=BS, num_blocks=N)
    sc = 1.0 / math.sqrt(128)
    out_a = torch.empty(B, T, Hq, 128, device=q.device, dtype=q.dtype).transpose(1, 2)
    big = torch.zeros(B, T, Hq, 136, device=q.device, dtype=q.dtype)
    out_b = big[..., 8:].transpose(1, 2)  # head stride 136 * 2 B: not a 32-byte multiple
    assert (out_b.stride(1) * 2) % 32 != 0 and (out_b.data_ptr() % 16) == 0
    prefill_attention_into(q, k, v, ks, vs, out_a, None, route, W, sc)
    prefill_attention_into(q, k, v, ks, vs, out_b, None, route, W, sc)
    torch.cuda.synchronize()
    assert torch.equal(out_a, out_b)
    assert torch.count_nonzero(big[..., :8]) == 0  # nothing written outside the view


def test_selection_device_equals_host():
    import ctypes
    for T, layer, rule in [(32768, 5, "causal_shift"), (4096, 3, "causal_shift"), (70000, 9, "xor")]:
        lay = _layout(T, 128, 2, 4, layer, rule)
        ls, idx, cnt = prefill_selection(lay, T, 64)
        r = lay.route
        didx = torch.empty((r.num_blocks, r.max_degree), dtype=torch.int32, device="cuda")
        dcnt = torch.empty((r.num_blocks,), dtype=torch.int32, device="cuda")
        _lib.check(_lib.lib().bna_prefill_selection_device(ctypes.byref(r), T, 64, didx.data_ptr(), dcnt.data_ptr(),
                                                           _lib.stream_ptr(didx.device)))
        np.testing.assert_array_equal(didx.cpu().numpy(), idx)
        np.testing.assert_array_equal(dcnt.cpu().numpy(), cnt)


@pytest.mark.parametrize("T,BS", [(4096, 128), (1000, 128), (77, 16), (32768, 128)])
def test_block_means(T, BS):
    _, k, _ = _inputs(2, 2, 2, T, 128, 7)
    N = -(-T // BS)
    got = _to_np(bb.block_mean_summaries(k, seq_len=T, block_size=BS, num_blocks=N))
    ref = oc.round_bf16(oc.block_means(_to_np(k), BS, N))
    ulp = np.abs(ref) * 2.0 ** -7 + 1e-30
    assert (np.abs(got - ref) <= ulp).all()


@pytest.mark.parametrize("Tk,layer", [(4096, 3), (1000, 1), (65537, 9)])
def test_active_rows(Tk, layer):
    B, Hq, Hkv, W, BS = 2, 8, 2, 64, 128
    q, k, v = _inputs(B, Hq, Hkv, Tk, 128, 11)
    pos = torch.tensor(sorted({0, 1, 63, 64, 200, Tk - 1, Tk // 2, Tk - 129}), dtype=torch.int64)
    qa = q[:, :, : len(pos)].contiguous()
    lay = _layout(Tk, BS, Hkv, Hq // Hkv, layer)
    out, lse = bb.butterfly_compressed_attention_active(qa, k, v, layout=lay, query_positions=pos,
                                                        local_window_tokens=W, return_lse=True)
    torch.cuda.synchronize()
    ref, ref_lse = oc.active_attention(_to_np(qa), _to_np(k), _to_np(v), lay.block_neighbors[0].tolist(),
                                       pos.numpy(), block_size=BS, window=W, summary_round=oc.round_bf16)
    assert np.abs(_to_np(out) - ref).max() <= OUT_TOL
    assert np.abs(_to_np(lse) - ref_lse).max() <= LSE_TOL


def _cache_run(chunks, BS, W, layer, B=2, Hq=8, Hkv=2, fused=True, seed=3):
    T = sum(chunks)
    g = torch.Generator().manual_seed(seed)
    k = torch.randn(B, Hkv, T, 128, generator=g).bfloat16()
    v = torch.randn(B, Hkv, T, 128, generator=g).bfloat16()
    kn, vn = _to_np(k), _to_np(v)
    dc = CompressedKVCache(block_size=BS, local_window_tokens=W, max_chunk_size=max(chunks), max_kv_size=T)
    rc = CompressedKVCacheRef(block_size=BS, local_window_tokens=W, max_chunk_size=max(chunks), max_kv_size=T,
                              summary_round=oc.round_bf16)
    pos = 0
    worst = 0.0
    for n in chunks:
        q = torch.randn(B, Hq, n, 128, generator=g).bfloat16()
        kv_len = pos + n
        N = -(-kv_len // BS)
        nb = ot.block_neighbors_table(N, layer, local_window_blocks=1, sink_count=1, partner_count=1,
                                      partner_rule="causal_shift")
        lay = _layout(kv_len, BS, Hkv, Hq // Hkv, layer)
        rc.update(kn[:, :, pos:pos + n], vn[:, :, pos:pos + n])
        if fused and n == 1:
            out = dc.decode_step(q.cuda(), k[:, :, pos:pos + 1].cuda(), v[:, :, pos:pos + 1].cuda(), lay)
        else:
            dc.append(k[:, :, pos:pos + n].cuda(), v[:, :, pos:pos + n].cuda())
            out = dc.attend(q.cuda(), lay)
        pos += n
        torch.cuda.synchronize()
        assert (dc.offset, dc.summary_offset, dc.summary_count, dc.tail_start, dc.tail_size) == tuple(
            rc.counters()[x] for x in ("offset", "summary_offset", "summary_count", "tail_start", "tail_size"))
        ref = attention_from_cache(_to_np(q), rc, nb, np.arange(pos - n, pos))
        worst = max(worst, float(np.abs(_to_np(out) - ref).max()))
    tk, tv, sk, sv = dc.state
    rtk, rtv, rsk, rsv = rc.state()
    np.testing.assert_array_equal(_to_np(tk), rtk)
    np.testing.assert_array_equal(_to_np(tv), rtv)
    ulp = np.abs(rsk) * 2.0 ** -7 + 1e-30
    assert (np.abs(_to_np(sk) - rsk) <= ulp).all()
    assert dc.nbytes == rc.nbytes(2)
    assert worst <= OUT_TOL, worst
    return dc


def test_cache_decode_fused_matches_oracle():
    _cache_run([600] + [1] * 300, BS=128, W=64, layer=3)


def test_cache_chunked_prefill_matches_oracle():
    _cache_run([37, 200, 1, 1, 64, 300, 5, 1, 1], BS=64, W=32, layer=2, fused=False)
    _cache_run([512] * 6 + [1] * 40, BS=128, W=64, layer=5)


def test_cache_state_round_trip():
    dc = _cache_run([300] + [1] * 20, BS=64, W=32, layer=1)
    st, meta = dc.state, dc.meta_state
    r = CompressedKVCache(block_size=1, local_window_tokens=1)
    r.state = st
    r.meta_state = meta
    assert (r.offset, r.summary_offset, r.block_size, r.local_window_tokens) == (dc.offset, dc.summary_offset, 64, 32)
    for a, b in zip(r.state, st):
        assert torch.equal(a, b)


def test_capacity_errors_raise_runtime_error():
    dc = CompressedKVCache(block_size=4, local_window_tokens=4, max_chunk_size=4)
    x = torch.zeros(1, 1, 30, 128, dtype=torch.bfloat16, device="cuda")
    with pytest.raises(RuntimeError):
        dc.append(x, x)


def test_no_device_error_word_left():
    import ctypes
    code = ctypes.c_int32(-1)
    _lib.check(_lib.lib().bna_take_device_error(torch.cuda.current_device(), ctypes.byref(code)))
    assert code.value == 0


def test_shard_offsets_match_unsharded_bitwise():
    """The prefill kernel run on one shard (global query offset, keys starting W-1 tokens
    earlier as the halo, global summaries) reproduces the unsharded run exactly."""
    from butterfly_b200.seqshard import cuda_ops
    T, BS, W, world = 8192, 128, 64, 4
    q, k, v = _inputs(1, 8, 2, T, 128, 21)
    lay = _layout(T, BS, 2, 4, 6)
    full = bb.butterfly_compressed_attention(q, k, v, layout=lay, local_window_tokens=W)
    ks = bb.block_mean_summaries(k, seq_len=T, block_size=BS, num_blocks=T // BS)
    vs = bb.block_mean_summaries(v, seq_len=T, block_size=BS, num_blocks=T // BS)
    ops = cuda_ops(lay, W)
    Tl, h = T // world, W - 1
    for r in range(world):
        kv0 = 0 if r == 0 else r * Tl - h
        y = ops.attend(q[:, :, r * Tl:(r + 1) * Tl], k[:, :, kv0:(r + 1) * Tl], v[:, :, kv0:(r + 1) * Tl],
                       ks, vs, r * Tl, kv0, T)
        torch.cuda.synchronize()
        assert torch.equal(y, full[:, :, r * Tl:(r + 1) * Tl]), r
