"""GPU parity at the benchmark workloads' own sizes, through the C ABI.

* one attention layer of the 128k model (T=131072, Hq8/Hkv2) and of the 262k model
  (T=262144, Hq16/Hkv4): sampled query blocks (first blocks, partner boundaries, the
  last block) against the oracle, output max-abs <= 2e-2 and LSE <= 1e-3, plus the
  whole output finite;
* the batched decode workload (64 sequences x 65536 pre-filled tokens, 128 fused steps):
  cache counters bit-exact at every step and four sequences' outputs against the
  restated two-pool cache and its decode;
* the prefill -> cache hand-off: identical state to chunked appends;
* greedy decode of a swapped model replayed from a CUDA graph equals the eager run.
"""
import math

import numpy as np
import pytest
import torch

import butterfly_b200 as bb
from oracle import compressed as oc
from oracle.cache import CompressedKVCacheRef, attention_from_cache

pytestmark = pytest.mark.gpu

OUT_TOL = 2e-2
LSE_TOL = 1e-3


def _np(x):
    return x.detach().float().cpu().numpy()


def _long_layer(T, Hq, Hkv, layer, blocks, seed):
    dev = torch.device("cuda")
    g = torch.Generator(device=dev).manual_seed(seed)
    q = torch.randn(1, Hq, T, 128, device=dev, generator=g).bfloat16()
    k = torch.randn(1, Hkv, T, 128, device=dev, generator=g).bfloat16()
    v = torch.randn(1, Hkv, T, 128, device=dev, generator=g).bfloat16()
    lay = bb.build_block_butterfly_layout(seq_len=T, block_size=128, num_key_value_heads=Hkv,
                                          num_key_value_groups=Hq // Hkv, layer_idx=layer, local_window_blocks=1,
                                          sink_count=1, partner_count=1, partner_rule="causal_shift")
    out, lse = bb.butterfly_compressed_attention(q, k, v, layout=lay, local_window_tokens=64, return_lse=True)
    torch.cuda.synchronize()
    assert bool(torch.isfinite(out).all()) and bool(torch.isfinite(lse).all())
    qb = torch.stack([q[:, :, b * 128:(b + 1) * 128] for b in blocks], 2)
    ref, ref_lse = oc.prefill_attention_blocks(_np(qb), _np(k), _np(v), lay.block_neighbors[0].tolist(), blocks,
                                               block_size=128, window=64, summary_round=oc.round_bf16)
    got = _np(torch.stack([out[:, :, b * 128:(b + 1) * 128] for b in blocks], 2))
    got_lse = _np(torch.stack([lse[:, :, b * 128:(b + 1) * 128] for b in blocks], 2))
    err = float(np.abs(got - ref).max())
    lerr = float(np.abs(got_lse - ref_lse).max())
    assert err <= OUT_TOL, err
    assert lerr <= LSE_TOL, lerr


def test_model_128k_attention_layer():
    # N=1024 blocks, width 10; layer 23 -> stage 3 (partner = block - 8)
    T = 131072
    _long_layer(T, 8, 2, 23, [0, 1, 2, 3, 8, 9, 10, 17, 511, 512, 513, 1000, 1022, 1023], seed=31)


def test_model_262k_attention_layer():
    # N=2048 blocks, width 11; layer 31 -> stage 9 (partner = block - 512), Hq16/Hkv4
    T = 262144
    _long_layer(T, 16, 4, 31, [0, 1, 2, 511, 512, 513, 1024, 1536, 2046, 2047], seed=32)


def test_batched_decode_workload_full_size():
    """64 sequences x 65536 tokens, 128 fused steps (the bench's batched-decode workload)."""
    import bench
    keep = 4
    dev = torch.device("cuda")
    cache, q, kn, vn, host = bench.decode_inputs(dev, seed=2000, keep=keep)
    lays = bench.decode_layouts()
    ref = CompressedKVCacheRef(block_size=bench.BS, local_window_tokens=bench.W,
                               max_kv_size=bench.DEC_CTX + bench.DEC_STEPS, max_chunk_size=bench.DEC_CHUNK,
                               summary_round=oc.round_bf16)
    for hk, hv in host:
        ref.update(hk.float().numpy(), hv.float().numpy())
    worst = 0.0
    for i in range(bench.DEC_STEPS):
        out = cache.decode_step(q[i], kn[i], vn[i], lays[i])
        ref.update(_np(kn[i][:keep]), _np(vn[i][:keep]))
        assert (cache.offset, cache.summary_offset, cache.summary_count, cache.tail_start, cache.tail_size) == tuple(
            ref.counters()[x] for x in ("offset", "summary_offset", "summary_count", "tail_start", "tail_size"))
        r = attention_from_cache(_np(q[i][:keep]), ref, lays[i].block_neighbors[0].tolist(), [cache.offset - 1])
        worst = max(worst, float(np.abs(_np(out[:keep]) - r).max()))
        assert bool(torch.isfinite(out).all())
    assert worst <= OUT_TOL, worst
    assert cache.nbytes == ref.nbytes(2) * (q.shape[1] // keep)


def test_prefill_handoff_equals_chunked_appends():
    from butterfly_b200.attention import block_mean_summaries_kv
    from butterfly_b200.cache import CompressedKVCache
    B, H, T, BS, W, chunk = 2, 2, 10000, 128, 64, 1024
    g = torch.Generator(device="cuda").manual_seed(9)
    k = torch.randn(B, H, T, 128, device="cuda", generator=g).bfloat16()
    v = torch.randn(B, H, T, 128, device="cuda", generator=g).bfloat16()
    a = CompressedKVCache(block_size=BS, local_window_tokens=W, max_chunk_size=chunk, max_kv_size=T + 200)
    for s in range(0, T, chunk):
        a.append(k[:, :, s:s + chunk], v[:, :, s:s + chunk])
    b = CompressedKVCache(block_size=BS, local_window_tokens=W, max_chunk_size=chunk, max_kv_size=T + 200)
    b.reserve(B, H, 128, k.dtype, k.device)
    N = -(-T // BS)
    ks, vs = b.summary_slots(N)
    block_mean_summaries_kv(k, v, seq_len=T, block_size=BS, num_blocks=N, k_out=ks, v_out=vs)
    b.adopt_prefill(k, v, ks, vs)
    assert (a.offset, a.summary_offset, a.summary_count, a.tail_size) == (
        b.offset, b.summary_offset, b.summary_count, b.tail_size)
    for x, y in zip(a.state, b.state):
        assert torch.equal(x, y)
    gq = torch.Generator(device="cuda").manual_seed(10)
    for s in range(150):  # decode across a block close
        q = torch.randn(B, 8, 1, 128, device="cuda", generator=gq).bfloat16()
        kn = torch.randn(B, H, 1, 128, device="cuda", generator=gq).bfloat16()
        vn = torch.randn(B, H, 1, 128, device="cuda", generator=gq).bfloat16()
        lay = bb.build_block_butterfly_layout(seq_len=T + s + 1, block_size=BS, num_key_value_heads=H,
                                              num_key_value_groups=4, layer_idx=5, local_window_blocks=1,
                                              sink_count=1, partner_count=1, partner_rule="causal_shift")
        assert torch.equal(a.decode_step(q, kn, vn, lay), b.decode_step(q, kn, vn, lay))


def test_graphed_greedy_decode_equals_eager():
    from transformers import DynamicCache, Qwen3_5TextConfig
    from transformers.models.qwen3_5.modeling_qwen3_5 import Qwen3_5ForCausalLM

    from butterfly_b200.integrations import qwen_torch as qt
    qt.patch_qwen35_full_attention_decode()
    cfg = Qwen3_5TextConfig(hidden_size=512, num_attention_heads=8, num_key_value_heads=2, head_dim=128,
                            num_hidden_layers=3, layer_types=["full_attention"] * 3, intermediate_size=768,
                            vocab_size=1000)
    torch.manual_seed(4)
    m = Qwen3_5ForCausalLM(cfg).eval().to(torch.bfloat16).cuda()
    qt.swap_qwen_attention_with_butterfly_cuda(m, qt.compressed_config())
    ids = torch.randint(0, 1000, (1, 3000), generator=torch.Generator().manual_seed(5)).cuda()
    steps = 40  # crosses a block close at offset 3072 + 64

    def fresh():
        cache = qt.make_compressed_cache(m, DynamicCache(config=m.config), max_kv_size=4096, max_chunk_size=1024)
        with torch.no_grad():
            out = m(input_ids=ids, past_key_values=cache, use_cache=True, logits_to_keep=1)
        for layer in qt.iter_qwen_butterfly_layers(m):
            assert layer.last_profile["block_sparse_backend"] == "compressed_prefill+cache_handoff"
        return out.logits[:, -1].argmax(-1, keepdim=True), cache

    tok, cache = fresh()
    eager = []
    with torch.no_grad():
        for _ in range(steps):
            out = m(input_ids=tok, past_key_values=cache, use_cache=True)
            tok = out.logits[:, -1].argmax(-1, keepdim=True)
            eager.append(int(tok))
    tok, cache = fresh()
    with torch.no_grad():
        gd = qt.GraphedGreedyDecode(m, cache, tok, steps)
        gd.replay()
        gd.replay()
    torch.cuda.synchronize()
    assert gd.tokens[0].tolist() == eager
    assert gd.eager_tokens[0].tolist() == eager
    torch.testing.assert_close(gd.logits.float(), gd.eager_logits.float(), atol=1e-2, rtol=0)
