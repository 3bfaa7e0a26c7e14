"""Fused decoder-layer glue kernels against the eager ops they replace, and a fused model
against the unfused swapped model.

Each kernel keeps the eager arithmetic (fp32 inside a norm, each elementwise result
rounded to bf16); the norms' fp32 sums run in a different order, so results may differ by
one bf16 rounding step: the bar is max |a - b| <= 2^-7 * max(|b|, 1) per element (one bf16
ulp) and at least 99% of elements bit-identical.  The fused model's logits must stay
within 3e-2 of the unfused model's (relative to the largest logit), its greedy tokens equal.
"""
import pytest
import torch
import torch.nn.functional as F

from butterfly_b200 import glue

pytestmark = pytest.mark.gpu


def _close(a, b, frac=0.99, ulps=1):
    a, b = a.float(), b.float()
    tol = ulps * (2.0 ** -7) * torch.clamp(b.abs(), min=1.0)
    assert bool(((a - b).abs() <= tol).all()), float((a - b).abs().max())
    assert float((a == b).float().mean()) >= frac


def _norm(dim, seed):
    from transformers.models.qwen3_5.modeling_qwen3_5 import Qwen3_5RMSNorm
    m = Qwen3_5RMSNorm(dim, eps=1e-6).cuda()
    with torch.no_grad():
        m.weight.copy_(torch.randn(dim, generator=torch.Generator().manual_seed(seed)) * 0.1)
    return m.to(torch.bfloat16)


def test_rmsnorm_matches_qwen35_norm():
    g = torch.Generator(device="cuda").manual_seed(1)
    for H in (1024, 2560, 256):
        m = _norm(H, H)
        x = torch.randn(3, 777, H, device="cuda", generator=g).bfloat16()
        r = torch.randn(3, 777, H, device="cuda", generator=g).bfloat16()
        _close(glue.rmsnorm(x, m.weight, m.eps), m(x))
        y, s = glue.rmsnorm(x, m.weight, m.eps, residual=r, want_sum=True)
        assert torch.equal(s, r + x)
        _close(y, m(r + x))
    # strided rows (a slice of a wider buffer)
    m = _norm(1024, 5)
    big = torch.randn(100, 2048, device="cuda", generator=g).bfloat16()
    _close(glue.rmsnorm(big[:, 512:1536], m.weight, m.eps), m(big[:, 512:1536]))


def test_qk_norm_rope_matches_eager():
    from transformers import Qwen3_5TextConfig
    from transformers.models.qwen3_5.modeling_qwen3_5 import Qwen3_5TextRotaryEmbedding, apply_rotary_pos_emb
    cfg = Qwen3_5TextConfig(hidden_size=1024, num_attention_heads=8, num_key_value_heads=2, head_dim=128,
                            num_hidden_layers=1, layer_types=["full_attention"])
    rope = Qwen3_5TextRotaryEmbedding(cfg).cuda()
    g = torch.Generator(device="cuda").manual_seed(2)
    B, T, Hq, Hkv, dh = 2, 700, 8, 2, 128
    qkv = torch.randn(B, T, 2 * Hq * dh + 2 * Hkv * dh, device="cuda", generator=g).bfloat16() * 3
    qg = qkv[..., :2 * Hq * dh].view(B, T, Hq, 2 * dh)
    k_raw = qkv[..., 2 * Hq * dh:2 * Hq * dh + Hkv * dh].view(B, T, Hkv, dh)
    qn, kn = _norm(dh, 11), _norm(dh, 12)
    pos = torch.arange(5000, 5000 + T, device="cuda").view(1, T).expand(B, T)
    cos, sin = rope(qkv, pos)
    q, k = glue.qk_norm_rope(qg[..., :dh], k_raw, qn.weight, kn.weight, cos, sin, qn.eps)
    rq = qn(qg[..., :dh]).transpose(1, 2)
    rk = kn(k_raw).transpose(1, 2)
    rq, rk = apply_rotary_pos_emb(rq, rk, cos, sin)
    _close(q.transpose(1, 2), rq)
    _close(k.transpose(1, 2), rk)
    # decode shapes (one warp per head row instead of a warp per token; the norm's sum runs
    # in another order, so within one rounding step)
    q1, k1 = glue.qk_norm_rope(qg[:, -1:, :, :dh], k_raw[:, -1:], qn.weight, kn.weight, cos[:, -1:], sin[:, -1:],
                               qn.eps)
    _close(q1, q[:, -1:], 0.95)
    _close(k1, k[:, -1:], 0.95)
    _close(q1.transpose(1, 2), rq[:, :, -1:], 0.95)


def test_gate_and_swiglu_match_eager():
    g = torch.Generator(device="cuda").manual_seed(3)
    B, T, H, dh = 2, 333, 8, 128
    o = torch.randn(B, T, H, dh, device="cuda", generator=g).bfloat16()
    qg = torch.randn(B, T, H, 2 * dh, device="cuda", generator=g).bfloat16() * 4
    gate = qg[..., dh:]
    ref = o.reshape(B, T, -1) * torch.sigmoid(gate.reshape(B, T, -1))
    _close(glue.gate_sigmoid_mul(o, gate), ref)
    gu = torch.randn(B, T, 2 * 3584, device="cuda", generator=g).bfloat16() * 3
    _close(glue.swiglu(gu, 3584), F.silu(gu[..., :3584]) * gu[..., 3584:])


def _model(seed=6, layers=3, hidden=512, vocab=1000):
    from transformers import Qwen3_5TextConfig
    from transformers.models.qwen3_5.modeling_qwen3_5 import Qwen3_5ForCausalLM

    from butterfly_b200.integrations import qwen_torch as qt
    qt.patch_qwen35_full_attention_decode()
    cfg = Qwen3_5TextConfig(hidden_size=hidden, num_attention_heads=8, num_key_value_heads=2, head_dim=128,
                            num_hidden_layers=layers, layer_types=["full_attention"] * layers,
                            intermediate_size=1536, vocab_size=vocab)
    torch.manual_seed(seed)
    m = Qwen3_5ForCausalLM(cfg).eval().to(torch.bfloat16).cuda()
    with torch.no_grad():  # non-trivial norm weights
        for n, p in m.named_parameters():
            if "norm" in n:
                p.copy_(torch.randn_like(p.float()).mul(0.1).to(p.dtype))
    qt.swap_qwen_attention_with_butterfly_cuda(m, qt.compressed_config())
    return m


@torch.no_grad()
def test_fused_model_matches_unfused_prefill_and_decode():
    from transformers import DynamicCache

    from butterfly_b200.integrations import qwen_torch as qt
    from butterfly_b200.integrations.qwen_fused import fuse_qwen_decoder_layers, unfuse_qwen_decoder_layers
    m = _model()
    ids = torch.randint(0, 1000, (2, 1500), generator=torch.Generator().manual_seed(7)).cuda()

    def run(cache_kind):
        cache = (qt.make_compressed_cache(m, DynamicCache(config=m.config), max_kv_size=2048, max_chunk_size=512)
                 if cache_kind == "compressed" else DynamicCache(config=m.config))
        out = m(input_ids=ids, past_key_values=cache, use_cache=True)
        logits = [out.logits[:, -64:].float()]
        tok = out.logits[:, -1].argmax(-1, keepdim=True)
        toks = []
        for _ in range(8):
            out = m(input_ids=tok, past_key_values=cache, use_cache=True)
            logits.append(out.logits[:, -1:].float())
            tok = out.logits[:, -1].argmax(-1, keepdim=True)
            toks.append(tok.view(-1).tolist())
        return torch.cat(logits, 1), toks

    ref_c, tok_c = run("compressed")
    ref_h, tok_h = run("hf")
    assert fuse_qwen_decoder_layers(m) == [0, 1, 2]
    got_c, gtok_c = run("compressed")
    for layer in qt.iter_qwen_butterfly_layers(m):
        assert layer.last_profile["fused_glue"] is True
    got_h, gtok_h = run("hf")
    for ref, got in ((ref_c, got_c), (ref_h, got_h)):
        scale = float(ref.abs().max())
        assert float((got - ref).abs().max()) / scale < 3e-2
    assert gtok_c[:4] == tok_c[:4] and gtok_h[:4] == tok_h[:4]
    unfuse_qwen_decoder_layers(m)
    back, _ = run("compressed")
    assert torch.equal(back, ref_c)


@torch.no_grad()
def test_fused_model_graphed_decode():
    from transformers import DynamicCache

    from butterfly_b200.integrations import qwen_torch as qt
    from butterfly_b200.integrations.qwen_fused import fuse_qwen_decoder_layers
    m = _model(seed=8)
    fuse_qwen_decoder_layers(m)
    ids = torch.randint(0, 1000, (1, 2000), generator=torch.Generator().manual_seed(9)).cuda()
    cache = qt.make_compressed_cache(m, DynamicCache(config=m.config), max_kv_size=4096, max_chunk_size=1024)
    out = m(input_ids=ids, past_key_values=cache, use_cache=True, logits_to_keep=1)
    gd = qt.GraphedGreedyDecode(m, cache, out.logits[:, -1].argmax(-1, keepdim=True), 16)
    gd.replay()
    torch.cuda.synchronize()
    assert torch.equal(gd.tokens, gd.eager_tokens)


def test_decode_gemv_kernels_match_eager():
    """The decode projections (fp32 dot products in another order than cuBLAS) against the
    eager ops: within one bf16 rounding step, 90% of elements bit-identical."""
    g = torch.Generator(device="cuda").manual_seed(4)
    H, N, I, Hq, dh = 1024, 2560, 3584, 8, 128
    norm = _norm(H, 21)
    W = (torch.randn(N, H, device="cuda", generator=g) * 0.03).bfloat16()
    Wgu = (torch.randn(2 * I, H, device="cuda", generator=g) * 0.03).bfloat16()
    Wd = (torch.randn(H, I, device="cuda", generator=g) * 0.03).bfloat16()
    Wo = (torch.randn(H, Hq * dh, device="cuda", generator=g) * 0.03).bfloat16()
    for M in (1, 3, 8):
        x = torch.randn(M, H, device="cuda", generator=g).bfloat16()
        r = torch.randn(M, H, device="cuda", generator=g).bfloat16()
        _close(glue.gemv_rmsnorm(x, norm.weight, norm.eps, W), F.linear(norm(x), W), 0.9)
        y, s = glue.gemv_rmsnorm(x, norm.weight, norm.eps, W, residual=r, want_sum=True)
        assert torch.equal(s, x + r)
        _close(y, F.linear(norm(x + r), W), 0.9)
        gu = F.linear(norm(x), Wgu)
        _close(glue.gemv_rmsnorm(x, norm.weight, norm.eps, Wgu, swiglu=True), F.silu(gu[:, :I]) * gu[:, I:], 0.9)
        act = torch.randn(M, I, device="cuda", generator=g).bfloat16()
        _close(glue.gemv(act, Wd), F.linear(act, Wd), 0.9)
        # the residual sum rounds once more: a one-ulp difference in the product can become
        # one ulp of the (larger) sum
        _close(glue.gemv(act, Wd, residual=r), r + F.linear(act, Wd), 0.9, ulps=2)
        o = torch.randn(M, Hq, dh, device="cuda", generator=g).bfloat16()
        qg = torch.randn(M, Hq, 2 * dh, device="cuda", generator=g).bfloat16()
        ref = r + F.linear(o.reshape(M, -1) * torch.sigmoid(qg[..., dh:].reshape(M, -1)), Wo)
        _close(glue.gemv_gated(o, qg[..., dh:], Wo, residual=r), ref, 0.9, ulps=2)


def test_decode_step_with_fused_qk_prep_equals_separate_kernels():
    """bna_decode_step_qk (q/k norm + RoPE inside the decode step) gives bit-identical
    outputs and ring contents to bna_qk_norm_rope followed by bna_decode_step."""
    from transformers import Qwen3_5TextConfig
    from transformers.models.qwen3_5.modeling_qwen3_5 import Qwen3_5TextRotaryEmbedding

    import butterfly_b200 as bb
    from butterfly_b200.cache import CompressedKVCache
    cfg = Qwen3_5TextConfig(hidden_size=1024, num_attention_heads=8, num_key_value_heads=2, head_dim=128,
                            num_hidden_layers=1, layer_types=["full_attention"])
    rope = Qwen3_5TextRotaryEmbedding(cfg).cuda()
    g = torch.Generator(device="cuda").manual_seed(8)
    B, Hq, Hkv, dh, T0 = 3, 8, 2, 128, 1000
    qn, kn = _norm(dh, 31), _norm(dh, 32)
    caches = [CompressedKVCache(block_size=128, local_window_tokens=64, max_chunk_size=1024) for _ in range(2)]
    k0 = torch.randn(B, Hkv, T0, dh, device="cuda", generator=g).bfloat16()
    for c in caches:
        c.append(k0, k0)
    for step in range(150):  # across a block close
        qkv = torch.randn(B, 1, 2 * Hq * dh + 2 * Hkv * dh, device="cuda", generator=g).bfloat16() * 2
        qg = qkv[..., :2 * Hq * dh].view(B, 1, Hq, 2 * dh)
        k_raw = qkv[..., 2 * Hq * dh:2 * Hq * dh + Hkv * dh].view(B, 1, Hkv, dh)
        v = qkv[..., 2 * Hq * dh + Hkv * dh:].view(B, 1, Hkv, dh)
        pos = T0 + step
        cos, sin = rope(qkv, torch.full((B, 1), pos, device="cuda"))
        lay = bb.build_block_butterfly_layout(seq_len=pos + 1, block_size=128, num_key_value_heads=Hkv,
                                              num_key_value_groups=Hq // Hkv, layer_idx=4, local_window_blocks=1,
                                              sink_count=1, partner_count=1, partner_rule="causal_shift")
        q, k = glue.qk_norm_rope(qg[..., :dh], k_raw, qn.weight, kn.weight, cos, sin, qn.eps)
        a = caches[0].decode_step(q.transpose(1, 2), k.transpose(1, 2), v.transpose(1, 2), lay)
        b = caches[1].decode_step(qg[..., :dh].transpose(1, 2), k_raw.transpose(1, 2), v.transpose(1, 2), lay,
                                  qk_prep=(qn.weight, kn.weight, cos, sin, qn.eps))
        assert torch.equal(a, b), step
    for x, y in zip(caches[0].state, caches[1].state):
        assert torch.equal(x, y)



@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("G,W", [(4, 64), (1, 64), (8, 32), (2, 130)])
def test_prefill_gated_epilogue_equals_separate_gate(dtype, G, W):
    """bna_prefill_attention_gated (the output gate applied in the prefill kernel's store)
    writes exactly what bna_prefill_attention followed by bna_gate_sigmoid_mul writes; a
    window beyond the ring-based kernel gates in a separate launch with the same result."""
    import butterfly_b200 as bb
    from butterfly_b200 import attention as A
    g = torch.Generator(device="cuda").manual_seed(9 + G)
    B, Hkv, T, dh = 2, 2, 1000, 128
    Hq = Hkv * G
    qg = (torch.randn(B, T, Hq, 2 * dh, device="cuda", generator=g) * 3).to(dtype)
    q = qg[..., :dh].transpose(1, 2)
    gate = qg[..., dh:].transpose(1, 2)
    k = torch.randn(B, T, Hkv, dh, device="cuda", generator=g).to(dtype).transpose(1, 2)
    v = torch.randn(B, T, Hkv, dh, device="cuda", generator=g).to(dtype).transpose(1, 2)
    lay = bb.build_block_butterfly_layout(seq_len=T, block_size=128, num_key_value_heads=Hkv, num_key_value_groups=G,
                                          layer_idx=3, local_window_blocks=1, sink_count=1, partner_count=1,
                                          partner_rule="causal_shift")
    out, _, _, _ = A.prefill_with_summaries(q, k, v, lay, W, None)
    ref = glue.gate_sigmoid_mul(out.transpose(1, 2), gate.transpose(1, 2))
    got, _, _, _ = A.prefill_with_summaries(q, k, v, lay, W, None, gate=gate)
    assert torch.equal(got.transpose(1, 2).reshape(B, T, Hq * dh), ref)
