"""The gate/up GEMM with SwiGLU in its epilogue (bna_gemm_swiglu) against the unfused
path it replaces (cuBLAS GEMM, then the SwiGLU kernel) and an fp32 reference.

The two paths round the same quantities (gate and up products, silu(gate), the product)
to the 16-bit type; they differ only in the order of the fp32 accumulation over K, so a
gate or up value may round to the neighbouring 16-bit value.  The bar: at least 90% of
outputs bit-identical to the unfused path, every output within 2% of the output scale of
it, and the fp32-reference error no larger than the unfused path's own plus 1%.
"""
import pytest
import torch
import torch.nn.functional as F

from butterfly_b200 import glue

pytestmark = pytest.mark.gpu


def _check(h, w, inter):
    got = glue.gemm_swiglu(h, w, inter)
    ref16 = glue.swiglu(F.linear(h, w), inter)
    hf, wf = h.float(), w.float()
    ref32 = F.silu(hf @ wf[:inter].t()) * (hf @ wf[inter:].t())
    scale = float(ref32.abs().max())
    assert got.shape == ref16.shape
    assert float((got.float() - ref16.float()).abs().max()) <= 0.02 * scale
    assert float((got == ref16).float().mean()) >= 0.90
    e_got = float((got.float() - ref32).abs().max())
    e_ref = float((ref16.float() - ref32).abs().max())
    assert e_got <= e_ref + 0.01 * scale, (e_got, e_ref, scale)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("M,K,inter", [(1000, 1024, 3584), (131, 1024, 3584), (640, 2560, 9728), (1, 64, 128),
                                       (4096, 1024, 3584)])
def test_gemm_swiglu_matches_unfused(dtype, M, K, inter):
    g = torch.Generator(device="cuda").manual_seed(M + K)
    h = torch.randn(M, K, device="cuda", generator=g).to(dtype)
    w = (torch.randn(2 * inter, K, device="cuda", generator=g) / K ** 0.5).to(dtype)
    _check(h, w, inter)


def test_gemm_swiglu_strided_rows_and_batch_dims():
    g = torch.Generator(device="cuda").manual_seed(3)
    big = torch.randn(2, 300, 1536, device="cuda", generator=g).bfloat16()
    h = big[..., 256:1280]  # rows of a wider buffer
    w = (torch.randn(2 * 3584, 1024, device="cuda", generator=g) / 32).bfloat16()
    got = glue.gemm_swiglu(h, w, 3584)
    assert got.shape == (2, 300, 3584)
    _check(h.reshape(600, 1024).contiguous(), w, 3584)
    assert torch.equal(got.reshape(600, 3584), glue.gemm_swiglu(h.reshape(600, 1024).contiguous(), w, 3584))


def test_gemm_swiglu_rejects_bad_shapes():
    h = torch.randn(10, 100, device="cuda").bfloat16()
    w = torch.randn(256, 100, device="cuda").bfloat16()
    with pytest.raises(Exception):
        glue.gemm_swiglu(h, w, 128)  # K not a multiple of 64


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("B,T,K,Hq,Hkv,rot", [(1, 1000, 1024, 8, 2, 32), (2, 300, 2560, 16, 4, 64), (1, 70, 1024, 8, 2, 128),
                                                 (1, 8192, 1024, 8, 2, 32)])
def test_gemm_qkv_norm_rope_matches_unfused(dtype, B, T, K, Hq, Hkv, rot):
    """The q/k/v GEMM with the q/k norm + RoPE epilogue against cuBLAS + bna_qk_norm_rope."""
    g = torch.Generator(device="cuda").manual_seed(T + K)
    dh = 128
    N = (2 * Hq + 2 * Hkv) * dh
    h = torch.randn(B, T, K, device="cuda", generator=g).to(dtype)
    w = (torch.randn(N, K, device="cuda", generator=g) / K ** 0.5).to(dtype)
    qw = (torch.randn(dh, device="cuda", generator=g) * 0.1).to(dtype)
    kw = (torch.randn(dh, device="cuda", generator=g) * 0.1).to(dtype)
    pos = torch.arange(T, device="cuda", dtype=torch.float32) + 5
    inv = 1.0 / (10000 ** (torch.arange(0, rot, 2, device="cuda", dtype=torch.float32) / rot))
    fr = torch.cat([pos[:, None] * inv[None], pos[:, None] * inv[None]], -1)
    cos, sin = fr.cos()[None].to(dtype), fr.sin()[None].to(dtype)
    got = glue.gemm_qkv_norm_rope(h, w, Hq, Hkv, qw, kw, cos, sin, 1e-6)
    ref = F.linear(h, w)
    nq = 2 * Hq * dh
    qg = ref[..., :nq].view(B, T, Hq, 2 * dh)
    q_ref, k_ref = glue.qk_norm_rope(qg[..., :dh], ref[..., nq:nq + Hkv * dh].view(B, T, Hkv, dh), qw, kw, cos, sin,
                                     1e-6)
    gg = got[..., :nq].view(B, T, Hq, 2 * dh)
    pairs = [(gg[..., :dh], q_ref), (got[..., nq:nq + Hkv * dh].view(B, T, Hkv, dh), k_ref),
             (gg[..., dh:], qg[..., dh:]), (got[..., nq + Hkv * dh:], ref[..., nq + Hkv * dh:])]
    for a, b in pairs:
        a, b = a.float(), b.float()
        scale = float(b.abs().max())
        assert float((a - b).abs().max()) <= 0.03 * scale
        assert float((a == b).float().mean()) >= 0.85


def _check_residual(h, w, res, got):
    ref16 = res + F.linear(h, w).view(res.shape)  # the eager decoder layer's ops
    ref32 = h.float() @ w.float().t() + res.float()
    scale = float(ref32.abs().max())
    assert float((got.float() - ref16.float()).abs().max()) <= 0.01 * scale
    assert float((got == ref16).float().mean()) >= 0.90
    e_got = float((got.float() - ref32).abs().max())
    e_ref = float((ref16.float() - ref32).abs().max())
    assert e_got <= e_ref + 0.005 * scale, (e_got, e_ref, scale)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("M,K,N", [(1000, 1024, 1024), (131, 3584, 1024), (1, 64, 256), (8192, 3584, 1024),
                                   (700, 9728, 2560)])
def test_gemm_residual_matches_cublas_addmm(dtype, M, K, N):
    """o_proj / down_proj with the residual add in the epilogue (bna_gemm_residual) against
    the eager ops it replaces (cuBLAS projection, then the rounded add), out of place and
    in place."""
    g = torch.Generator(device="cuda").manual_seed(M + K + N)
    h = torch.randn(M, K, device="cuda", generator=g).to(dtype)
    w = (torch.randn(N, K, device="cuda", generator=g) / K ** 0.5).to(dtype)
    res = torch.randn(M, N, device="cuda", generator=g).to(dtype)
    got = glue.gemm_residual(h, w, res)
    _check_residual(h, w, res, got)
    inplace = res.clone()
    out = glue.gemm_residual(h, w, inplace, out=inplace)
    assert out.data_ptr() == inplace.data_ptr()
    assert torch.equal(inplace, got)


def test_gemm_residual_strided_and_rejects_partial_overlap():
    g = torch.Generator(device="cuda").manual_seed(5)
    big = torch.randn(2, 300, 1536, device="cuda", generator=g).bfloat16()
    h = big[..., 256:1280]
    w = (torch.randn(1024, 1024, device="cuda", generator=g) / 32).bfloat16()
    res = torch.randn(2, 300, 1024, device="cuda", generator=g).bfloat16()
    got = glue.gemm_residual(h, w, res)
    assert got.shape == (2, 300, 1024)
    _check_residual(h.reshape(600, 1024).contiguous(), w, res.reshape(600, 1024), got.reshape(600, 1024))
    buf = torch.zeros(601, 1024, device="cuda").bfloat16()
    with pytest.raises(ValueError):
        glue.gemm_residual(torch.randn(600, 1024, device="cuda").bfloat16(), w, buf[:600], out=buf[1:])


def _norm32(x, g, eps):
    xf = x.float()
    return xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps) * (1 + g.float())


@pytest.mark.parametrize("M,K,inter", [(1000, 1024, 3584), (4096, 2560, 9728)])
def test_gemm_swiglu_folded_rmsnorm(M, K, inter):
    """The MLP's RMSNorm folded into the gate/up GEMM (row statistics + (1 + w) in the weight
    columns) against the unfolded path (RMSNorm kernel, then the GEMM): both within the same
    distance of the fp32 reference."""
    g = torch.Generator(device="cuda").manual_seed(M + inter)
    x = (torch.randn(M, K, device="cuda", generator=g) * 3).bfloat16()
    nw = (torch.randn(K, device="cuda", generator=g) * 0.2).bfloat16()
    w = (torch.randn(2 * inter, K, device="cuda", generator=g) / K ** 0.5).bfloat16()
    eps = 1e-6
    wf = (w.float() * (1 + nw.float())[None]).bfloat16()
    got = glue.gemm_swiglu(x, wf, inter, row_ss=glue.row_sumsq(x), norm_eps=eps)
    ref16 = glue.gemm_swiglu(glue.rmsnorm(x, nw, eps), w, inter)
    n32 = _norm32(x, nw, eps)
    ref32 = F.silu(n32 @ w[:inter].float().t()) * (n32 @ w[inter:].float().t())
    scale = float(ref32.abs().max())
    assert float((got.float() - ref16.float()).abs().max()) <= 0.03 * scale
    e_got = float((got.float() - ref32).abs().max())
    e_ref = float((ref16.float() - ref32).abs().max())
    assert e_got <= e_ref + 0.01 * scale, (e_got, e_ref, scale)


def test_gemm_qkv_folded_rmsnorm_and_residual_statistics():
    """Input RMSNorm folded into the q/k/v GEMM, with the row statistics written by the
    residual GEMM that produced its input (bna_gemm_residual ss_out), against the unfolded
    path; and the statistics themselves against torch."""
    g = torch.Generator(device="cuda").manual_seed(11)
    T, K, Hq, Hkv, dh, rot = 3000, 1024, 8, 2, 128, 32
    N = (2 * Hq + 2 * Hkv) * dh
    a = torch.randn(T, 2048, device="cuda", generator=g).bfloat16()
    wo = (torch.randn(K, 2048, device="cuda", generator=g) / 2048 ** 0.5).bfloat16()
    res = torch.randn(T, K, device="cuda", generator=g).bfloat16()
    ss = torch.empty(T, 16, device="cuda", dtype=torch.float32)
    x = glue.gemm_residual(a, wo, res, ss_out=ss)
    want = x.float().pow(2).sum(-1)
    assert torch.allclose(ss.sum(-1), want, rtol=1e-4, atol=1e-3)
    assert torch.allclose(glue.row_sumsq(x)[:, 0], want, rtol=1e-4, atol=1e-3)
    nw = (torch.randn(K, device="cuda", generator=g) * 0.2).bfloat16()
    w = (torch.randn(N, K, device="cuda", generator=g) / K ** 0.5).bfloat16()
    qw = (torch.randn(dh, device="cuda", generator=g) * 0.1).bfloat16()
    kw = (torch.randn(dh, device="cuda", generator=g) * 0.1).bfloat16()
    pos = torch.arange(T, device="cuda", dtype=torch.float32)
    inv = 1.0 / (10000 ** (torch.arange(0, rot, 2, device="cuda", dtype=torch.float32) / rot))
    fr = torch.cat([pos[:, None] * inv[None], pos[:, None] * inv[None]], -1)
    cos, sin = fr.cos()[None].bfloat16(), fr.sin()[None].bfloat16()
    wf = (w.float() * (1 + nw.float())[None]).bfloat16()
    got = glue.gemm_qkv_norm_rope(x.view(1, T, K), wf, Hq, Hkv, qw, kw, cos, sin, 1e-6, row_ss=ss, norm_eps=1e-6)
    ref = glue.gemm_qkv_norm_rope(glue.rmsnorm(x, nw, 1e-6).view(1, T, K), w, Hq, Hkv, qw, kw, cos, sin, 1e-6)
    for lo, hi in ((0, 2 * Hq * dh), (2 * Hq * dh, N)):
        d = (got[..., lo:hi].float() - ref[..., lo:hi].float()).abs()
        scale = float(ref[..., lo:hi].float().abs().max())
        assert float(d.max()) <= 0.04 * scale
        assert float(d.mean()) <= 0.002 * scale
