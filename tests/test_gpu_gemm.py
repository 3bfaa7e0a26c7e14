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
