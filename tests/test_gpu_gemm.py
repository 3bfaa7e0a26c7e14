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
