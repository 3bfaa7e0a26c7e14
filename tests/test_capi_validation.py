"""Argument validation of the decoder-glue, decode-GEMV and fused decode-step entry points:
every rejected call returns its status before touching a device, so these run without a
GPU.  The Python wrappers refuse CPU tensors (there is no CPU path)."""
import ctypes

import pytest
import torch

from butterfly_b200 import _lib, glue

OK, BAD_SHAPE, BAD_STRIDE, BAD_DTYPE, UNSUPPORTED = _lib.OK, _lib.BAD_SHAPE, _lib.BAD_STRIDE, _lib.BAD_DTYPE, _lib.UNSUPPORTED
P = 1 << 20  # a 16-byte-aligned stand-in pointer: never dereferenced by a rejected call
BF = _lib.BF16


def L():
    return _lib.lib()


def test_rmsnorm_rejections():
    assert L().bna_rmsnorm(P, 1024, None, 0, P, P, 1024, None, 0, 0, 1024, 1e-6, BF, None) == OK  # no rows: no launch
    assert L().bna_rmsnorm(P, 1024, None, 0, P, P, 1024, None, 0, 5, 100, 1e-6, BF, None) == UNSUPPORTED
    assert L().bna_rmsnorm(None, 1024, None, 0, P, P, 1024, None, 0, 5, 1024, 1e-6, BF, None) == BAD_SHAPE
    assert L().bna_rmsnorm(P + 2, 1024, None, 0, P, P, 1024, None, 0, 5, 1024, 1e-6, BF, None) == BAD_STRIDE
    assert L().bna_rmsnorm(P, 1020, None, 0, P, P, 1024, None, 0, 5, 1024, 1e-6, BF, None) == BAD_STRIDE
    assert L().bna_rmsnorm(P, 1024, None, 0, P, P, 1024, P, 1024, 5, 1024, 1e-6, BF, None) == BAD_SHAPE
    assert L().bna_rmsnorm(P, 1024, None, 0, P, P, 1024, None, 0, 5, 1024, 1e-6, 7, None) == BAD_DTYPE
    assert b"bfloat16 or float16" in L().bna_last_error()


def test_qk_norm_rope_rejections():
    f = L().bna_qk_norm_rope
    args = dict(q=P, qt=2560, qh=256, k=P, kt=2560, kh=128, qw=P, kw=P, cos=P, sin=P, cs=32, rot=32, qo=P, ko=P,
                v=None, vt=0, vh=0, vo=None, tokens=4, hq=8, hkv=2, hd=128, eps=1e-6, dt=BF, s=None)

    def call(**kw):
        a = dict(args, **kw)
        return f(*a.values())

    assert call(tokens=0) == OK
    assert call(hd=64) == UNSUPPORTED
    assert call(rot=12) == UNSUPPORTED
    assert call(v=P) == BAD_SHAPE          # v without v_out
    assert call(q=None) == BAD_SHAPE
    assert call(qh=255) == BAD_STRIDE
    assert call(q=P + 2) == BAD_STRIDE


def test_gate_and_swiglu_rejections():
    assert L().bna_gate_sigmoid_mul(P, P, 2560, 256, P, 0, 8, 128, BF, None) == OK
    assert L().bna_gate_sigmoid_mul(P, P, 2560, 256, P, 4, 8, 12, BF, None) == BAD_SHAPE
    assert L().bna_gate_sigmoid_mul(P, P, 2561, 256, P, 4, 8, 128, BF, None) == BAD_STRIDE
    assert L().bna_swiglu(P, 7168, 3584, P, 4, 12, BF, None) == BAD_SHAPE
    assert L().bna_swiglu(P + 8, 7168, 3584, P, 4, 3584, BF, None) == BAD_STRIDE


def test_gemv_rejections():
    # bna_gemv(x, x_stride, w, out_features, in_features, res, res_stride, out, out_stride, tokens, dtype, stream)
    assert L().bna_gemv(P, 1024, P, 1024, 1024, None, 0, P, 1024, 9, BF, None) == UNSUPPORTED   # > 8 tokens
    assert L().bna_gemv(P, 1024, P, 1024, 1000, None, 0, P, 1024, 1, BF, None) == UNSUPPORTED   # K % 256
    assert L().bna_gemv(P, 16384, P, 1024, 16384, None, 0, P, 1024, 1, BF, None) == UNSUPPORTED  # K > 8192
    assert L().bna_gemv(P, 1024, P, 0, 1024, None, 0, P, 1024, 1, BF, None) == BAD_SHAPE
    assert L().bna_gemv(P, 1024, P + 4, 1024, 1024, None, 0, P, 1024, 1, BF, None) == BAD_STRIDE
    # odd row count with SwiGLU
    assert L().bna_gemv_rmsnorm(P, 1024, None, 0, P, 1e-6, None, 0, P, 7167, 1024, 1, P, 3583, 1, BF, None) == BAD_SHAPE
    # sum_out without a residual
    assert L().bna_gemv_rmsnorm(P, 1024, None, 0, P, 1e-6, P, 1024, P, 2560, 1024, 0, P, 2560, 1, BF, None) == BAD_SHAPE
    # gated: in_features not a multiple of head_dim
    assert L().bna_gemv_gated(P, P, 2560, 256, 96, P, 1024, 1024, None, 0, P, 1024, 1, BF, None) == BAD_SHAPE


def test_decode_step_qk_rejections():
    t = _lib.Tensor4()
    r = _lib.Route()
    args = [ctypes.byref(t)] * 8 + [None, 0, 0, BF, ctypes.byref(r), 64, 100, 8512, -1, -1, 5, 0.088, P, P, P, P, 32]
    assert L().bna_decode_step_qk(*args, 12, 1e-6, None) == UNSUPPORTED       # rotary dims not a multiple of 8
    assert L().bna_decode_step_qk(*args, 32, 1e-6, None) != OK                 # empty tensors: rejected before launch
    args_bad = list(args)
    args_bad[20] = None                                                       # null q norm weight
    assert L().bna_decode_step_qk(*args_bad, 32, 1e-6, None) == BAD_SHAPE


def test_gemm_rejections():
    raw = L().bna_gemm_swiglu

    def sw(h, ldh, w, ldw, out, ldo, M, K, inter, dt, s, rs=None, rs_ld=0, rs_parts=0):
        return raw(h, ldh, w, ldw, out, ldo, M, K, inter, rs, rs_ld, rs_parts, 1e-6, dt, s)

    assert sw(P, 1024, P, 1024, P, 3584, 0, 1024, 3584, BF, None) == OK          # no rows: no launch
    assert sw(P, 1024, P, 1024, P, 3584, 8, 1000, 3584, BF, None) == UNSUPPORTED  # K % 64
    assert sw(P, 1024, P, 1024, P, 3584, 8, 1024, 3500, BF, None) == UNSUPPORTED  # inter % 128
    assert sw(P, 1024, P, 1024, P, 3584, 8, 1024, 3584, 7, None) == BAD_DTYPE
    assert sw(P + 2, 1024, P, 1024, P, 3584, 8, 1024, 3584, BF, None) == BAD_STRIDE
    assert sw(P, 1000, P, 1024, P, 3584, 8, 1024, 3584, BF, None) == BAD_STRIDE     # ldh < K
    assert sw(None, 1024, P, 1024, P, 3584, 8, 1024, 3584, BF, None) == BAD_SHAPE
    # folded RMSNorm statistics: parts a positive multiple of 4 within the row stride, aligned
    assert sw(P, 1024, P, 1024, P, 3584, 8, 1024, 3584, BF, None, P, 16, 6) == BAD_STRIDE
    assert sw(P, 1024, P, 1024, P, 3584, 8, 1024, 3584, BF, None, P, 8, 16) == BAD_STRIDE
    assert sw(P, 1024, P, 1024, P, 3584, 8, 1024, 3584, BF, None, P + 4, 16, 16) == BAD_STRIDE
    qk = L().bna_gemm_qkv_norm_rope

    def q(**kw):
        a = dict(h=P, ldh=1024, w=P, ldw=1024, out=P, ldo=2560, M=8, K=1024, N=2560, hq=8, hkv=2, qw=P, kw=P,
                 cos=P, sin=P, rot=32, eps=1e-6, rs=None, rs_ld=0, rs_parts=0, rs_eps=0.0, dt=BF, s=None)
        a.update(kw)
        return qk(*a.values())

    assert q(M=0) == OK
    assert q(N=2304) == BAD_SHAPE       # not (2 Hq + 2 Hkv) * 128
    assert q(N=2432) == UNSUPPORTED     # not a multiple of 256
    assert q(rot=16) == UNSUPPORTED
    assert q(qw=None) == BAD_SHAPE
    assert q(cos=P + 8) == BAD_STRIDE
    assert q(ldo=2048) == BAD_STRIDE
    assert q(rs=P, rs_ld=4, rs_parts=0) == BAD_STRIDE
    res = L().bna_gemm_residual

    def rr(**kw):
        a = dict(h=P, ldh=1024, w=P, ldw=1024, r=P + 4096, ldr=1024, out=P + (1 << 30), ldo=1024, M=8, K=1024, N=1024,
                 ss=None, ss_ld=0, dt=BF, s=None)
        a.update(kw)
        return res(*a.values())

    assert rr(M=0) == OK
    assert rr(N=1000) == UNSUPPORTED
    assert rr(r=None) == BAD_SHAPE
    assert rr(ldr=1000) == BAD_STRIDE
    assert rr(out=P + 4096 + 2048) == BAD_SHAPE      # partial overlap with the residual
    assert rr(ss=P, ss_ld=8) == BAD_STRIDE            # fewer than 4 * N / 256 partial sums per row
    rs = L().bna_row_sumsq
    assert rs(P, 1024, P, 4, 0, 1024, BF, None) == OK
    assert rs(P, 1024, P, 4, 8, 1001, BF, None) == BAD_SHAPE
    assert rs(P, 1024, P, 2, 8, 1024, BF, None) == BAD_STRIDE
    assert rs(P, 1024, P, 4, 8, 1024, 7, None) == BAD_DTYPE


def test_prefill_gated_rejects_null_gate():
    t = _lib.Tensor4()
    r = _lib.Route()
    f = L().bna_prefill_attention_gated
    assert f(ctypes.byref(t), ctypes.byref(t), ctypes.byref(t), ctypes.byref(t), ctypes.byref(t), None,
             ctypes.byref(t), None, 0, 0, BF, ctypes.byref(r), 64, 0, 0, 1, 0.1, None) == BAD_SHAPE


def test_python_wrappers_refuse_cpu_tensors():
    x = torch.zeros(2, 1024, dtype=torch.bfloat16)
    w = torch.zeros(1024, dtype=torch.bfloat16)
    with pytest.raises(ValueError):
        glue.rmsnorm(x, w, 1e-6)
    with pytest.raises(ValueError):
        glue.gemv(x, torch.zeros(512, 1024, dtype=torch.bfloat16))
    with pytest.raises(ValueError):
        glue.swiglu(torch.zeros(2, 2048, dtype=torch.bfloat16), 1024)
    with pytest.raises(ValueError):
        glue.gemm_swiglu(x, torch.zeros(256, 1024, dtype=torch.bfloat16), 128)
    with pytest.raises(ValueError):
        glue.gemm_qkv_norm_rope(x.view(1, 2, 1024), torch.zeros(2560, 1024, dtype=torch.bfloat16), 8, 2,
                                torch.zeros(128, dtype=torch.bfloat16), torch.zeros(128, dtype=torch.bfloat16),
                                torch.zeros(1, 2, 32, dtype=torch.bfloat16), torch.zeros(1, 2, 32, dtype=torch.bfloat16),
                                1e-6)
    from butterfly_b200 import attention as A
    q = torch.zeros(1, 8, 128, 128, dtype=torch.bfloat16)
    with pytest.raises(ValueError):
        A.butterfly_compressed_attention(q, q[:, :2], q[:, :2], layout=None, local_window_tokens=64)
