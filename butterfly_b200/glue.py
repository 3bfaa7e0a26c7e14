"""Fused decoder-layer steps around the compressed attention (through libbna_b200.so).

Each function replaces a chain of eager ops of the Qwen3.5 decoder layer with one sm_100a
kernel and keeps the eager arithmetic: fp32 inside a norm, each elementwise result rounded
to the 16-bit storage type.

  rmsnorm             Qwen3_5RMSNorm (x * rsqrt(mean(x^2) + eps) * (1 + w)), optionally
                      after the residual add, returning the sum as well
  qk_norm_rope        q_norm / k_norm + apply_rotary_pos_emb of extract_qkv_from_qwen_attention
                      (reference bna/integrations/qwen_torch.py:535-573)
  gate_sigmoid_mul    attn_output * sigmoid(gate) (reference qwen_torch.py:1585-1591)
  swiglu              act_fn(gate_proj(x)) * up_proj(x) of Qwen3_5MLP, on a merged gate/up output

Decode-time projections (1..8 tokens), each one HBM-bound weight stream with the step
before it and after it fused in:
  gemv_rmsnorm        W @ rmsnorm(x [+ res]), optionally followed by SwiGLU over [gate; up] rows
  gemv_gated          [res +] W @ (o * sigmoid(gate))
  gemv                [res +] W @ x
"""
from __future__ import annotations

from typing import Optional

import torch

from . import _lib


def _rows(x: torch.Tensor, hidden: int) -> tuple[int, int]:
    """(rows, row stride) of a tensor whose last dim is contiguous and whose leading dims
    flatten to evenly strided rows."""
    if x.shape[-1] != hidden or x.stride(-1) != 1:
        raise ValueError("last dimension must be contiguous and of the normalised size")
    rows = x.numel() // hidden if hidden else 0
    if x.dim() == 1:
        return 1, hidden
    st = x.stride(-2)
    # leading dims must collapse onto the row stride
    exp = st
    for d in range(x.dim() - 2, -1, -1):
        if x.shape[d] > 1 and x.stride(d) != exp:
            raise ValueError("rows of the input must be evenly strided")
        exp *= x.shape[d]
    return rows, st


def _token_stride(x: torch.Tensor) -> int:
    """Stride between consecutive tokens of a [B,T,H,dh] view whose batch and token dims
    flatten to one evenly strided token index (a size-1 dim's stride does not matter)."""
    B, T = int(x.shape[0]), int(x.shape[1])
    ts = x.stride(1) if T > 1 else x.stride(0)
    if B > 1 and T > 1 and x.stride(0) != T * ts:
        raise ValueError("batch and token dims must flatten to one token stride")
    return ts


def rmsnorm(x: torch.Tensor, weight: torch.Tensor, eps: float, residual: Optional[torch.Tensor] = None,
            want_sum: bool = False):
    """RMSNorm over the last dim; with ``residual`` the input is round(x + residual).
    Returns y, or (y, x + residual) when ``want_sum``."""
    _lib.require_cuda(x, weight)
    H = int(x.shape[-1])
    if weight.dtype != x.dtype or weight.numel() != H or not weight.is_contiguous():
        raise ValueError("weight must be a contiguous [hidden] tensor of the input's dtype")
    rows, xs = _rows(x, H)
    out = torch.empty(x.shape, device=x.device, dtype=x.dtype)
    rp, rs, sp, ss = None, 0, None, 0
    s = None
    if residual is not None:
        if residual.shape != x.shape or residual.dtype != x.dtype:
            raise ValueError("residual must match x")
        _, rs = _rows(residual, H)
        rp = residual.data_ptr()
        if want_sum:
            s = torch.empty(x.shape, device=x.device, dtype=x.dtype)
            sp, ss = s.data_ptr(), H
    _lib.check(_lib.lib().bna_rmsnorm(x.data_ptr(), xs, rp, rs, weight.data_ptr(), out.data_ptr(), H, sp, ss, rows,
                                      H, float(eps), _lib.dtype_code(x.dtype), _lib.stream_ptr(x.device)))
    return (out, s) if want_sum else out


def qk_norm_rope(q: torch.Tensor, k: torch.Tensor, q_weight: torch.Tensor, k_weight: torch.Tensor,
                 cos: torch.Tensor, sin: torch.Tensor, eps: float, *, k_out: Optional[torch.Tensor] = None,
                 v: Optional[torch.Tensor] = None, v_out: Optional[torch.Tensor] = None):
    """q [B,T,Hq,128], k [B,T,Hkv,128] (token-major, any token/head strides, dim
    contiguous; q may be the query half of a gated q_proj output) -> normalised, rotated
    q and k as contiguous [B,T,H,128].  cos/sin [B,T,rot] (rot = rotary dims).

    With ``k_out`` (and ``v`` / ``v_out``) the K rows (and a copy of the V rows) are written
    into those contiguous [B,T,Hkv,128] views instead, e.g. the local part of a pre-sized
    buffer whose leading rows hold a sequence shard's halo (B == 1)."""
    _lib.require_cuda(q, k, q_weight, k_weight, cos, sin)
    B, T, Hq, dh = q.shape
    Hkv = int(k.shape[2])
    rot = int(cos.shape[-1])
    if q.stride(-1) != 1 or k.stride(-1) != 1:
        raise ValueError("head_dim must be contiguous")
    qts, kts = _token_stride(q), _token_stride(k)
    cs = cos.reshape(B * T, rot) if cos.shape[0] == B else cos.expand(B, T, rot).reshape(B * T, rot)
    sn = sin.reshape(B * T, rot) if sin.shape[0] == B else sin.expand(B, T, rot).reshape(B * T, rot)
    cs, sn = cs.contiguous(), sn.contiguous()
    for w in (q_weight, k_weight):
        if w.dtype != q.dtype or w.numel() != dh or not w.is_contiguous():
            raise ValueError("norm weights must be contiguous [head_dim] tensors of q's dtype")
    qo = torch.empty((B, T, Hq, dh), device=q.device, dtype=q.dtype)
    for o in (k_out, v_out):
        if o is not None and (tuple(o.shape) != (B, T, Hkv, dh) or not o.is_contiguous()):
            raise ValueError("k_out / v_out must be contiguous [B,T,Hkv,128] views")
    if (v is None) != (v_out is None):
        raise ValueError("v and v_out go together")
    ko = k_out if k_out is not None else torch.empty((B, T, Hkv, dh), device=q.device, dtype=q.dtype)
    vp, vts, vhs, vop = None, 0, 0, None
    if v is not None:
        if v.shape != k.shape or v.stride(-1) != 1:
            raise ValueError("v must be shaped like k with a contiguous head_dim")
        vp, vts, vhs, vop = v.data_ptr(), _token_stride(v), v.stride(2), v_out.data_ptr()
    _lib.check(_lib.lib().bna_qk_norm_rope(
        q.data_ptr(), qts, q.stride(2), k.data_ptr(), kts, k.stride(2), q_weight.data_ptr(),
        k_weight.data_ptr(), cs.data_ptr(), sn.data_ptr(), rot, rot, qo.data_ptr(), ko.data_ptr(), vp, vts, vhs, vop,
        B * T, Hq, Hkv, dh, float(eps), _lib.dtype_code(q.dtype), _lib.stream_ptr(q.device)))
    return qo, ko


def gate_sigmoid_mul(o: torch.Tensor, gate: torch.Tensor) -> torch.Tensor:
    """o [B,T,H,dh] contiguous, gate [B,T,H,dh] (dim contiguous) -> [B,T,H*dh]."""
    _lib.require_cuda(o, gate)
    B, T, H, dh = o.shape
    if not o.is_contiguous():
        raise ValueError("attention output must be contiguous [B,T,H,dh]")
    if gate.stride(-1) != 1:
        raise ValueError("gate head_dim must be contiguous")
    gts = _token_stride(gate)
    out = torch.empty((B, T, H * dh), device=o.device, dtype=o.dtype)
    _lib.check(_lib.lib().bna_gate_sigmoid_mul(o.data_ptr(), gate.data_ptr(), gts, gate.stride(2),
                                               out.data_ptr(), B * T, H, dh, _lib.dtype_code(o.dtype),
                                               _lib.stream_ptr(o.device)))
    return out


def swiglu(gate_up: torch.Tensor, inter: int) -> torch.Tensor:
    """gate_up [..., 2*inter] (gate first, then up) -> silu(gate) * up [..., inter]."""
    _lib.require_cuda(gate_up)
    rows, st = _rows(gate_up, int(gate_up.shape[-1]))
    out = torch.empty((*gate_up.shape[:-1], inter), device=gate_up.device, dtype=gate_up.dtype)
    _lib.check(_lib.lib().bna_swiglu(gate_up.data_ptr(), st, inter, out.data_ptr(), rows, inter,
                                     _lib.dtype_code(gate_up.dtype), _lib.stream_ptr(gate_up.device)))
    return out


def _row_ss_args(row_ss: Optional[torch.Tensor], rows: int, eps: float):
    """(pointer, row stride, parts, eps) of per-row partial sums of squares [rows, parts] fp32."""
    if row_ss is None:
        return None, 0, 0, 0.0
    if (row_ss.dtype != torch.float32 or row_ss.dim() != 2 or int(row_ss.shape[0]) != rows or row_ss.stride(1) != 1
            or row_ss.device.type != "cuda"):
        raise ValueError(f"row_ss must be a [{rows}, parts] float32 CUDA tensor with a contiguous last dim")
    return row_ss.data_ptr(), int(row_ss.stride(0)), int(row_ss.shape[1]), float(eps)


def row_sumsq(x: torch.Tensor) -> torch.Tensor:
    """Per-row sums of squares of x [..., H] as a [rows, 4] float32 tensor (the sum in column 0):
    the ``row_ss`` of the folded-RMSNorm GEMMs for rows no residual GEMM produced."""
    _lib.require_cuda(x)
    H = int(x.shape[-1])
    rows, xs = _rows(x, H)
    out = torch.empty((rows, 4), device=x.device, dtype=torch.float32)
    _lib.check(_lib.lib().bna_row_sumsq(x.data_ptr(), xs, out.data_ptr(), 4, rows, H, _lib.dtype_code(x.dtype),
                                        _lib.stream_ptr(x.device)))
    return out


def gemm_swiglu(h: torch.Tensor, w_gate_up: torch.Tensor, inter: int, row_ss: Optional[torch.Tensor] = None,
                norm_eps: float = 0.0) -> torch.Tensor:
    """silu(h @ Wg^T) * (h @ Wu^T) for h [..., K] and w_gate_up [2*inter, K] = [Wg; Wu], on
    the tcgen05 GEMM with SwiGLU in its epilogue -> [..., inter] (the [.., 2*inter]
    product never reaches HBM).  With ``row_ss`` (per-row partial sums of squares of h,
    [rows, parts] float32) the RMSNorm before the MLP is folded in: h is un-normalised, the
    norm weight (1 + w) is already in w_gate_up's columns, and row m's products are scaled
    by rsqrt(sum(row_ss[m]) / K + norm_eps)."""
    _lib.require_cuda(h, w_gate_up)
    K = int(h.shape[-1])
    rows, ldh = _rows(h, K)
    if w_gate_up.dim() != 2 or int(w_gate_up.shape[0]) != 2 * inter or int(w_gate_up.shape[1]) != K:
        raise ValueError(f"w_gate_up must be [2*inter, K] = [{2 * inter}, {K}], got {tuple(w_gate_up.shape)}")
    if w_gate_up.stride(1) != 1 or w_gate_up.dtype != h.dtype:
        raise ValueError("w_gate_up must be row-major with h's dtype")
    out = torch.empty((*h.shape[:-1], inter), device=h.device, dtype=h.dtype)
    rp, rl, rn, re = _row_ss_args(row_ss, rows, norm_eps)
    _lib.check(_lib.lib().bna_gemm_swiglu(h.data_ptr(), ldh, w_gate_up.data_ptr(), w_gate_up.stride(0),
                                          out.data_ptr(), inter, rows, K, inter, rp, rl, rn, re,
                                          _lib.dtype_code(h.dtype), _lib.stream_ptr(h.device)))
    return out


def gemm_qkv_norm_rope(h: torch.Tensor, w_qkv: torch.Tensor, num_q_heads: int, num_kv_heads: int,
                       q_weight: torch.Tensor, k_weight: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor,
                       eps: float, row_ss: Optional[torch.Tensor] = None, norm_eps: float = 0.0) -> torch.Tensor:
    """h [B,T,K] @ w_qkv^T on the tcgen05 GEMM, w_qkv [N, K] the merged gated q_proj, k_proj and
    v_proj rows (per query head 128 query then 128 gate rows; N = (2 Hq + 2 Hkv) * 128), with
    the q/k RMSNorm and the rotary embedding (cos/sin [B,T,rot] or [1,T,rot]) applied to the
    query and key columns in the epilogue -> [B,T,N] (the layout the projection had).
    ``row_ss`` / ``norm_eps`` fold the layer's input RMSNorm in, as for ``gemm_swiglu``."""
    _lib.require_cuda(h, w_qkv, q_weight, k_weight, cos, sin)
    B, T, K = h.shape
    N = int(w_qkv.shape[0])
    rows, ldh = _rows(h, K)
    if w_qkv.dim() != 2 or int(w_qkv.shape[1]) != K or w_qkv.stride(1) != 1 or w_qkv.dtype != h.dtype:
        raise ValueError("w_qkv must be a row-major [N, K] matrix of h's dtype")
    rot = int(cos.shape[-1])
    cs = cos.reshape(B * T, rot) if cos.shape[0] == B else cos.expand(B, T, rot).reshape(B * T, rot)
    sn = sin.reshape(B * T, rot) if sin.shape[0] == B else sin.expand(B, T, rot).reshape(B * T, rot)
    cs, sn = cs.to(h.dtype).contiguous(), sn.to(h.dtype).contiguous()
    for w in (q_weight, k_weight):
        if w.dtype != h.dtype or w.numel() != 128 or not w.is_contiguous():
            raise ValueError("norm weights must be contiguous [128] tensors of h's dtype")
    out = torch.empty((B, T, N), device=h.device, dtype=h.dtype)
    _lib.check(_lib.lib().bna_gemm_qkv_norm_rope(
        h.data_ptr(), ldh, w_qkv.data_ptr(), w_qkv.stride(0), out.data_ptr(), N, rows, K, N, int(num_q_heads),
        int(num_kv_heads), q_weight.data_ptr(), k_weight.data_ptr(), cs.data_ptr(), sn.data_ptr(), rot, float(eps),
        *_row_ss_args(row_ss, rows, norm_eps), _lib.dtype_code(h.dtype), _lib.stream_ptr(h.device)))
    return out


def gemm_residual(h: torch.Tensor, w: torch.Tensor, residual: torch.Tensor,
                  out: Optional[torch.Tensor] = None, ss_out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """residual + h @ w^T for h [..., K], w [N, K] row-major and residual [..., N] with the
    eager ops' rounding (the projection rounded, then the sum), on the tcgen05 GEMM with the
    residual add in its epilogue.
    ``out`` may be ``residual`` itself (an in-place add, as ``residual.addmm_``).  ``ss_out``
    ([rows, >= 4 N / 256] float32) receives per-row partial sums of squares of the output,
    the ``row_ss`` of a following folded-RMSNorm GEMM."""
    _lib.require_cuda(h, w, residual)
    K = int(h.shape[-1])
    N = int(w.shape[0])
    rows, ldh = _rows(h, K)
    if w.dim() != 2 or int(w.shape[1]) != K or w.stride(1) != 1 or w.dtype != h.dtype:
        raise ValueError("w must be a row-major [N, K] matrix of h's dtype")
    if tuple(residual.shape) != (*h.shape[:-1], N) or residual.dtype != h.dtype:
        raise ValueError(f"residual must be [..., {N}] with h's leading dims and dtype")
    rr, ldr = _rows(residual, N)
    if out is None:
        out = torch.empty(residual.shape, device=h.device, dtype=h.dtype)
    elif tuple(out.shape) != tuple(residual.shape) or out.dtype != h.dtype:
        raise ValueError("out must match residual")
    ro, ldo = _rows(out, N)
    sp, sl = None, 0
    if ss_out is not None:
        if (ss_out.dtype != torch.float32 or ss_out.dim() != 2 or int(ss_out.shape[0]) != rows
                or int(ss_out.shape[1]) < 4 * (N // 256) or ss_out.stride(1) != 1 or ss_out.device != h.device):
            raise ValueError(f"ss_out must be a [{rows}, >= {4 * (N // 256)}] float32 tensor on h's device")
        sp, sl = ss_out.data_ptr(), int(ss_out.stride(0))
    _lib.check(_lib.lib().bna_gemm_residual(h.data_ptr(), ldh, w.data_ptr(), w.stride(0), residual.data_ptr(), ldr,
                                            out.data_ptr(), ldo, rows, K, N, sp, sl, _lib.dtype_code(h.dtype),
                                            _lib.stream_ptr(h.device)))
    return out


def _mat(x: torch.Tensor, K: int) -> tuple[int, int]:
    """(tokens, row stride) of a [M, K] matrix view with a contiguous last dim."""
    if x.dim() != 2 or x.shape[1] != K or x.stride(1) != 1:
        raise ValueError(f"expected a [tokens, {K}] matrix with a contiguous last dim, got {tuple(x.shape)}")
    return int(x.shape[0]), int(x.stride(0)) if x.shape[0] > 1 else K


def gemv_rmsnorm(x: torch.Tensor, norm_weight: torch.Tensor, eps: float, w: torch.Tensor, *,
                 residual: Optional[torch.Tensor] = None, want_sum: bool = False, swiglu: bool = False):
    """W @ rmsnorm(x [+ residual]) for x [M, K] (M <= 8).  With ``swiglu`` W holds the gate
    rows then the up rows and the result is silu(gate) * up [M, N/2].  Returns y, or
    (y, x + residual) when ``want_sum``."""
    _lib.require_cuda(x, norm_weight, w)
    N, K = int(w.shape[0]), int(w.shape[1])
    M, xs = _mat(x, K)
    if not w.is_contiguous() or w.dtype != x.dtype or norm_weight.dtype != x.dtype or norm_weight.numel() != K:
        raise ValueError("weights must be contiguous and of x's dtype")
    out = torch.empty((M, N // 2 if swiglu else N), device=x.device, dtype=x.dtype)
    rp, rs, sp, ss, s = None, 0, None, 0, None
    if residual is not None:
        _, rs = _mat(residual, K)
        rp = residual.data_ptr()
        if want_sum:
            s = torch.empty((M, K), device=x.device, dtype=x.dtype)
            sp, ss = s.data_ptr(), K
    _lib.check(_lib.lib().bna_gemv_rmsnorm(x.data_ptr(), xs, rp, rs, norm_weight.data_ptr(), float(eps), sp, ss,
                                           w.data_ptr(), N, K, int(bool(swiglu)), out.data_ptr(), out.shape[1], M,
                                           _lib.dtype_code(x.dtype), _lib.stream_ptr(x.device)))
    return (out, s) if want_sum else out


def gemv_gated(o: torch.Tensor, gate: torch.Tensor, w: torch.Tensor, residual: Optional[torch.Tensor] = None):
    """[residual +] W @ (o * sigmoid(gate)); o [M,H,dh] contiguous, gate [M,H,dh] (dim contiguous)."""
    _lib.require_cuda(o, gate, w)
    M, H, dh = o.shape
    N, K = int(w.shape[0]), int(w.shape[1])
    if K != H * dh or not o.is_contiguous() or gate.stride(-1) != 1 or not w.is_contiguous():
        raise ValueError("gemv_gated: o must be contiguous [M, H, dh] with H*dh = in_features")
    out = torch.empty((M, N), device=o.device, dtype=o.dtype)
    rp, rs = None, 0
    if residual is not None:
        _, rs = _mat(residual, N)
        rp = residual.data_ptr()
    gts = gate.stride(0) if M > 1 else H * gate.stride(1)
    _lib.check(_lib.lib().bna_gemv_gated(o.data_ptr(), gate.data_ptr(), gts, gate.stride(1), dh, w.data_ptr(), N, K,
                                         rp, rs, out.data_ptr(), N, M, _lib.dtype_code(o.dtype),
                                         _lib.stream_ptr(o.device)))
    return out


def gemv(x: torch.Tensor, w: torch.Tensor, residual: Optional[torch.Tensor] = None) -> torch.Tensor:
    """[residual +] W @ x for x [M, K] (M <= 8)."""
    _lib.require_cuda(x, w)
    N, K = int(w.shape[0]), int(w.shape[1])
    M, xs = _mat(x, K)
    if not w.is_contiguous() or w.dtype != x.dtype:
        raise ValueError("weight must be contiguous and of x's dtype")
    out = torch.empty((M, N), device=x.device, dtype=x.dtype)
    rp, rs = None, 0
    if residual is not None:
        _, rs = _mat(residual, N)
        rp = residual.data_ptr()
    _lib.check(_lib.lib().bna_gemv(x.data_ptr(), xs, w.data_ptr(), N, K, rp, rs, out.data_ptr(), N, M,
                                   _lib.dtype_code(x.dtype), _lib.stream_ptr(x.device)))
    return out

