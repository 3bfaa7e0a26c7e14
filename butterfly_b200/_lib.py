"""ctypes binding of libbna_b200.so (the C ABI declared in include/bna_b200.h).

The shared library is built in-tree (``butterfly_b200/libbna_b200.so``).  Loading fails
loudly if it is missing: there is no CPU or PyTorch fallback for any operation.
"""
from __future__ import annotations

import ctypes
import os

import torch

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libbna_b200.so")

OK, BAD_SHAPE, BAD_STRIDE, BAD_DTYPE, CAPACITY, UNSUPPORTED, CUDA_ERROR, DEVICE_TIMEOUT = range(8)
BF16, F16 = 0, 1
RULES = {"causal_shift": 0, "xor": 1, "bit_reversal": 2, "benes": 3}

EXPORTED = (
    "bna_last_error", "bna_version", "bna_take_device_error", "bna_set_prefill_trace", "bna_route_init",
    "bna_block_neighbors_host", "bna_prefill_selection_host", "bna_active_selection_host",
    "bna_prefill_selection_device", "bna_compress_blocks", "bna_compress_kv_blocks", "bna_prefill_attention",
    "bna_active_attention", "bna_cache_append", "bna_decode_step", "bna_prefill_attention_static_scratch",
    "bna_rmsnorm", "bna_qk_norm_rope", "bna_gate_sigmoid_mul", "bna_swiglu", "bna_gemv_rmsnorm", "bna_gemv_gated",
    "bna_gemv", "bna_launch_probe", "bna_decode_step_qk", "bna_prefill_attention_gated",
    "bna_gemm_swiglu", "bna_gemm_qkv_norm_rope", "bna_gemm_residual", "bna_row_sumsq",
)


class Tensor4(ctypes.Structure):
    _fields_ = [("data", ctypes.c_void_p), ("size", ctypes.c_int64 * 4), ("stride", ctypes.c_int64 * 4)]


class Route(ctypes.Structure):
    _fields_ = [(n, ctypes.c_int32) for n in (
        "block_size", "num_blocks", "max_degree", "rule", "width", "stage_idx", "stage_count",
        "partner_count", "local_window_blocks", "sink_count")] + [("neighbors", ctypes.c_void_p)]


class BnaError(RuntimeError):
    def __init__(self, status: int, msg: str):
        super().__init__(f"[bna status {status}] {msg}")
        self.status = status


_lib = None


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise ImportError(f"{LIB_PATH} is missing: build it with `python -m butterfly_b200.build`")
        L = ctypes.CDLL(LIB_PATH)
        vp, i32, i64, f32 = ctypes.c_void_p, ctypes.c_int32, ctypes.c_int64, ctypes.c_float
        T4 = ctypes.POINTER(Tensor4)
        R = ctypes.POINTER(Route)
        P32 = ctypes.POINTER(ctypes.c_int32)
        P64 = ctypes.POINTER(ctypes.c_int64)
        sig = {
            "bna_last_error": (ctypes.c_char_p, []),
            "bna_version": (ctypes.c_char_p, []),
            "bna_take_device_error": (i32, [i32, P32]),
            "bna_set_prefill_trace": (i32, [vp]),
            "bna_route_init": (i32, [R, i32, i32, i32, i32, i32, i32, i32]),
            "bna_block_neighbors_host": (i32, [R, P32]),
            "bna_prefill_selection_host": (i32, [R, i32, i32, P32, P32, P32]),
            "bna_active_selection_host": (i32, [R, i32, P64, i32, i32, P32, P32, P32, P32]),
            "bna_prefill_selection_device": (i32, [R, i32, i32, vp, vp, vp]),
            "bna_compress_blocks": (i32, [T4, T4, i32, i32, i64, i32, i64, i64, i64, vp]),
            "bna_compress_kv_blocks": (i32, [T4, T4, T4, T4, i32, i32, i64, i32, i64, i64, i64, vp]),
            "bna_prefill_attention": (i32, [T4, T4, T4, T4, T4, T4, vp, i64, i64, i32, R, i32, i64, i64, i64, f32, vp]),
            "bna_prefill_attention_gated": (i32, [T4, T4, T4, T4, T4, T4, T4, vp, i64, i64, i32, R, i32, i64, i64, i64,
                                                  f32, vp]),
            "bna_active_attention": (i32, [T4, T4, T4, T4, T4, T4, vp, i64, i64, i32, R, i32, vp, i64, i64, i64, i32, f32, vp]),
            "bna_cache_append": (i32, [T4, T4, T4, T4, i32, i64, i64, vp]),
            "bna_prefill_attention_static_scratch": (i32, [T4, T4, T4, T4, vp, i64, i64, i32, R, i32, f32, vp]),
            "bna_rmsnorm": (i32, [vp, i64, vp, i64, vp, vp, i64, vp, i64, i64, i32, f32, i32, vp]),
            "bna_qk_norm_rope": (i32, [vp, i64, i64, vp, i64, i64, vp, vp, vp, vp, i64, i32, vp, vp, vp, i64, i64, vp,
                                       i64, i32, i32, i32, f32, i32, vp]),
            "bna_gate_sigmoid_mul": (i32, [vp, vp, i64, i64, vp, i64, i32, i32, i32, vp]),
            "bna_swiglu": (i32, [vp, i64, i64, vp, i64, i32, i32, vp]),
            "bna_gemm_swiglu": (i32, [vp, i64, vp, i64, vp, i64, i64, i32, i32, vp, i64, i32, f32, i32, vp]),
            "bna_gemm_qkv_norm_rope": (i32, [vp, i64, vp, i64, vp, i64, i64, i32, i32, i32, i32, vp, vp, vp, vp, i32,
                                             f32, vp, i64, i32, f32, i32, vp]),
            "bna_row_sumsq": (i32, [vp, i64, vp, i64, i64, i32, i32, vp]),
            "bna_gemm_residual": (i32, [vp, i64, vp, i64, vp, i64, vp, i64, i64, i32, i32, vp, i64, i32, vp]),
            "bna_gemv_rmsnorm": (i32, [vp, i64, vp, i64, vp, f32, vp, i64, vp, i64, i64, i32, vp, i64, i32, i32, vp]),
            "bna_gemv_gated": (i32, [vp, vp, i64, i64, i32, vp, i64, i64, vp, i64, vp, i64, i32, i32, vp]),
            "bna_launch_probe": (i32, [i32, vp]),
            "bna_decode_step_qk": (i32, [T4, T4, T4, T4, T4, T4, T4, T4, vp, i64, i64, i32, R, i32, i64, i64, i64, i64, i32,
                                         f32, vp, vp, vp, vp, i64, i32, f32, vp]),
            "bna_gemv": (i32, [vp, i64, vp, i64, i64, vp, i64, vp, i64, i32, i32, vp]),
            "bna_decode_step": (i32, [T4, T4, T4, T4, T4, T4, T4, T4, vp, i64, i64, i32, R, i32, i64, i64, i64, i64, i32, f32, vp]),
        }
        for name, (res, args) in sig.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


def check(status: int) -> None:
    if status != OK:
        msg = lib().bna_last_error().decode(errors="replace")
        if status in (BAD_SHAPE, BAD_DTYPE):
            raise ValueError(msg)
        if status == BAD_STRIDE:
            raise ValueError(f"unsupported strides/alignment: {msg}")
        raise BnaError(status, msg)


def dtype_code(dt: torch.dtype) -> int:
    if dt == torch.bfloat16:
        return BF16
    if dt == torch.float16:
        return F16
    raise ValueError(f"compressed attention kernels take bfloat16 or float16 tensors, got {dt}")


_I64x4 = ctypes.c_int64 * 4


def t4(x: torch.Tensor) -> Tensor4:
    if x.dim() != 4:
        raise ValueError(f"expected a 4-D tensor, got shape {tuple(x.shape)}")
    return Tensor4(x.data_ptr(), _I64x4(*x.shape), _I64x4(*x.stride()))


def stream_ptr(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def require_cuda(*xs: torch.Tensor) -> None:
    for x in xs:
        if not x.is_cuda:
            raise ValueError("butterfly_b200 kernels run on CUDA tensors only (no CPU path)")
    dev = xs[0].device
    for x in xs[1:]:
        if x.device != dev:
            raise ValueError("all tensors must be on the same CUDA device")
