"""The static-scratch prefill entry point, for callers that cannot allocate device memory.

Hosts that embed this library inside another framework's graph-capture or allocator
regions, or that run with a fixed device-memory plan, cannot cudaMalloc the two block-mean
buffers the regular prefill path needs.  bna_prefill_attention_static_scratch keeps them
in a fixed device array of the library.  This test calls it through the C ABI
twice in a row (different problems, so the second call starts from the first call's
leftover scratch contents) and checks each result against the regular entry point, with
the same tolerance as the other parity tests.  It lives in its own file, collected last.
"""
import ctypes
import math

import numpy as np
import pytest
import torch

import butterfly_b200 as bb
from butterfly_b200 import _lib

pytestmark = pytest.mark.gpu

TOL = 2e-2


def _case(B, Hq, Hkv, T, layer, seed, dtype=torch.bfloat16):
    g = torch.Generator(device="cuda").manual_seed(seed)
    q = torch.randn(B, Hq, T, 128, device="cuda", generator=g).to(dtype)
    k = torch.randn(B, Hkv, T, 128, device="cuda", generator=g).to(dtype)
    v = torch.randn(B, Hkv, T, 128, device="cuda", generator=g).to(dtype)
    lay = bb.build_block_butterfly_layout(seq_len=T, block_size=128, num_key_value_heads=Hkv,
                                          num_key_value_groups=Hq // Hkv, layer_idx=layer, local_window_blocks=1,
                                          sink_count=1, partner_count=1, partner_rule="causal_shift")
    return q, k, v, lay


def _static_call(q, k, v, lay):
    B, Hq, T, dh = q.shape
    out = torch.empty_like(q)
    lse = torch.empty(B, Hq, T, device=q.device, dtype=torch.float32)
    tq, tk, tv, to = (_lib.t4(x) for x in (q, k, v, out))
    _lib.check(_lib.lib().bna_prefill_attention_static_scratch(
        ctypes.byref(tq), ctypes.byref(tk), ctypes.byref(tv), ctypes.byref(to), lse.data_ptr(),
        lse.stride(0), lse.stride(1), _lib.dtype_code(q.dtype), ctypes.byref(lay.route), 64, 1.0 / math.sqrt(dh),
        _lib.stream_ptr(q.device)))
    return out, lse


def _check(B, Hq, Hkv, T, layer, seed, dtype=torch.bfloat16):
    q, k, v, lay = _case(B, Hq, Hkv, T, layer, seed, dtype)
    got, got_lse = _static_call(q, k, v, lay)
    ref, ref_lse = bb.butterfly_compressed_attention(q, k, v, layout=lay, local_window_tokens=64, return_lse=True)
    torch.cuda.synchronize()
    assert np.abs((got.float() - ref.float()).cpu().numpy()).max() <= TOL
    assert np.abs((got_lse - ref_lse).cpu().numpy()).max() <= 1e-3


def test_static_scratch_matches_regular_entry_point_twice():
    for (B, Hq, Hkv, T, layer, seed) in [(2, 8, 2, 5000, 3, 1), (1, 8, 2, 1300, 6, 2)]:
        _check(B, Hq, Hkv, T, layer, seed)


def test_static_scratch_fp16_and_full_capacity():
    _check(1, 8, 2, 3000, 4, 3, dtype=torch.float16)
    # B * Hkv * num_blocks = 8 * 2 * 1024 = 16384: the V means end at the array's last byte
    _check(8, 8, 2, 131072, 5, 4)


def test_static_scratch_rejects_oversized_problem():
    B, Hkv, T = 8, 8, 262144  # block means need 2 * 8 * 8 * 2048 * 256 B = 64 MiB > 8 MiB
    lay = bb.build_block_butterfly_layout(seq_len=T, block_size=128, num_key_value_heads=Hkv,
                                          num_key_value_groups=1, layer_idx=0, local_window_blocks=1,
                                          sink_count=1, partner_count=1, partner_rule="causal_shift")
    x = torch.empty(1, 1, T, 128, dtype=torch.bfloat16, device="cuda").expand(B, Hkv, T, 128)
    tx = _lib.t4(x)
    lse = torch.empty(1, 1, T, device="cuda")
    rc = _lib.lib().bna_prefill_attention_static_scratch(
        ctypes.byref(tx), ctypes.byref(tx), ctypes.byref(tx), ctypes.byref(tx), lse.data_ptr(), lse.stride(0),
        lse.stride(1), _lib.BF16, ctypes.byref(lay.route), 64, 0.088, _lib.stream_ptr(x.device))
    assert rc == _lib.CAPACITY
    assert b"static scratch" in _lib.lib().bna_last_error()
