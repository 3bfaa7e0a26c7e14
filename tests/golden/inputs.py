"""Regenerate the seeded inputs used by ``make_golden.py`` (numpy PCG64, bit-stable)."""
from __future__ import annotations

import zlib

import numpy as np

RULES = ("causal_shift", "xor", "bit_reversal", "benes")


def case_inputs(name: str, B: int, Hq: int, Hkv: int, T: int, dh: int, act_positions: np.ndarray):
    """Return q, k, v, q_active exactly as the generator drew them."""
    rng = np.random.default_rng(zlib.crc32(name.encode()))
    q = rng.standard_normal((B, Hq, T, dh), dtype=np.float32)
    k = rng.standard_normal((B, Hkv, T, dh), dtype=np.float32)
    v = rng.standard_normal((B, Hkv, T, dh), dtype=np.float32)
    rng.integers(0, T, 6)  # the draw that picked the active positions
    qa = rng.standard_normal((B, Hq, len(act_positions), dh), dtype=np.float32)
    return q, k, v, qa


def config1_inputs():
    """Config 1: B1, Hq8/Hkv2, T4096, dh128; N(0,1) from seed 0, q scaled by 1/sqrt(128)."""
    rng = np.random.default_rng(0)
    q = rng.standard_normal((1, 8, 4096, 128), dtype=np.float32) / np.float32(np.sqrt(128.0))
    k = rng.standard_normal((1, 2, 4096, 128), dtype=np.float32)
    v = rng.standard_normal((1, 2, 4096, 128), dtype=np.float32)
    return q, k, v
