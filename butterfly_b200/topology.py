"""Butterfly block topology: layout object and builder (host side).

Mirrors ``bna.topology.butterfly`` (butterfly_width :39-42, butterfly_stage_meta :52-65)
and ``bna.torch.attention_wayfinder_permute`` (BlockHamiltonianLayout :382-405,
build_block_butterfly_layout :568-682).  Neighbour rows are produced by the C++ route
code in libbna_b200.so — the same code the kernels evaluate in closed form — so the
layout the caller sees is, by construction, the one the device uses.
"""
from __future__ import annotations

import ctypes
import math
from dataclasses import dataclass, field
from typing import Optional

import numpy as np
import torch

from . import _lib

_VALID_RULES = ("xor", "bit_reversal", "benes", "causal_shift")


def num_blocks_for_seq_len(seq_len: int, block_size: int) -> int:
    """ceil(seq_len / block_size) (reference bna/cycles.py:75-81)."""
    if seq_len <= 0:
        raise ValueError("seq_len must be positive")
    if block_size <= 0:
        raise ValueError("block_size must be positive")
    return (int(seq_len) + int(block_size) - 1) // int(block_size)


def butterfly_width(num_blocks: int) -> int:
    if int(num_blocks) <= 1:
        return 1
    return int(math.ceil(math.log2(int(num_blocks))))


def butterfly_stage_meta(*, num_blocks: int, layer_idx: int, partner_rule: str) -> tuple[int, int]:
    width = butterfly_width(num_blocks)
    stage_count = max(1, 2 * width - 2) if partner_rule == "benes" else width
    return int(layer_idx) % stage_count, stage_count


@dataclass(frozen=True)
class BlockHamiltonianLayout:
    """Block-level routing of one layer (field names as the reference's :382-405).

    ``block_neighbors`` is ``[H_q, N, K]`` int64 (-1 padded), identical for every head.
    ``route`` carries the C-ABI description the kernels consume.
    """

    seq_len: int
    block_size: int
    num_blocks: int
    block_neighbors: torch.Tensor
    block_perm: torch.Tensor
    landmark_blocks: tuple[int, ...]
    sink_blocks: tuple[int, ...]
    num_cycles: int
    strategy: str
    topology_name: str = "hamiltonian"
    stage_idx: int = 0
    stage_count: int = 1
    local_window_blocks: int = 0
    partner_rule: str = "none"
    partner_count: int = 0
    route: Optional[_lib.Route] = field(default=None, compare=False, repr=False)


def make_route(*, seq_len: int, block_size: int, layer_idx: int, local_window_blocks: int,
               sink_count: int, partner_count: int, partner_rule: str) -> _lib.Route:
    if partner_rule not in _VALID_RULES:
        raise ValueError(f"Unsupported block-sparse Butterfly partner rule: {partner_rule!r}")
    r = _lib.Route()
    _lib.check(_lib.lib().bna_route_init(ctypes.byref(r), int(seq_len), int(block_size), int(layer_idx),
                                         int(local_window_blocks), int(sink_count), int(partner_count),
                                         _lib.RULES[partner_rule]))
    return r


def route_neighbors(r: _lib.Route) -> np.ndarray:
    out = np.empty((r.num_blocks, r.max_degree), np.int32)
    _lib.check(_lib.lib().bna_block_neighbors_host(ctypes.byref(r), out.ctypes.data_as(ctypes.POINTER(ctypes.c_int32))))
    return out


def build_block_butterfly_layout(
    *,
    seq_len: int,
    block_size: int,
    num_key_value_heads: int,
    num_key_value_groups: int,
    layer_idx: int,
    local_window_blocks: int = 4,
    sink_count: int = 1,
    partner_count: int = 1,
    partner_rule: str = "xor",
    device: torch.device | None = None,
) -> BlockHamiltonianLayout:
    """Staged Butterfly block topology; same arguments and errors as the reference."""
    if seq_len <= 0:
        raise ValueError("seq_len must be positive")
    if block_size <= 0:
        raise ValueError("block_size must be positive")
    if num_key_value_heads <= 0:
        raise ValueError("num_key_value_heads must be positive")
    if num_key_value_groups <= 0:
        raise ValueError("num_key_value_groups must be positive")
    if local_window_blocks < 0:
        raise ValueError("local_window_blocks must be >= 0")
    if sink_count < 0:
        raise ValueError("sink_count must be >= 0")
    if partner_count < 0:
        raise ValueError("partner_count must be >= 0")
    if partner_rule not in _VALID_RULES:
        raise ValueError(f"Unsupported block-sparse Butterfly partner rule: {partner_rule!r}")
    r = make_route(seq_len=seq_len, block_size=block_size, layer_idx=layer_idx,
                   local_window_blocks=local_window_blocks, sink_count=sink_count,
                   partner_count=partner_count, partner_rule=partner_rule)
    nb = torch.from_numpy(route_neighbors(r).astype(np.int64))
    hq = int(num_key_value_heads) * int(num_key_value_groups)
    dev = device or torch.device("cpu")
    N = int(r.num_blocks)
    return BlockHamiltonianLayout(
        seq_len=int(seq_len), block_size=int(block_size), num_blocks=N,
        block_neighbors=nb.unsqueeze(0).expand(hq, N, nb.shape[1]).to(dev),
        block_perm=torch.arange(N, dtype=torch.long).repeat(hq, 1).to(dev),
        landmark_blocks=(), sink_blocks=tuple(range(min(int(sink_count), N))), num_cycles=1,
        strategy="butterfly", topology_name="butterfly", stage_idx=int(r.stage_idx),
        stage_count=int(r.stage_count), local_window_blocks=int(local_window_blocks),
        partner_rule=str(partner_rule), partner_count=int(partner_count), route=r)


build_block_wayfinder_layout = build_block_butterfly_layout
