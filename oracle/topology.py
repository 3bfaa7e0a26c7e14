"""Oracle restatement of the butterfly block topology (test infrastructure only).

Follows ``bna/topology/butterfly.py`` of the reference:
  butterfly_width          :39-42
  bit_reverse              :45-49
  butterfly_stage_meta     :52-65
  butterfly_partner_bits   :77-105
  butterfly_partner_block  :108-141
and the row construction of ``build_block_butterfly_layout``
(``bna/torch/attention_wayfinder_permute.py:568-682``) plus
``num_blocks_for_seq_len`` (``bna/cycles.py:75-81``).
"""
from __future__ import annotations

import math

RULES = ("xor", "bit_reversal", "benes", "causal_shift")


def num_blocks_for_seq_len(seq_len: int, block_size: int) -> int:
    # bna/cycles.py:75-81
    if seq_len <= 0 or block_size <= 0:
        raise ValueError("seq_len and block_size must be positive")
    return (int(seq_len) + int(block_size) - 1) // int(block_size)


def butterfly_width(num_blocks: int) -> int:
    # butterfly.py:39-42 (ceil(log2 N), 1 for N <= 1)
    if int(num_blocks) <= 1:
        return 1
    return int(math.ceil(math.log2(int(num_blocks))))


def bit_reverse(value: int, width: int) -> int:
    # butterfly.py:45-49
    out = 0
    for i in range(int(width)):
        out = (out << 1) | ((int(value) >> i) & 1)
    return out


def butterfly_stage_meta(num_blocks: int, layer_idx: int, partner_rule: str) -> tuple[int, int]:
    # butterfly.py:52-65
    width = butterfly_width(num_blocks)
    stage_count = max(1, 2 * width - 2) if partner_rule == "benes" else width
    return int(layer_idx) % stage_count, stage_count


def butterfly_partner_bits(stage_idx: int, stage_count: int, width: int,
                           partner_count: int, partner_rule: str) -> list[int]:
    # butterfly.py:77-105
    if width <= 0 or partner_count <= 0:
        return []
    if partner_rule == "benes":
        base = 0 if stage_count <= 1 else stage_idx % stage_count

        def phase_to_bit(phase: int) -> int:
            if width <= 1:
                return 0
            return phase if phase < width else 2 * width - 2 - phase

        return [phase_to_bit((base + o) % stage_count) for o in range(partner_count)]
    return [(stage_idx + o) % width for o in range(partner_count)]


def butterfly_partner_block(block_idx: int, bit_idx: int, num_blocks: int,
                            partner_rule: str, width: int | None = None) -> int | None:
    # butterfly.py:108-141 (rules named by the block-sparse layout builder)
    w = butterfly_width(num_blocks) if width is None else int(width)
    if bit_idx < 0 or bit_idx >= max(1, w):
        return None
    if partner_rule == "causal_shift":
        partner = block_idx - (1 << bit_idx)
    elif partner_rule in ("xor", "benes"):
        partner = block_idx ^ (1 << bit_idx)
    elif partner_rule == "bit_reversal":
        partner = bit_reverse(bit_reverse(block_idx, w) ^ (1 << bit_idx), w)
    else:
        raise ValueError(f"unsupported partner rule {partner_rule!r}")
    if partner < 0 or partner >= num_blocks or partner > block_idx:
        return None
    return partner


def block_neighbor_rows(num_blocks: int, layer_idx: int, *, local_window_blocks: int,
                        sink_count: int, partner_count: int, partner_rule: str) -> list[list[int]]:
    """Per-block ordered-unique neighbour rows (attention_wayfinder_permute.py:630-652)."""
    width = butterfly_width(num_blocks)
    stage_idx, stage_count = butterfly_stage_meta(num_blocks, layer_idx, partner_rule)
    bits = butterfly_partner_bits(stage_idx, stage_count, width, partner_count, partner_rule)
    sinks = list(range(min(sink_count, num_blocks)))
    rows = []
    for b in range(num_blocks):
        row = [b]
        for off in range(1, local_window_blocks + 1):
            if b - off < 0:
                break
            row.append(b - off)
        for bit in bits:
            p = butterfly_partner_block(b, bit, num_blocks, partner_rule, width)
            if p is not None:
                row.append(p)
        row.extend(sinks)
        seen, out = set(), []
        for v in row:
            if v not in seen:
                seen.add(v)
                out.append(v)
        rows.append([v for v in out if 0 <= v < num_blocks])
    return rows


def block_neighbors_table(num_blocks: int, layer_idx: int, **kw) -> "list[list[int]]":
    """Rows padded with -1 to max_degree (max_degree starts at 1, as the reference)."""
    rows = block_neighbor_rows(num_blocks, layer_idx, **kw)
    k = max([1] + [len(r) for r in rows])
    return [r + [-1] * (k - len(r)) for r in rows]
