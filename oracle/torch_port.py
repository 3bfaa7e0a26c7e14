"""PyTorch-CPU restatement of the reference's vectorised compressed prefill — TEST
INFRASTRUCTURE ONLY (the timed CPU baseline of ``bench.py --impl reference``).

It follows the reference's own CPU algorithm (bna/torch/attention_wayfinder_permute.py
:1046-1122): per-block index tensors (:912-966), fp32 block means cast to the input
dtype (:1022-1043), a gather of each block's raw window and routed summaries, and one
``F.scaled_dot_product_attention`` call with a boolean mask and GQA over the
concatenated keys.  Its outputs are checked against the numpy oracle in the tests.
"""
from __future__ import annotations

import numpy as np
import torch
import torch.nn.functional as F

from .compressed import prefill_index_tensors


def block_means_torch(x: torch.Tensor, block_size: int, num_blocks: int) -> torch.Tensor:
    B, H, T, dh = x.shape
    pad = num_blocks * block_size - T
    xf = x.float()
    if pad:
        xf = F.pad(xf, (0, 0, 0, pad))
    s = xf.view(B, H, num_blocks, block_size, dh).sum(dim=3)
    cnt = torch.clamp(torch.minimum(torch.full((num_blocks,), block_size),
                                    T - torch.arange(num_blocks) * block_size), min=1).float().to(x.device)
    return (s / cnt.view(1, 1, -1, 1)).to(x.dtype)


def prefill(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, neighbors, *, block_size: int,
            window: int, block_chunk: int = 0, index_tensors=None) -> torch.Tensor:
    B, Hq, T, dh = q.shape
    Hkv = k.shape[1]
    N = len(neighbors)
    BS = block_size
    if index_tensors is None:
        index_tensors = [torch.from_numpy(np.ascontiguousarray(a)).to(q.device)
                         for a in prefill_index_tensors(neighbors, T, BS, window)]
    raw_idx, raw_mask, sum_idx, sum_mask = index_tensors
    R, S = raw_idx.shape[1], sum_idx.shape[1]
    ks, vs = block_means_torch(k, BS, N), block_means_torch(v, BS, N)
    pad = N * BS - T
    qb = (F.pad(q, (0, 0, 0, pad)) if pad else q).view(B, Hq, N, BS, dh)
    C = N if block_chunk <= 0 else min(block_chunk, N)
    pieces = []
    for c0 in range(0, N, C):
        c1 = min(N, c0 + C)
        n = c1 - c0
        qc = qb[:, :, c0:c1].transpose(1, 2).reshape(B * n, Hq, BS, dh)
        keys = torch.cat([k[:, :, raw_idx[c0:c1]], ks[:, :, sum_idx[c0:c1]]], dim=3)  # [B,Hkv,n,R+S,dh]
        vals = torch.cat([v[:, :, raw_idx[c0:c1]], vs[:, :, sum_idx[c0:c1]]], dim=3)
        keys = keys.transpose(1, 2).reshape(B * n, Hkv, R + S, dh)
        vals = vals.transpose(1, 2).reshape(B * n, Hkv, R + S, dh)
        mask = torch.cat([raw_mask[c0:c1], sum_mask[c0:c1]], dim=2)                       # [n,BS,R+S]
        mask = mask.unsqueeze(0).expand(B, n, BS, R + S).reshape(B * n, 1, BS, R + S)
        y = F.scaled_dot_product_attention(qc, keys, vals, attn_mask=mask, enable_gqa=Hkv < Hq)
        pieces.append(y.view(B, n, Hq, BS, dh))
    out = torch.cat(pieces, dim=1).transpose(1, 2).reshape(B, Hq, N * BS, dh)
    return out[:, :, :T]


def active(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, neighbors, positions, *, block_size: int,
           window: int) -> torch.Tensor:
    """Active rows over a full K/V history, restating :1125-1197 (gather + masked SDPA)."""
    from .compressed import active_index_tensors
    B, Hq, Tq, dh = q.shape
    Hkv, Tk = k.shape[1], k.shape[2]
    N = len(neighbors)
    ri, rm, si, sm = [torch.from_numpy(np.ascontiguousarray(a)).to(q.device) for a in
                      active_index_tensors(neighbors, Tk, [int(p) for p in positions], block_size, window)]
    ks, vs = block_means_torch(k, block_size, N), block_means_torch(v, block_size, N)
    R, S = ri.shape[1], si.shape[1]
    keys = torch.cat([k[:, :, ri], ks[:, :, si]], dim=3).transpose(1, 2).reshape(B * Tq, Hkv, R + S, dh)
    vals = torch.cat([v[:, :, ri], vs[:, :, si]], dim=3).transpose(1, 2).reshape(B * Tq, Hkv, R + S, dh)
    qr = q.transpose(1, 2).reshape(B * Tq, Hq, 1, dh)
    mask = torch.cat([rm, sm], dim=1).unsqueeze(0).expand(B, Tq, R + S).reshape(B * Tq, 1, 1, R + S)
    y = F.scaled_dot_product_attention(qr, keys, vals, attn_mask=mask, enable_gqa=Hkv < Hq)
    return y.reshape(B, Tq, Hq, dh).transpose(1, 2)


def prefill_shard(q: torch.Tensor, k_ext: torch.Tensor, v_ext: torch.Tensor, k_sum: torch.Tensor,
                  v_sum: torch.Tensor, neighbors, *, block_size: int, window: int, q_pos0: int, kv_pos0: int,
                  total_len: int) -> torch.Tensor:
    """The reference prefill restricted to queries [q_pos0, q_pos0 + Tq) of a total_len-token
    sequence, with keys given from global position kv_pos0 and global block means supplied."""
    B, Hq, Tq, dh = q.shape
    Hkv = k_ext.shape[1]
    BS = block_size
    raw_idx, raw_mask, sum_idx, sum_mask = [torch.from_numpy(np.ascontiguousarray(a)).to(q.device)
                                            for a in prefill_index_tensors(neighbors, total_len, BS, window)]
    b0, nb = q_pos0 // BS, -(-Tq // BS)
    raw_idx = (raw_idx[b0:b0 + nb] - kv_pos0).clamp(0, k_ext.shape[2] - 1)
    raw_mask, sum_idx, sum_mask = raw_mask[b0:b0 + nb], sum_idx[b0:b0 + nb], sum_mask[b0:b0 + nb]
    R, S = raw_idx.shape[1], sum_idx.shape[1]
    pad = nb * BS - Tq
    qb = (F.pad(q, (0, 0, 0, pad)) if pad else q).view(B, Hq, nb, BS, dh).transpose(1, 2).reshape(B * nb, Hq, BS, dh)
    keys = torch.cat([k_ext[:, :, raw_idx], k_sum[:, :, sum_idx]], dim=3).transpose(1, 2).reshape(B * nb, Hkv, R + S, dh)
    vals = torch.cat([v_ext[:, :, raw_idx], v_sum[:, :, sum_idx]], dim=3).transpose(1, 2).reshape(B * nb, Hkv, R + S, dh)
    mask = torch.cat([raw_mask, sum_mask], dim=2).unsqueeze(0).expand(B, nb, BS, R + S).reshape(B * nb, 1, BS, R + S)
    y = F.scaled_dot_product_attention(qb, keys, vals, attn_mask=mask, enable_gqa=Hkv < Hq)
    return y.view(B, nb, Hq, BS, dh).transpose(1, 2).reshape(B, Hq, nb * BS, dh)[:, :, :Tq]
