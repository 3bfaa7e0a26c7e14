"""Sequence-sharded compressed prefill over several GPUs (one process per GPU).

The reference has no sequence parallelism; this is the multi-GPU form of its prefill
(bna/torch/attention_wayfinder_permute.py:1046-1122) for sequences too long for one GPU.
Rank r owns the contiguous token range [r * T_local, (r + 1) * T_local) — whole blocks —
with its Q/K/V already projected (RoPE at global positions).  Exactness needs two
exchanges and nothing else:

  * block summaries: every rank mean-pools its own blocks, then an all-gather assembles the
    global [B, Hkv, N, dh] summary tensor (partner and sink blocks may live on any earlier
    rank).  c4 sizes: 2048 blocks x 4 KV heads x 128 x 2 (K, V) x 2 B = 4.2 MB per layer.
  * halo: the first query block of rank r reaches back W - 1 tokens into rank r - 1, so the
    last W - 1 keys and values of every rank are all-gathered as well (~129 KB per layer).

Both are NCCL all-gathers over NVLink into buffers in each GPU's own HBM; the kernels then
read local memory only.  The data-path functions are injectable so the host logic can be
exercised on CPU ranks (gloo) with reference implementations.
"""
from __future__ import annotations

import math
from dataclasses import dataclass
from typing import Callable, Optional

import torch
import torch.distributed as dist


@dataclass
class ShardOps:
    """Data-path operations used by ``sequence_sharded_prefill``.

    summaries(x, block_size) -> [B, H, N_local, dh] means of the local blocks.
    attend(q, k_ext, v_ext, k_sum, v_sum, q_pos0, kv_pos0, total_len) -> [B, Hq, T_local, dh]
    """

    summaries: Callable
    attend: Callable


def cuda_ops(layout, local_window_tokens: int, scale: Optional[float] = None) -> ShardOps:
    """The sm_100a kernels (compressor + tcgen05 prefill) through the C ABI."""
    from . import attention as A

    def summaries(x, block_size):
        T = int(x.shape[2])
        return A.block_mean_summaries(x, seq_len=T, block_size=block_size, num_blocks=-(-T // block_size))

    def attend(q, k_ext, v_ext, ks, vs, q_pos0, kv_pos0, total_len):
        route, _keep = A.route_for(layout, q.device)
        B, Hq, T, dh = q.shape
        out = torch.empty((B, T, Hq, dh), device=q.device, dtype=q.dtype).transpose(1, 2)
        sc = float(scale) if scale is not None else 1.0 / math.sqrt(dh)
        A.prefill_attention_into(q, k_ext, v_ext, ks, vs, out, None, route, local_window_tokens, sc,
                                 q_pos0=q_pos0, kv_pos0=kv_pos0, total_len=total_len)
        return out

    return ShardOps(summaries=summaries, attend=attend)


def _all_gather(x: torch.Tensor, world: int, group) -> torch.Tensor:
    """[world, *x.shape] (rank-major) via one all-gather of contiguous buffers."""
    if world == 1:
        return x.unsqueeze(0)
    x = x.contiguous()
    out = torch.empty((world * x.shape[0],) + tuple(x.shape[1:]), dtype=x.dtype, device=x.device)
    dist.all_gather_into_tensor(out, x, group=group)  # concatenated along dim 0
    return out.view((world,) + tuple(x.shape))


def shard_exchange(k_ext: torch.Tensor, v_ext: torch.Tensor, halo: int, block_size: int, ops: ShardOps,
                   group=None):
    """The two exchanges of a sequence-sharded layer, on pre-sized K/V buffers.

    ``k_ext`` / ``v_ext`` [B, Hkv, halo + T_local, dh] hold this rank's keys / values at
    rows [halo, halo + T_local) (global positions rank * T_local onwards); their first
    ``halo`` rows are filled here with the previous rank's last ``halo`` rows (rank 0 leaves
    them unused).  Returns (global K summaries, global V summaries, the K/V views the
    attention reads, their global start position)."""
    world = dist.get_world_size(group) if dist.is_initialized() else 1
    rank = dist.get_rank(group) if dist.is_initialized() else 0
    h = int(halo)
    B, Hkv, Tx, dh = k_ext.shape
    Tl = Tx - h
    k, v = k_ext[:, :, h:], v_ext[:, :, h:]
    # 1. local summaries -> global summaries (rank-major blocks == global block order)
    ks_l = ops.summaries(k, block_size)
    vs_l = ops.summaries(v, block_size)
    g = _all_gather(torch.stack([ks_l, vs_l]), world, group)       # [world, 2, B, Hkv, Nl, dh]
    g = g.permute(1, 2, 3, 0, 4, 5).reshape(2, B, Hkv, world * ks_l.shape[2], dh)
    # 2. halo: the last h rows of every rank; rank r uses rank r - 1's, written in place
    if h > 0 and world > 1:
        hg = _all_gather(torch.stack([k[:, :, Tl - h:], v[:, :, Tl - h:]]), world, group)
        if rank > 0:
            k_ext[:, :, :h].copy_(hg[rank - 1, 0])
            v_ext[:, :, :h].copy_(hg[rank - 1, 1])
    if rank > 0 and h > 0:
        return g[0], g[1], k_ext, v_ext, rank * Tl - h
    return g[0], g[1], k, v, 0


def sequence_sharded_prefill(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, *, layout,
                             local_window_tokens: int, ops: ShardOps, group=None) -> torch.Tensor:
    """Compressed Butterfly prefill of this rank's token shard.

    q [B, Hq, T_local, dh], k / v [B, Hkv, T_local, dh] hold global positions
    [rank * T_local, (rank + 1) * T_local).  T_local must be a multiple of the block size and
    equal on every rank; ``layout`` describes the whole sequence (world * T_local tokens).
    Returns this rank's [B, Hq, T_local, dh] output.  K and V are staged into buffers with
    W - 1 leading halo rows (one copy of the local rows); callers that can produce K / V
    straight into such buffers use ``shard_exchange`` directly and skip that copy.
    """
    world = dist.get_world_size(group) if dist.is_initialized() else 1
    rank = dist.get_rank(group) if dist.is_initialized() else 0
    B, Hq, Tl, dh = q.shape
    BS = int(layout.block_size)
    W = int(local_window_tokens)
    check_shard(Tl, BS, W, world, layout)
    h = W - 1
    Hkv = int(k.shape[1])
    k_ext = torch.empty((B, Hkv, h + Tl, dh), dtype=k.dtype, device=k.device)
    v_ext = torch.empty_like(k_ext)
    k_ext[:, :, h:].copy_(k)
    v_ext[:, :, h:].copy_(v)
    ks, vs, ka, va, kv_pos0 = shard_exchange(k_ext, v_ext, h, BS, ops, group)
    return ops.attend(q, ka, va, ks, vs, rank * Tl, kv_pos0, world * Tl)


def check_shard(Tl: int, BS: int, W: int, world: int, layout) -> None:
    if Tl % BS != 0:
        raise ValueError(f"each rank must own whole blocks: T_local={Tl} is not a multiple of {BS}")
    if int(layout.num_blocks) != world * Tl // BS:
        raise ValueError("layout must describe the whole sharded sequence")
    if W - 1 > Tl:
        raise ValueError("the local window must not reach past the previous rank")
