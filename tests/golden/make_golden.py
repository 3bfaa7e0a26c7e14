"""Generate golden vectors by running the reference's own PyTorch implementation.

Usage:  python tests/golden/make_golden.py --reference <path-to-Butterfly-checkout>

The reference (Hmbown/Butterfly) is imported read-only from the given checkout; the
functions exercised are
  bna.topology.butterfly.butterfly_stage_meta / butterfly_width
  bna.torch.attention_wayfinder_permute.build_block_butterfly_layout            (:568-682)
  bna.torch.attention_wayfinder_permute._compressed_butterfly_block_index_tensors (:912-966)
  bna.torch.attention_wayfinder_permute._compressed_butterfly_active_index_tensors (:969-1019)
  bna.torch.attention_wayfinder_permute._block_mean_summaries_torch            (:1022-1043)
  bna.torch.attention_wayfinder_permute.butterfly_compressed_attention          (:1046-1122)
  bna.torch.attention_wayfinder_permute.butterfly_compressed_attention_active   (:1125-1197)
Inputs come from numpy's PCG64 generator (seed = crc32 of the case name) and are not
stored: ``tests/golden/inputs.py`` regenerates them bit-identically.
Outputs are written next to this script as ``golden.npz`` (a few MB at most).
"""
from __future__ import annotations

import argparse
import os
import zlib
import sys

import numpy as np


def topology_cases():
    cases = []
    for N in (1, 2, 3, 7, 13, 16, 32, 33, 100, 256, 257):
        for layer in range(0, 12):
            for rule in ("causal_shift", "xor", "bit_reversal", "benes"):
                for (lwb, sink, pc) in ((1, 1, 1), (0, 0, 1), (2, 2, 2), (4, 1, 1)):
                    cases.append((N, layer, rule, lwb, sink, pc))
    for N in (512, 513, 1024, 1025, 2048):
        for layer in (0, 3, 7, 10, 11):
            cases.append((N, layer, "causal_shift", 1, 1, 1))
    return cases


def attention_cases():
    # name, B, Hq, Hkv, T, dh, BS, W, layer, (lwb, sink, pc), rule
    return [
        ("ref_small", 1, 2, 2, 18, 8, 4, 4, 2, (1, 1, 1), "causal_shift"),
        ("gqa_ragged", 2, 8, 2, 200, 16, 32, 16, 3, (1, 1, 1), "causal_shift"),
        ("gqa_w_gt_bs", 1, 4, 1, 300, 32, 16, 40, 5, (2, 1, 1), "causal_shift"),
        ("xor_rule", 1, 4, 2, 257, 16, 16, 8, 1, (1, 1, 2), "xor"),
        ("c1_like_small", 1, 8, 2, 640, 128, 128, 64, 3, (1, 1, 1), "causal_shift"),
    ]


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True)
    ap.add_argument("--out", default=os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden.npz"))
    args = ap.parse_args()
    sys.path.insert(0, os.path.abspath(args.reference))
    import torch
    torch.set_num_threads(max(1, os.cpu_count() or 1))
    from bna.topology.butterfly import butterfly_stage_meta, butterfly_width
    from bna.torch import attention_wayfinder_permute as awp

    out = {}
    # ---- topology: block_neighbors rows (head 0) for many configurations -------------
    rows = []
    for ci, (N, layer, rule, lwb, sink, pc) in enumerate(topology_cases()):
        lay = awp.build_block_butterfly_layout(
            seq_len=N * 4, block_size=4, num_key_value_heads=2, num_key_value_groups=2,
            layer_idx=layer, local_window_blocks=lwb, sink_count=sink, partner_count=pc,
            partner_rule=rule)
        nb = lay.block_neighbors.numpy()
        assert (nb == nb[0:1]).all()
        out[f"topo_{ci}"] = nb[0].astype(np.int32)
        rows.append([N, layer, ("causal_shift", "xor", "bit_reversal", "benes").index(rule),
                     lwb, sink, pc, lay.stage_idx, lay.stage_count, butterfly_width(N)])
    out["topo_meta"] = np.asarray(rows, np.int32)

    # ---- attention / selection cases ---------------------------------------------------
    for (name, B, Hq, Hkv, T, dh, BS, W, layer, (lwb, sink, pc), rule) in attention_cases():
        rng = np.random.default_rng(zlib.crc32(name.encode()))
        q = rng.standard_normal((B, Hq, T, dh), dtype=np.float32)
        k = rng.standard_normal((B, Hkv, T, dh), dtype=np.float32)
        v = rng.standard_normal((B, Hkv, T, dh), dtype=np.float32)
        lay = awp.build_block_butterfly_layout(
            seq_len=T, block_size=BS, num_key_value_heads=Hkv, num_key_value_groups=Hq // Hkv,
            layer_idx=layer, local_window_blocks=lwb, sink_count=sink, partner_count=pc,
            partner_rule=rule)
        y = awp.butterfly_compressed_attention(torch.from_numpy(q), torch.from_numpy(k), torch.from_numpy(v),
                                               layout=lay, local_window_tokens=W)
        ri, rm, si, sm = awp._compressed_butterfly_block_index_tensors(
            lay, T=T, local_window_tokens=W, device=torch.device("cpu"))
        out[f"{name}_out"] = y.numpy().astype(np.float32)
        out[f"{name}_neighbors"] = lay.block_neighbors[0].numpy().astype(np.int32)
        out[f"{name}_raw_idx"] = ri.numpy().astype(np.int32)
        out[f"{name}_raw_mask"] = np.packbits(rm.numpy(), axis=None)
        out[f"{name}_summary_idx"] = si.numpy().astype(np.int32)
        out[f"{name}_summary_mask"] = np.packbits(sm.numpy(), axis=None)
        out[f"{name}_cfg"] = np.asarray([B, Hq, Hkv, T, dh, BS, W, layer, lwb, sink, pc,
                                         ("causal_shift", "xor", "bit_reversal", "benes").index(rule)], np.int64)
        # active rows at a handful of positions, with kv_len = T
        qpos = np.unique(np.concatenate([[0, 1, T - 1], rng.integers(0, T, 6)])).astype(np.int64)
        qa = rng.standard_normal((B, Hq, len(qpos), dh), dtype=np.float32)
        ya = awp.butterfly_compressed_attention_active(
            torch.from_numpy(qa), torch.from_numpy(k), torch.from_numpy(v), layout=lay,
            query_positions=torch.from_numpy(qpos), local_window_tokens=W)
        ari, arm, asi, asm = awp._compressed_butterfly_active_index_tensors(
            lay, kv_len=T, query_positions=torch.from_numpy(qpos), local_window_tokens=W,
            device=torch.device("cpu"))
        out[f"{name}_act_pos"] = qpos
        out[f"{name}_act_out"] = ya.numpy().astype(np.float32)
        out[f"{name}_act_raw_idx"] = ari.numpy().astype(np.int32)
        out[f"{name}_act_raw_mask"] = arm.numpy()
        out[f"{name}_act_summary_idx"] = asi.numpy().astype(np.int32)
        out[f"{name}_act_summary_mask"] = asm.numpy()
        # bf16 block means (pins the reference's fp32-mean-then-cast rounding)
        kb = torch.from_numpy(k).to(torch.bfloat16)
        mb = awp._block_mean_summaries_torch(kb, seq_len=T, block_size=BS, num_blocks=lay.num_blocks)
        out[f"{name}_kbf16_bits"] = kb.view(torch.int16).numpy()
        out[f"{name}_kmean_bf16_bits"] = mb.view(torch.int16).numpy()

    # ---- config 1 at full size: checksums + sampled rows ------------------------------
    B, Hq, Hkv, T, dh, BS, W, layer = 1, 8, 2, 4096, 128, 128, 64, 3
    rng = np.random.default_rng(0)
    q = rng.standard_normal((B, Hq, T, dh), dtype=np.float32) / np.float32(np.sqrt(128.0))
    k = rng.standard_normal((B, Hkv, T, dh), dtype=np.float32)
    v = rng.standard_normal((B, Hkv, T, dh), dtype=np.float32)
    lay = awp.build_block_butterfly_layout(
        seq_len=T, block_size=BS, num_key_value_heads=Hkv, num_key_value_groups=Hq // Hkv,
        layer_idx=layer, local_window_blocks=1, sink_count=1, partner_count=1,
        partner_rule="causal_shift")
    y = awp.butterfly_compressed_attention(torch.from_numpy(q), torch.from_numpy(k), torch.from_numpy(v),
                                           layout=lay, local_window_tokens=W).numpy()
    ri, rm, si, sm = awp._compressed_butterfly_block_index_tensors(
        lay, T=T, local_window_tokens=W, device=torch.device("cpu"))
    sample = np.random.default_rng(1).integers(0, T, 256)
    out["c1_neighbors"] = lay.block_neighbors.numpy().astype(np.int32)
    out["c1_stage"] = np.asarray([lay.stage_idx, lay.stage_count, lay.num_blocks], np.int32)
    out["c1_summary_idx"] = si.numpy().astype(np.int32)
    out["c1_summary_mask"] = np.packbits(sm.numpy(), axis=None)
    out["c1_raw_idx"] = ri.numpy().astype(np.int32)
    out["c1_raw_mask"] = np.packbits(rm.numpy(), axis=None)
    out["c1_sum_per_head"] = y.astype(np.float64).sum(axis=(0, 2, 3))
    out["c1_abssum_per_head"] = np.abs(y.astype(np.float64)).sum(axis=(0, 2, 3))
    out["c1_sample_pos"] = sample
    out["c1_sample_rows"] = y[:, :, sample, :].astype(np.float32)
    np.savez_compressed(args.out, **out)
    print(f"wrote {args.out}: {len(out)} arrays, {os.path.getsize(args.out)/1e6:.2f} MB")


if __name__ == "__main__":
    main()
