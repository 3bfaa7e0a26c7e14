"""C ABI checks that need no GPU: exported symbols, route construction and the host
selection dumps (the same C++ selection code the kernels run), pinned to the reference's
golden vectors."""
import ctypes
import os
import re

import numpy as np
import pytest
import torch

from butterfly_b200 import _lib
from butterfly_b200.attention import active_selection, prefill_selection
from butterfly_b200.topology import build_block_butterfly_layout, make_route, route_neighbors
from oracle import compressed as oc
from tests.golden.inputs import RULES

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
G = np.load(os.path.join(ROOT, "tests", "golden", "golden.npz"))
CASES = ["ref_small", "gqa_ragged", "gqa_w_gt_bs", "xor_rule", "c1_like_small"]


def test_library_exports_every_declared_symbol():
    hdr = open(os.path.join(ROOT, "include", "bna_b200.h")).read()
    declared = set(re.findall(r"BNA_API\s+[\w\s\*]+?\b(bna_\w+)\s*\(", hdr))
    assert declared == set(_lib.EXPORTED)
    L = _lib.lib()
    for name in declared:
        assert hasattr(L, name), name
    assert b"sm_100a" in L.bna_version()


def test_topology_rows_match_reference():
    for ci, (N, layer, rule, lwb, sink, pc, st, sc, width) in enumerate(G["topo_meta"].tolist()):
        r = make_route(seq_len=N * 4, block_size=4, layer_idx=layer, local_window_blocks=lwb,
                       sink_count=sink, partner_count=pc, partner_rule=RULES[rule])
        assert (r.num_blocks, r.width, r.stage_idx, r.stage_count) == (N, width, st, sc)
        np.testing.assert_array_equal(route_neighbors(r), G[f"topo_{ci}"], err_msg=f"case {ci}")


def _layout(name):
    B, Hq, Hkv, T, dh, BS, W, layer, lwb, sink, pc, rule = [int(x) for x in G[f"{name}_cfg"]]
    lay = build_block_butterfly_layout(seq_len=T, block_size=BS, num_key_value_heads=Hkv,
                                       num_key_value_groups=Hq // Hkv, layer_idx=layer,
                                       local_window_blocks=lwb, sink_count=sink, partner_count=pc,
                                       partner_rule=RULES[rule])
    return lay, T, BS, W


@pytest.mark.parametrize("name", CASES + ["c1"])
def test_prefill_selection_bit_exact(name):
    if name == "c1":
        lay = build_block_butterfly_layout(seq_len=4096, block_size=128, num_key_value_heads=2,
                                           num_key_value_groups=4, layer_idx=3, local_window_blocks=1,
                                           sink_count=1, partner_count=1, partner_rule="causal_shift")
        T, BS, W = 4096, 128, 64
        np.testing.assert_array_equal(lay.block_neighbors.numpy(), G["c1_neighbors"])
    else:
        lay, T, BS, W = _layout(name)
        np.testing.assert_array_equal(lay.block_neighbors[0].numpy(), G[f"{name}_neighbors"])
    ls, idx, cnt = prefill_selection(lay, T, W)
    si = G[f"{name}_summary_idx"]
    N, K = si.shape
    sm = np.unpackbits(G[f"{name}_summary_mask"])[: N * (si.shape[1] * BS)].reshape(N, BS, K)[:, 0, :].astype(bool)
    # compare the valid (index where mask) lists in slot order
    for b in range(N):
        assert idx[b, :cnt[b]].tolist() == si[b][sm[b]].tolist(), b
        assert (idx[b, cnt[b]:] == -1).all()
    np.testing.assert_array_equal(ls, G[f"{name}_raw_idx"][:, 0] if name != "c1" else G["c1_raw_idx"][:, 0])


@pytest.mark.parametrize("name", CASES)
def test_active_selection_bit_exact(name):
    lay, T, BS, W = _layout(name)
    pos = G[f"{name}_act_pos"]
    blk, ls, idx, cnt = active_selection(lay, pos, W)
    si, sm = G[f"{name}_act_summary_idx"], G[f"{name}_act_summary_mask"]
    for i in range(len(pos)):
        assert idx[i, :cnt[i]].tolist() == si[i][sm[i]].tolist()
    np.testing.assert_array_equal(ls, np.maximum(0, pos - W + 1))


@pytest.mark.parametrize("N", [1, 2, 5, 100, 1025, 2048, 4097])
@pytest.mark.parametrize("rule", ["causal_shift", "xor", "bit_reversal", "benes"])
def test_route_matches_oracle_large(N, rule):
    from oracle import topology as ot
    for layer in (0, 1, 5, 13):
        r = make_route(seq_len=N * 128, block_size=128, layer_idx=layer, local_window_blocks=1,
                       sink_count=1, partner_count=1, partner_rule=rule)
        ref = np.asarray(ot.block_neighbors_table(N, layer, local_window_blocks=1, sink_count=1,
                                                  partner_count=1, partner_rule=rule))
        np.testing.assert_array_equal(route_neighbors(r), ref)


def test_error_codes_map_to_reference_exceptions():
    with pytest.raises(ValueError):
        make_route(seq_len=0, block_size=128, layer_idx=0, local_window_blocks=1, sink_count=1,
                   partner_count=1, partner_rule="causal_shift")
    with pytest.raises(ValueError):
        build_block_butterfly_layout(seq_len=10, block_size=4, num_key_value_heads=1, num_key_value_groups=1,
                                     layer_idx=0, partner_rule="nope")
    with pytest.raises(_lib.BnaError):
        make_route(seq_len=100, block_size=4, layer_idx=0, local_window_blocks=1, sink_count=1,
                   partner_count=9, partner_rule="xor")
    with pytest.raises(ValueError):
        from butterfly_b200 import butterfly_compressed_attention
        lay = build_block_butterfly_layout(seq_len=16, block_size=4, num_key_value_heads=1,
                                           num_key_value_groups=1, layer_idx=0)
        x = torch.zeros(1, 1, 16, 128)
        butterfly_compressed_attention(x, x, x, layout=lay, local_window_tokens=4)
