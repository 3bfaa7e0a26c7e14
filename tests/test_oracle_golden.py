"""Pin the CPU oracle against vectors produced by the reference's own torch functions."""
import os

import numpy as np
import pytest

from oracle import compressed as oc
from oracle import topology as ot
from tests.golden.inputs import RULES, case_inputs, config1_inputs

G = np.load(os.path.join(os.path.dirname(__file__), "golden", "golden.npz"))
CASES = ["ref_small", "gqa_ragged", "gqa_w_gt_bs", "xor_rule", "c1_like_small"]


def _cfg(name):
    B, Hq, Hkv, T, dh, BS, W, layer, lwb, sink, pc, rule = [int(x) for x in G[f"{name}_cfg"]]
    return dict(B=B, Hq=Hq, Hkv=Hkv, T=T, dh=dh, BS=BS, W=W, layer=layer, lwb=lwb, sink=sink,
                pc=pc, rule=RULES[rule])


def test_topology_rows_match_reference():
    meta = G["topo_meta"]
    for ci, (N, layer, rule, lwb, sink, pc, st, sc, width) in enumerate(meta.tolist()):
        r = RULES[rule]
        assert ot.butterfly_width(N) == width
        assert ot.butterfly_stage_meta(N, layer, r) == (st, sc)
        tab = np.asarray(ot.block_neighbors_table(N, layer, local_window_blocks=lwb, sink_count=sink,
                                                  partner_count=pc, partner_rule=r), np.int32)
        np.testing.assert_array_equal(tab, G[f"topo_{ci}"], err_msg=f"case {ci}")


def test_width_integer_form_matches_float_form():
    for n in list(range(1, 5000)) + [2**k + d for k in range(12, 24) for d in (-1, 0, 1)]:
        assert ot.butterfly_width(n) == (1 if n <= 1 else (n - 1).bit_length())


def test_causal_shift_known_answers():
    # reference tests/pytorch/test_butterfly_topology.py:454-475 and :316-322
    assert ot.butterfly_stage_meta(32, 0, "causal_shift") == (0, 5)
    w = ot.butterfly_width(33)
    for b in range(33):
        for bit in range(w):
            exp = b - (1 << bit)
            assert ot.butterfly_partner_block(b, bit, 33, "causal_shift", w) == (exp if exp >= 0 else None)


@pytest.mark.parametrize("name", CASES)
def test_prefill_selection_tensors_bit_exact(name):
    c = _cfg(name)
    nb = G[f"{name}_neighbors"].tolist()
    ri, rm, si, sm = oc.prefill_index_tensors(nb, c["T"], c["BS"], c["W"])
    np.testing.assert_array_equal(ri, G[f"{name}_raw_idx"])
    np.testing.assert_array_equal(np.packbits(rm, axis=None), G[f"{name}_raw_mask"])
    np.testing.assert_array_equal(si, G[f"{name}_summary_idx"])
    np.testing.assert_array_equal(np.packbits(sm, axis=None), G[f"{name}_summary_mask"])
    tab = ot.block_neighbors_table(-(-c["T"] // c["BS"]), c["layer"], local_window_blocks=c["lwb"],
                                   sink_count=c["sink"], partner_count=c["pc"], partner_rule=c["rule"])
    np.testing.assert_array_equal(np.asarray(tab), G[f"{name}_neighbors"])


@pytest.mark.parametrize("name", CASES)
def test_prefill_output_matches_reference(name):
    c = _cfg(name)
    pos = G[f"{name}_act_pos"]
    q, k, v, qa = case_inputs(name, c["B"], c["Hq"], c["Hkv"], c["T"], c["dh"], pos)
    nb = G[f"{name}_neighbors"].tolist()
    out, lse = oc.prefill_attention(q, k, v, nb, block_size=c["BS"], window=c["W"])
    np.testing.assert_allclose(out, G[f"{name}_out"], atol=3e-4, rtol=3e-4)
    assert np.isfinite(lse).all()


@pytest.mark.parametrize("name", CASES)
def test_active_rows_match_reference(name):
    c = _cfg(name)
    pos = G[f"{name}_act_pos"]
    q, k, v, qa = case_inputs(name, c["B"], c["Hq"], c["Hkv"], c["T"], c["dh"], pos)
    nb = G[f"{name}_neighbors"].tolist()
    ri, rm, si, sm = oc.active_index_tensors(nb, c["T"], pos, c["BS"], c["W"])
    np.testing.assert_array_equal(ri, G[f"{name}_act_raw_idx"])
    np.testing.assert_array_equal(rm, G[f"{name}_act_raw_mask"])
    np.testing.assert_array_equal(si, G[f"{name}_act_summary_idx"])
    np.testing.assert_array_equal(sm, G[f"{name}_act_summary_mask"])
    out, lse = oc.active_attention(qa, k, v, nb, pos, block_size=c["BS"], window=c["W"])
    np.testing.assert_allclose(out, G[f"{name}_act_out"], atol=3e-4, rtol=3e-4)


@pytest.mark.parametrize("name", CASES)
def test_bf16_block_means_match_reference(name):
    c = _cfg(name)
    kb = G[f"{name}_kbf16_bits"].astype(np.int32).astype(np.uint32) << 16
    k = (kb & 0xFFFFFFFF).astype(np.uint32).view(np.float32)
    got = oc.round_bf16(oc.block_means(k, c["BS"]))
    ref = ((G[f"{name}_kmean_bf16_bits"].astype(np.int32).astype(np.uint32) << 16) & 0xFFFFFFFF).view(np.float32)
    # summation order may differ from torch's: allow one bf16 ulp
    ulp = np.abs(ref) * 2.0**-7 + 1e-30
    assert (np.abs(got - ref) <= ulp).all()
    assert (got == ref).mean() > 0.97


def test_config1_full_size():
    q, k, v = config1_inputs()
    nb = G["c1_neighbors"][0].tolist()
    st, sc, N = G["c1_stage"].tolist()
    assert ot.butterfly_stage_meta(N, 3, "causal_shift") == (st, sc)
    ri, rm, si, sm = oc.prefill_index_tensors(nb, 4096, 128, 64)
    np.testing.assert_array_equal(si, G["c1_summary_idx"])
    np.testing.assert_array_equal(np.packbits(sm, axis=None), G["c1_summary_mask"])
    np.testing.assert_array_equal(ri, G["c1_raw_idx"])
    np.testing.assert_array_equal(np.packbits(rm, axis=None), G["c1_raw_mask"])
    out, lse = oc.prefill_attention(q, k, v, nb, block_size=128, window=64)
    np.testing.assert_allclose(out[:, :, G["c1_sample_pos"]], G["c1_sample_rows"], atol=3e-4, rtol=3e-4)
    np.testing.assert_allclose(out.astype(np.float64).sum(axis=(0, 2, 3)), G["c1_sum_per_head"], rtol=1e-4, atol=1e-2)
    np.testing.assert_allclose(np.abs(out.astype(np.float64)).sum(axis=(0, 2, 3)), G["c1_abssum_per_head"], rtol=1e-5)


@pytest.mark.parametrize("name", CASES)
def test_torch_port_matches_reference(name):
    import torch
    from oracle import torch_port
    c = _cfg(name)
    pos = G[f"{name}_act_pos"]
    q, k, v, _ = case_inputs(name, c["B"], c["Hq"], c["Hkv"], c["T"], c["dh"], pos)
    y = torch_port.prefill(torch.from_numpy(q), torch.from_numpy(k), torch.from_numpy(v),
                           G[f"{name}_neighbors"].tolist(), block_size=c["BS"], window=c["W"])
    np.testing.assert_allclose(y.numpy(), G[f"{name}_out"], atol=3e-4, rtol=3e-4)
