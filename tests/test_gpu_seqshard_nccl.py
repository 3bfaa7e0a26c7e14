"""Sequence-sharded prefill on 2 GPUs over NCCL (skipped with fewer GPUs): the all-gathered
summaries and halo reproduce the single-GPU result on every rank."""
import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, out_dir):
    import datetime
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    import butterfly_b200 as bb
    from butterfly_b200.seqshard import cuda_ops, sequence_sharded_prefill
    T, W = 16384, 64
    g = torch.Generator().manual_seed(0)
    q = torch.randn(1, 8, T, 128, generator=g).bfloat16().cuda()
    k = torch.randn(1, 2, T, 128, generator=g).bfloat16().cuda()
    v = torch.randn(1, 2, T, 128, generator=g).bfloat16().cuda()
    lay = bb.build_block_butterfly_layout(seq_len=T, block_size=128, num_key_value_heads=2, num_key_value_groups=4,
                                          layer_idx=7, local_window_blocks=1, sink_count=1, partner_count=1,
                                          partner_rule="causal_shift")
    Tl = T // world
    sl = slice(rank * Tl, (rank + 1) * Tl)
    y = sequence_sharded_prefill(q[:, :, sl].contiguous(), k[:, :, sl].contiguous(), v[:, :, sl].contiguous(),
                                 layout=lay, local_window_tokens=W, ops=cuda_ops(lay, W))
    ref = bb.butterfly_compressed_attention(q, k, v, layout=lay, local_window_tokens=W)[:, :, sl]
    torch.cuda.synchronize()
    ok = torch.equal(y, ref)
    open(os.path.join(out_dir, f"ok{rank}"), "w").write("1" if ok else "0")
    dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_two_gpu_sharded_prefill(tmp_path):
    mp.spawn(_worker, args=(2, _port(), str(tmp_path)), nprocs=2)
    assert (tmp_path / "ok0").read_text() == "1" and (tmp_path / "ok1").read_text() == "1"


def _model_worker(rank, world, port, out_dir, fused):
    import datetime
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    from transformers import Qwen3_5TextConfig
    from transformers.models.qwen3_5.modeling_qwen3_5 import Qwen3_5ForCausalLM

    from butterfly_b200.integrations import qwen_torch as qt
    from butterfly_b200.integrations.qwen_fused import fuse_qwen_decoder_layers
    qt.patch_qwen35_full_attention_decode()
    cfg = Qwen3_5TextConfig(hidden_size=512, num_attention_heads=16, num_key_value_heads=4, head_dim=128,
                            num_hidden_layers=3, layer_types=["full_attention"] * 3, intermediate_size=1024,
                            vocab_size=1000)
    torch.manual_seed(11)
    m = Qwen3_5ForCausalLM(cfg).eval().to(torch.bfloat16).cuda()
    qt.swap_qwen_attention_with_butterfly_cuda(m, qt.compressed_config())
    if fused:
        fuse_qwen_decoder_layers(m)
    T = 8192
    ids = torch.randint(0, 1000, (1, T), generator=torch.Generator().manual_seed(12)).cuda()
    Tl = T // world
    hidden = {}
    hook = m.model.norm.register_forward_hook(lambda mod, i, o: hidden.__setitem__("h", o.detach().float().clone()))
    with torch.no_grad():
        m(input_ids=ids, use_cache=False)  # unsharded reference on every rank
        ref = hidden["h"][:, rank * Tl:(rank + 1) * Tl]
        with qt.sequence_sharded(m, T):
            m(input_ids=ids[:, rank * Tl:(rank + 1) * Tl],
              position_ids=torch.arange(rank * Tl, (rank + 1) * Tl, device="cuda").view(1, -1), use_cache=False)
        got = hidden["h"]
        for layer in qt.iter_qwen_butterfly_layers(m):
            assert layer.last_profile["block_sparse_backend"] == "compressed_sequence_shard"
    hook.remove()
    err = float((got - ref).abs().max() / ref.abs().max())
    open(os.path.join(out_dir, f"err{rank}"), "w").write(repr(err))
    dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
@pytest.mark.parametrize("fused", [False, True])
def test_two_gpu_sequence_sharded_model(tmp_path, fused):
    """A swapped (and optionally glue-fused) model's prefill sharded over 2 GPUs: each rank's
    final hidden states equal the unsharded run's rows (GEMMs over different token counts
    may round differently, so within 2e-2 of the largest value)."""
    mp.spawn(_model_worker, args=(2, _port(), str(tmp_path), fused), nprocs=2)
    for r in range(2):
        assert float((tmp_path / f"err{r}").read_text()) < 2e-2
