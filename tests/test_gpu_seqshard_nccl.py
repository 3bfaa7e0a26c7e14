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
