"""Sequence-sharded prefill host logic on CPU ranks (gloo, world sizes 2 and 4): the
summary all-gather and the window halo make every shard equal to the unsharded
reference, with reference (oracle) data-path ops standing in for the GPU kernels."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, T, BS, W, layer, q_np, k_np, v_np, out_dir, drop_rank):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    import datetime
    # Spawned interpreters can take tens of seconds to import torch on a loaded host, so the
    # rendezvous gets a generous limit; the dropped-rank case keeps a short one so that its
    # collective fails quickly once the peer has gone.
    limit = 20 if drop_rank >= 0 else 180
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=limit))
    from butterfly_b200.seqshard import ShardOps, sequence_sharded_prefill
    from oracle import topology as ot
    from oracle import torch_port

    class _Layout:
        block_size = BS
        num_blocks = T // BS

    nb = ot.block_neighbors_table(T // BS, layer, local_window_blocks=1, sink_count=1, partner_count=1,
                                  partner_rule="causal_shift")
    ops = ShardOps(
        summaries=lambda x, bs: torch_port.block_means_torch(x, bs, x.shape[2] // bs),
        attend=lambda q, ke, ve, ks, vs, qp0, kp0, tot: torch_port.prefill_shard(
            q, ke, ve, ks, vs, nb, block_size=BS, window=W, q_pos0=qp0, kv_pos0=kp0, total_len=tot))
    Tl = T // world
    sl = slice(rank * Tl, (rank + 1) * Tl)
    q, k, v = (torch.from_numpy(a[:, :, sl].copy()) for a in (q_np, k_np, v_np))
    try:
        if rank == drop_rank:
            raise SystemExit(3)  # this rank leaves before the collectives
        y = sequence_sharded_prefill(q, k, v, layout=_Layout, local_window_tokens=W, ops=ops)
        np.save(os.path.join(out_dir, f"y{rank}.npy"), y.numpy())
    except RuntimeError as exc:  # a peer vanished: the collective times out with an error
        open(os.path.join(out_dir, f"err{rank}.txt"), "w").write(str(exc))
    finally:
        if dist.is_initialized() and rank != drop_rank:
            dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4])
def test_sharded_equals_unsharded(world, tmp_path):
    from oracle import topology as ot
    from oracle import torch_port
    T, BS, W, layer = 1024, 64, 24, 3
    g = np.random.default_rng(5)
    q = g.standard_normal((1, 4, T, 16), dtype=np.float32)
    k = g.standard_normal((1, 2, T, 16), dtype=np.float32)
    v = g.standard_normal((1, 2, T, 16), dtype=np.float32)
    mp.spawn(_worker, args=(world, _free_port(), T, BS, W, layer, q, k, v, str(tmp_path), -1), nprocs=world)
    got = np.concatenate([np.load(tmp_path / f"y{r}.npy") for r in range(world)], axis=2)
    nb = ot.block_neighbors_table(T // BS, layer, local_window_blocks=1, sink_count=1, partner_count=1,
                                  partner_rule="causal_shift")
    ref = torch_port.prefill(torch.from_numpy(q), torch.from_numpy(k), torch.from_numpy(v), nb,
                             block_size=BS, window=W).numpy()
    np.testing.assert_allclose(got, ref, atol=1e-5, rtol=1e-5)


def test_dropped_rank_surfaces_as_error(tmp_path):
    T, BS, W = 512, 64, 24
    g = np.random.default_rng(6)
    q = g.standard_normal((1, 2, T, 8), dtype=np.float32)
    k = g.standard_normal((1, 1, T, 8), dtype=np.float32)
    ctx = mp.start_processes(_worker, args=(2, _free_port(), T, BS, W, 1, q, k, k, str(tmp_path), 1), nprocs=2,
                             join=False, start_method="spawn")
    for p in ctx.processes:
        p.join(60)
    assert all(not p.is_alive() for p in ctx.processes)
    assert (tmp_path / "err0.txt").exists() or not (tmp_path / "y0.npy").exists()
