"""Multi-rank host logic on CPU: the (batch x head) shard plan, and a
world_size-2 gloo run where each rank regenerates only its batch rows,
computes its shards with the oracle (standing in for its GPU) and the
gathered result equals the single-process result bit for bit."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from metalllm_b200.shards import plan, plan_all


@pytest.mark.parametrize("B,H,world", [(4, 32, 8), (8, 16, 2), (8, 16, 4), (8, 16, 8), (16, 6, 3),
                                       (1, 5, 8), (64, 12, 1)])
def test_plan_covers_every_shard_once(B, H, world):
    plans = plan_all(B, H, world)
    covered = []
    for p in plans:
        covered.extend(range(p.bh_begin, p.bh_end))
        assert 0 <= p.local_bh_begin <= p.local_bh_end <= p.local_batch * H
        assert p.bh_begin - p.b_begin * H == p.local_bh_begin
        assert p.b_end <= B
    assert covered == list(range(B * H))
    sizes = [p.shards for p in plans]
    assert max(sizes) - min(sizes) <= 1


def test_config4_on_8_gpus_is_half_a_batch_each():
    """Config 4: 128 shards, 16 per GPU: each GPU holds one batch row and half its heads."""
    for r in range(8):
        p = plan(4, 32, 8, r)
        assert p.shards == 16 and p.local_batch == 1
        assert (p.local_bh_begin, p.local_bh_end) == ((0, 16) if r % 2 == 0 else (16, 32))


def test_bad_rank():
    with pytest.raises(ValueError):
        plan(2, 2, 2, 2)


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _worker(rank, world, port, B, T, H, D, out_path):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from metalllm_b200.inputs import normal_bf16
        from oracle import oracle as o
        p = plan(B, H, world, rank)
        N = H * D
        row = T * N
        # regenerate only this rank's batch rows (element offsets into the global tensors)
        loc = [normal_bf16(p.local_batch * row, 5, s, offset=p.b_begin * row).reshape(p.local_batch, T, N)
               for s in (1, 2, 3, 4)]
        q, k, v, do = loc
        out = np.zeros_like(q)
        lse = np.zeros((p.local_batch, T, H), np.float32)
        o.flash_forward(q, k, v, H, shard=(p.local_bh_begin, p.local_bh_end), out=out, lse=lse,
                        nthreads=2)
        Dv = o.compute_d(do, out, H, shard=(p.local_bh_begin, p.local_bh_end), nthreads=2)
        dq, dk, dv = o.flash_backward(do, Dv, lse, q, k, v, H,
                                      shard=(p.local_bh_begin, p.local_bh_end), nthreads=2)
        # every rank contributes its shards' head slabs to a global buffer (sum of disjoint parts)
        g_out = torch.zeros((B, T, N), dtype=torch.float64)
        g_dk = torch.zeros((B, T, N), dtype=torch.float64)
        from metalllm_b200.inputs import bf16_bits_to_f32
        for bh in range(p.bh_begin, p.bh_end):
            b, h = divmod(bh, H)
            lb = b - p.b_begin
            cols = slice(h * D, (h + 1) * D)
            g_out[b, :, cols] = torch.from_numpy(bf16_bits_to_f32(out[lb, :, cols]).astype(np.float64))
            g_dk[b, :, cols] = torch.from_numpy(bf16_bits_to_f32(dk[lb, :, cols]).astype(np.float64))
        dist.all_reduce(g_out)
        dist.all_reduce(g_dk)
        # timing reduction used by bench.py: max over ranks
        t = torch.tensor([float(rank + 1)], dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        if rank == 0:
            np.savez(out_path, out=g_out.numpy(), dk=g_dk.numpy(), tmax=t.numpy())
    finally:
        dist.destroy_process_group()


def test_two_gloo_ranks_match_single_process(tmp_path, oracle_mod):
    B, T, H, D = 3, 128, 3, 64   # 9 shards over 2 ranks: a batch row is split between ranks
    world = 2
    out_path = str(tmp_path / "gathered.npz")
    mp.start_processes(_worker, args=(world, _free_port(), B, T, H, D, out_path), nprocs=world,
                       start_method="spawn", join=True)
    got = np.load(out_path)
    from metalllm_b200.inputs import attention_inputs, bf16_bits_to_f32
    x = attention_inputs(B, T, H, D, seed=5)
    out, lse = oracle_mod.flash_forward(x["q"], x["k"], x["v"], H, nthreads=2)
    Dv = oracle_mod.compute_d(x["do"], out, H, nthreads=2)
    dq, dk, dv = oracle_mod.flash_backward(x["do"], Dv, lse, x["q"], x["k"], x["v"], H, nthreads=2)
    assert np.array_equal(got["out"], bf16_bits_to_f32(out).astype(np.float64))
    assert np.array_equal(got["dk"], bf16_bits_to_f32(dk).astype(np.float64))
    assert got["tmax"][0] == world
