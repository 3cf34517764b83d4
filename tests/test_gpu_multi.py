"""Two ranks on two GPUs: each rank computes its (batch, head) shards through
the *_shard entry points on its own device (metalllm_b200.shards.plan); the
gathered results equal a single-GPU run bit for bit (independent shards,
deterministic kernels; dQ to fp32 rounding).  Skipped with fewer than two GPUs."""
import os
import socket

import numpy as np
import pytest

torch = pytest.importorskip("torch")

pytestmark = pytest.mark.gpu


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _worker(rank, world, port, B, T, H, D, out_path):
    import datetime

    import torch.distributed as dist

    from metalllm_b200 import attention as A
    from metalllm_b200.inputs import normal_bf16
    from metalllm_b200.shards import plan

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=120))
    try:
        p = plan(B, H, world, rank)
        N = H * D
        row = T * N
        dev = torch.device("cuda", rank)
        up = lambda a: torch.from_numpy(a.view(np.int16)).view(torch.bfloat16).to(dev)
        loc = [up(normal_bf16(p.local_batch * row, 3, s, offset=p.b_begin * row)
                  .reshape(p.local_batch, T, N)) for s in (1, 2, 3, 4)]
        q, k, v, do = loc
        prm = A.make_params(T, H, D)
        sh = (p.local_bh_begin, p.local_bh_end)
        out = torch.zeros_like(q)
        l = torch.zeros(p.local_batch, T, H, device=dev)
        Dv = torch.zeros(p.local_batch, T, H, dtype=torch.bfloat16, device=dev)
        dQ = torch.zeros(p.local_batch, T, N, device=dev)
        dK = torch.zeros_like(q)
        dV = torch.zeros_like(q)
        A.flashAttentionForward(q, k, v, prm, p.local_batch, out=out, l=l, shard=sh)
        A.computeD(do, out, prm, p.local_batch, D=Dv, shard=sh)
        A.flashAttentionBackward(do, Dv, l, q, k, v, prm, p.local_batch, dQ=dQ, dK=dK, dV=dV, shard=sh)
        torch.cuda.synchronize(dev)
        assert A.device_status() == 0
        # place this rank's shards into global-shaped buffers (disjoint parts)
        g = {n: torch.zeros((B, T, N), dtype=torch.float64) for n in ("out", "dQ", "dK", "dV")}
        for bh in range(p.bh_begin, p.bh_end):
            b, h = divmod(bh, H)
            lb = b - p.b_begin
            cols = slice(h * D, (h + 1) * D)
            for n, t in (("out", out), ("dQ", dQ), ("dK", dK), ("dV", dV)):
                g[n][b, :, cols] = t[lb, :, cols].double().cpu()
        for n in g:
            dist.all_reduce(g[n])
        if rank == 0:
            np.savez(out_path, **{n: g[n].numpy() for n in g})
    finally:
        dist.destroy_process_group()


def test_two_gpus_shards_match_one_gpu(tmp_path):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    import torch.multiprocessing as mp

    from metalllm_b200 import attention as A
    from metalllm_b200.inputs import normal_bf16

    B, T, H, D = 3, 512, 3, 128   # 9 shards: rank 0 gets 5, rank 1 gets 4 (split inside a batch row)
    out_path = str(tmp_path / "two.npz")
    mp.start_processes(_worker, args=(2, _free_port(), B, T, H, D, out_path), nprocs=2,
                       start_method="spawn", join=True)
    got = np.load(out_path)
    N = H * D
    up = lambda a: torch.from_numpy(a.view(np.int16)).view(torch.bfloat16).cuda(0)
    q, k, v, do = (up(normal_bf16(B * T * N, 3, s).reshape(B, T, N)) for s in (1, 2, 3, 4))
    prm = A.make_params(T, H, D)
    out, l = A.flashAttentionForward(q, k, v, prm, B)
    Dv = A.computeD(do, out, prm, B)
    dQ, dK, dV = A.flashAttentionBackward(do, Dv, l, q, k, v, prm, B)
    torch.cuda.synchronize()
    for n, t in (("out", out), ("dK", dK), ("dV", dV)):
        assert np.array_equal(got[n], t.double().cpu().numpy()), n
    ref = dQ.double().cpu().numpy()
    assert np.abs(got["dQ"] - ref).max() <= 1e-5 * max(1.0, np.abs(ref).max())
