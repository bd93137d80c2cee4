"""N-sharded dense_fused_i8 on 2 GPUs (NCCL) vs one GPU, bit for bit.

Runs as two spawned ranks (one per GPU).  Skipped when fewer than two GPUs are
visible.  NVLS is switched off (NCCL_NVLS_ENABLE=0): the kernels use no
multicast and the test needs none.
"""
import os
import socket

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, M, N, K, scale, relu, shard, result_q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    import datetime

    import torch
    import torch.distributed as dist

    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=dev)
    try:
        import ane_b200 as ane
        from ane_b200.sharded import ShardedDense

        g = torch.Generator(device=dev).manual_seed(11)
        A = torch.randn((M, K), device=dev, generator=g)
        B = torch.randn((K, N), device=dev, generator=g)  # same full B on every rank
        if shard == "cols":
            n_local = N // world
            part = ShardedDense(M, n_local, K, world, dev, shard="cols")
            C = part.forward(A, B[:, rank * n_local:(rank + 1) * n_local].contiguous(), scale, relu)
        else:
            m_local = M // world
            part = ShardedDense(m_local, N, K, world, dev, shard="rows")
            C = part.forward(A[rank * m_local:(rank + 1) * m_local].contiguous(), B, scale, relu)
        ref = ane.dense_fused_i8(A, B, scale, relu)  # single-GPU result on the same inputs
        torch.cuda.synchronize()
        same = torch.equal(C.view(torch.int32), ref.view(torch.int32))
        flags = torch.tensor([1 if same else 0], device=dev)
        dist.all_reduce(flags, op=dist.ReduceOp.MIN)
        if rank == 0:
            result_q.put(int(flags.item()))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("M,N,K,scale,relu,shard", [(512, 1024, 512, 1.0, False, "cols"),
                                                    (64, 14336, 4096, 0.125, True, "cols"),
                                                    (1024, 768, 4096, 1.0, True, "rows")])
def test_sharded_dense_fused_two_gpus_bit_exact(M, N, K, scale, relu, shard):
    import torch

    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, M, N, K, scale, relu, shard, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    assert q.get(timeout=5) == 1
