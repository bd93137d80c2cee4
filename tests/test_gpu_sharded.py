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


def _worker(rank, world, port, M, N, K, scale, relu, shard, fused, result_q):
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
        ref = ane.dense_fused_i8(A, B, scale, relu)  # single-GPU result on the same inputs
        if shard == "cols":
            n_local = N // world
            part = ShardedDense(M, n_local, K, world, dev, shard="cols", fused_gather=fused)
            args = (A, B[:, rank * n_local:(rank + 1) * n_local].contiguous())
        else:
            m_local = M // world
            part = ShardedDense(m_local, N, K, world, dev, shard="rows", fused_gather=fused)
            args = (A[rank * m_local:(rank + 1) * m_local].contiguous(), B)
        same = True
        for _ in range(3):  # repeated calls: the fused gather's counters only grow
            C = part.forward(*args, scale, relu).clone()
            torch.cuda.synchronize()
            same = same and torch.equal(C.view(torch.int32), ref.view(torch.int32))
        same = same and ane.lib.ane_device_timeouts() == 0
        torch.cuda.synchronize()
        dist.barrier()  # no rank unmaps a peer buffer while a peer still writes it
        part.close()
        flags = torch.tensor([1 if same else 0], device=dev)
        dist.all_reduce(flags, op=dist.ReduceOp.MIN)
        if rank == 0:
            result_q.put(int(flags.item()))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("fused", [False, True])
@pytest.mark.parametrize("M,N,K,scale,relu,shard", [(512, 1024, 512, 1.0, False, "cols"),
                                                    (64, 14336, 4096, 0.125, True, "cols"),
                                                    (1024, 768, 4096, 1.0, True, "rows"),
                                                    (4096, 4096, 4096, 1.0, False, "rows")])
def test_sharded_dense_fused_two_gpus_bit_exact(M, N, K, scale, relu, shard, fused):
    """NCCL all-gather (fused=False) or the gather fused into the GEMM epilogue
    (peer stores, fused=True): either way the gathered C equals one GPU's."""
    import torch

    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, M, N, K, scale, relu, shard, fused, q))
             for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    assert q.get(timeout=5) == 1


def _stack_worker(rank, world, port, layers, result_q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    import datetime

    import torch
    import torch.distributed as dist

    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=dev)
    fused = peer = peer16 = peer_r = None
    try:
        import ane_b200 as ane
        from ane_b200.decode import FusedDecodeStack, PeerBatchDecodeStack, PeerChainDecodeStack, gpu_stack

        sharded = gpu_stack(layers, dev, world=world, rank=rank, seed=33)
        nccl_out = sharded.forward().clone()            # NCCL all-gather per projection
        fused = FusedDecodeStack(sharded, dev)           # peer stores + counters, one launch
        outs = [fused.forward().clone() for _ in range(3)]
        peer = PeerChainDecodeStack(sharded, dev)        # peer stores + counters, a launch per projection
        outs += [peer.forward().clone() for _ in range(3)]
        single = gpu_stack(layers, dev, world=1, rank=0, seed=33).forward()  # one GPU, all rows
        torch.cuda.synchronize()
        ok = torch.equal(nccl_out.view(torch.int32), single.view(torch.int32)) and all(
            torch.equal(o.view(torch.int32), single.view(torch.int32)) for o in outs)
        # mode R (the reference's q8_0_gemv arithmetic) as the peer-store chain
        sharded_r = gpu_stack(layers, dev, world=world, rank=rank, seed=33, mode="r", weights=sharded.weights)
        peer_r = PeerChainDecodeStack(sharded_r, dev, mode="r")
        outs_r = [peer_r.forward().clone() for _ in range(3)]
        single_r = gpu_stack(layers, dev, world=1, rank=0, seed=33, mode="r").forward()
        torch.cuda.synchronize()
        ok = ok and all(torch.equal(o.view(torch.int32), single_r.view(torch.int32)) for o in outs_r)
        # batch 16: the batched chain with peer stores == the 1-GPU batched stack
        sharded16 = gpu_stack(layers, dev, world=world, rank=rank, seed=33, batch=16)
        peer16 = PeerBatchDecodeStack(sharded16, dev)
        outs16 = [peer16.forward().clone() for _ in range(3)]
        single16 = gpu_stack(layers, dev, world=1, rank=0, seed=33, batch=16).forward()
        torch.cuda.synchronize()
        ok = ok and all(torch.equal(o.view(torch.int32), single16.view(torch.int32)) for o in outs16)
        ok = ok and ane.lib.ane_device_timeouts() == 0
        flags = torch.tensor([1 if ok else 0], device=dev)
        dist.all_reduce(flags, op=dist.ReduceOp.MIN)
        if rank == 0:
            result_q.put(int(flags.item()))
    finally:
        if fused is not None or peer is not None or peer16 is not None or peer_r is not None:
            torch.cuda.synchronize()
            dist.barrier()  # no rank unmaps a peer buffer while a peer still writes it
            for s in (fused, peer, peer16, peer_r):
                if s is not None:
                    s.close()
        dist.destroy_process_group()


def test_decode_stack_two_gpus_fused_and_nccl_equal_one_gpu():
    """Config-5 decode stack (2 layers) row-sharded over 2 GPUs: the NCCL
    all-gather version, the one-launch peer-store version and the
    launch-per-projection peer-store chain all give the 1-GPU vector bit for
    bit, on repeated tokens; so does the batch-16 chain of batched MUL_MATs
    with peer stores."""
    import torch

    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_stack_worker, args=(r, 2, port, 2, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    assert q.get(timeout=5) == 1
