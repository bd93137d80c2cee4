"""Host logic of the N-sharded dense_fused_i8 with world_size-2 gloo ranks (CPU).

ShardPlan (ane_b200/sharded.py) carries the collective steps: all-reduce MAX
of the two absmax values (NaN-preserving) and the all-gather + interleave of
the column shards.  Here the compute callables are the CPU oracle, so the test
runs without a GPU; the sharded result must be bit-identical to the
single-process oracle on the full matrices.
"""
import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, case, result_q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    import datetime

    import torch.distributed as dist

    import oracle
    from ane_b200.sharded import ShardPlan

    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        M, N, K, scale, relu, nan_rank, shard = case
        rng = np.random.default_rng(7)
        A = rng.standard_normal((M, K)).astype(np.float32)
        B = rng.standard_normal((K, N)).astype(np.float32)
        if nan_rank is not None:  # a NaN inside one rank's part only
            if shard == "cols":
                B[3, nan_rank * (N // world) + 1] = np.nan
            else:
                A[nan_rank * (M // world) + 1, 3] = np.nan
        if shard == "cols":
            n_local = N // world
            A_part, B_part = A, np.ascontiguousarray(B[:, rank * n_local:(rank + 1) * n_local])
        else:
            m_local = M // world
            A_part, B_part = np.ascontiguousarray(A[rank * m_local:(rank + 1) * m_local]), B

        def absmax2(A_, B_):
            return torch.tensor([oracle.absmax(A_.numpy()), oracle.absmax(B_.numpy())], dtype=torch.float32)

        def quantize_gemm(A_, B_, am):
            qa, sa = oracle.quantize_with_absmax(A_.numpy(), am[0].item())
            qb, sb = oracle.quantize_with_absmax(B_.numpy(), am[1].item())
            acc = oracle.gemm_s8_s32(qa.reshape(A_.shape[0], K), qb.reshape(K, B_.shape[1]))
            return torch.from_numpy(oracle.dense_fused_epilogue(acc, sa, sb, scale, relu))

        C = ShardPlan(world, shard=shard).run(torch.from_numpy(A_part), torch.from_numpy(B_part), absmax2,
                                              quantize_gemm)
        if rank == 0:
            ref = oracle.dense_fused_i8(A, B, scale, relu)
            c = C.numpy()
            same = np.array_equal(np.isnan(c), np.isnan(ref)) and np.array_equal(
                c[~np.isnan(c)].view(np.uint32), ref[~np.isnan(ref)].view(np.uint32))
            result_q.put(("ok" if same else "mismatch", int(np.isnan(c).sum())))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("case", [(33, 64, 96, 1.0, False, None, "cols"), (50, 128, 784, 0.5, True, None, "cols"),
                                  (16, 32, 64, 1.0, False, 1, "cols"), (34, 64, 96, 1.0, False, None, "rows"),
                                  (50, 128, 784, 0.5, True, None, "rows"), (16, 32, 64, 1.0, False, 0, "rows")])
def test_sharded_plan_matches_single_process(case):
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, case, q)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    status, n_nan = q.get(timeout=5)
    assert status == "ok"
    if case[-2] is not None:  # a NaN in one rank's part poisons every rank's scale
        assert n_nan == case[0] * case[1]


def test_interleave_shards_layout():
    from ane_b200.sharded import interleave_shards

    g = torch.arange(2 * 3 * 4).reshape(2, 3, 4)
    out = interleave_shards(g)
    assert out.shape == (3, 8)
    assert torch.equal(out[:, :4], g[0]) and torch.equal(out[:, 4:], g[1])
