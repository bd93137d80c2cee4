"""Host logic of the row-sharded Q8_0 decode stack with gloo ranks (CPU).

DecodeStack (ane_b200/decode.py) runs quantize -> matvec -> all-gather per
projection.  Bound to the CPU oracle, a world-2 run must give bit-identical
vectors to a world-1 run (every output row is computed the same way on any
rank), and every step must equal the oracle applied to that step's input.
"""
import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

SHAPES = (("qkv", 512, 256), ("o", 256, 256), ("gate_up", 512, 256), ("down", 256, 256))


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _oracle_stack(layers, world, rank, gather, batch=1):
    import oracle
    from ane_b200.decode import ROW_BLOCK, DecodeStack, block_seed

    def make_rows(layer, p, blk, K):
        rng = np.random.default_rng(block_seed(3, layer, p, blk))
        w = (rng.standard_normal(ROW_BLOCK * K) * 0.02).astype(np.float32)
        return torch.from_numpy(oracle.quantize_q8_0(w, ROW_BLOCK, K))

    def quantize(x):
        if batch > 1:  # [batch, K] rows -> batch rows of Q8_0 blocks
            return torch.from_numpy(oracle.quantize_q8_0(x.contiguous().numpy(), x.shape[0], x.shape[1]))
        return torch.from_numpy(oracle.quantize_q8_0(x.numpy(), 1, x.numel()))

    def matvec(W, xq, rows, K, out):
        if batch > 1:
            out.copy_(torch.from_numpy(oracle.mul_mat_q8_0_batch(W.numpy(), xq.numpy(), rows, K, batch)))
        else:
            out.copy_(torch.from_numpy(oracle.q8_0_gemv_q8(W.numpy(), xq.numpy(), rows, K)))
        return out

    def make_inputs(n, K):
        return torch.from_numpy(np.random.default_rng(11).standard_normal((n, K)).astype(np.float32))

    return DecodeStack(layers, world, rank, make_rows, quantize, matvec, gather, SHAPES, None, make_inputs, batch)


def _worker(rank, world, port, layers, result_q, batch=1):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    import datetime

    import torch.distributed as dist

    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        def gather(y_loc, y_full):
            if batch == 1:
                dist.all_gather(list(y_full.view(world, -1).unbind(0)), y_loc)
                return
            parts = [torch.empty_like(y_loc) for _ in range(world)]
            dist.all_gather(parts, y_loc)
            m = y_loc.shape[1]
            for r, part in enumerate(parts):
                y_full[:, r * m:(r + 1) * m] = part

        trace = []
        out = _oracle_stack(layers, world, rank, gather, batch).forward(trace)
        if rank == 0:
            result_q.put((out.numpy().copy(), [(l, p, x.numpy(), y.numpy()) for l, p, x, y in trace]))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("batch", [1, 3])
def test_decode_stack_sharded_equals_single(batch):
    import oracle

    layers, world = 2, 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, layers, q, batch)) for r in range(world)]
    for p in procs:
        p.start()
    out2, trace2 = q.get(timeout=120)
    for p in procs:
        p.join(timeout=120)
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]

    trace1 = []
    out1 = _oracle_stack(layers, 1, 0, None, batch).forward(trace1).numpy()
    assert np.array_equal(out1.view(np.uint32), out2.view(np.uint32))
    assert len(trace1) == len(trace2) == layers * len(SHAPES)
    for (l, p, x, y), (_, _, x2, y2) in zip(trace1, trace2):
        assert np.array_equal(x.numpy().view(np.uint32), x2.view(np.uint32))
        assert np.array_equal(y.numpy().view(np.uint32), y2.view(np.uint32))
    # each step is the oracle's product of that step's quantized input
    stack = _oracle_stack(layers, 1, 0, None, batch)
    for (l, p, x, y) in trace1:
        _, M, K = SHAPES[p]
        W = stack.weights[l][p].numpy()
        if batch == 1:
            ref = oracle.q8_0_gemv_q8(W, oracle.quantize_q8_0(x.numpy(), 1, K), M, K)
        else:
            xq = oracle.quantize_q8_0(x.contiguous().numpy(), batch, K)
            ref = oracle.mul_mat_q8_0_batch(W, xq, M, K, batch)
        assert np.array_equal(ref.view(np.uint32), y.numpy().view(np.uint32))


def test_shard_rows_rules():
    from ane_b200.decode import LAYER_SHAPES, shard_rows, stack_weight_bytes

    for _, M, _ in LAYER_SHAPES:
        for world in (1, 2, 4, 8):
            spans = [shard_rows(M, world, r) for r in range(world)]
            assert spans[0][0] == 0 and spans[-1][1] == M
            assert all(a[1] == b[0] for a, b in zip(spans, spans[1:]))
    with pytest.raises(ValueError):
        shard_rows(100, 2, 0)
    assert stack_weight_bytes(32) == 32 * 202_375_168 // 32 * 34  # 6.88 GB of Q8_0 weights
