"""The Q8_0 decode stack on the GPU (config 5 shapes, 1 GPU), step by step
against the oracle: each projection's fp32 output must lie within 1e-5 of the
sum of |block terms| of the oracle's Q8_0 x Q8_0 matvec of the same input."""
import numpy as np
import pytest

import oracle

pytestmark = pytest.mark.gpu


def _check_step(W, x, M, K, y):
    xq = oracle.quantize_q8_0(x, 1, K)
    ref, dots = oracle.q8_0_gemv_q8(W, xq, M, K, with_dots=True)
    dw = W.reshape(M, K // 32, 34)[:, :, 0:2].copy().view(np.float16)[..., 0].astype(np.float64)
    dx = xq.reshape(K // 32, 34)[:, 0:2].copy().view(np.float16)[:, 0].astype(np.float64)
    bound = np.abs(dots.astype(np.float64) * dw * dx[None, :]).sum(axis=1)
    assert np.all(np.abs(y.astype(np.float64) - ref.astype(np.float64)) <= 1e-5 * bound + 1e-30)


@pytest.mark.parametrize("shapes", ["small", "config5"])
def test_decode_stack_steps(ane, shapes):
    import torch

    from ane_b200.decode import LAYER_SHAPES, gpu_stack

    sh = LAYER_SHAPES if shapes == "config5" else (("qkv", 512, 256), ("o", 256, 256), ("gate_up", 512, 256),
                                                   ("down", 256, 256))
    layers = 1 if shapes == "config5" else 2
    stack = gpu_stack(layers, torch.device("cuda", 0), shapes=sh, seed=9)
    trace = []
    out = stack.forward(trace)
    torch.cuda.synchronize()
    assert torch.isfinite(out).all()
    for (l, p, x, y) in trace:
        _, M, K = sh[p]
        _check_step(stack.weights[l][p].cpu().numpy(), x.cpu().numpy(), M, K, y.cpu().numpy())


@pytest.mark.parametrize("shapes,batch", [("small", 16), ("config5", 16), ("small", 5)])
def test_decode_stack_batch_steps_exact(ane, shapes, batch):
    """Config 5 at batch > 1: every projection of the stack equals the
    oracle's batched Q8_0 product of that step's input rows, bit for bit."""
    import torch

    from ane_b200.decode import LAYER_SHAPES, gpu_stack

    sh = LAYER_SHAPES if shapes == "config5" else (("qkv", 512, 256), ("o", 256, 256), ("gate_up", 512, 256),
                                                   ("down", 256, 256))
    stack = gpu_stack(1 if shapes == "config5" else 2, torch.device("cuda", 0), shapes=sh, seed=9, batch=batch)
    trace = []
    out = stack.forward(trace)
    torch.cuda.synchronize()
    assert out.shape == (batch, sh[-1][1]) and torch.isfinite(out).all()
    for (l, p, x, y) in trace:
        _, M, K = sh[p]
        xq = oracle.quantize_q8_0(x.contiguous().cpu().numpy(), batch, K)
        ref = oracle.mul_mat_q8_0_batch(stack.weights[l][p].cpu().numpy(), xq, M, K, batch)
        assert np.array_equal(ref.view(np.uint32), y.contiguous().cpu().numpy().view(np.uint32)), (l, p)


def test_decode_stack_graph_replay_matches_eager(ane):
    import torch

    from ane_b200.decode import gpu_stack

    sh = (("qkv", 512, 256), ("o", 256, 256), ("gate_up", 512, 256), ("down", 256, 256))
    stack = gpu_stack(3, torch.device("cuda", 0), shapes=sh, seed=4)
    eager = stack.forward().clone()
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        res = stack.forward()
    res.fill_(float("nan"))
    g.replay()
    torch.cuda.synchronize()
    assert torch.equal(res, eager)
    del g


@pytest.mark.parametrize("shapes,layers", [("small", 3), ("config5", 2)])
def test_peer_chain_mode_r_equals_q8_0_gemv_chain(ane, shapes, layers):
    """Mode R (the reference's q8_0_gemv on the fp32 activation) as a chain whose
    rows go into the next projection's tagged vector (ane_q8_0_gemv_gather_dev)
    == the plain chain of q8_0_gemv launches, bit for bit, on repeated tokens and
    under graph replay."""
    import torch

    from ane_b200.decode import LAYER_SHAPES, PeerChainDecodeStack, gpu_stack

    sh = LAYER_SHAPES if shapes == "config5" else (("qkv", 512, 256), ("o", 256, 256), ("gate_up", 512, 256),
                                                   ("down", 256, 256))
    dev = torch.device("cuda", 0)
    stack = gpu_stack(layers, dev, shapes=sh, seed=31, mode="r")
    ref = stack.forward().clone()
    peer = PeerChainDecodeStack(stack, dev, mode="r")
    try:
        for _ in range(3):
            out = peer.forward()
            torch.cuda.synchronize()
            assert torch.equal(out.view(torch.int32), ref.view(torch.int32))
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            peer.forward()
        for _ in range(2):
            peer.out.fill_(float("nan"))
            g.replay()
            torch.cuda.synchronize()
            assert torch.equal(peer.out.view(torch.int32), ref.view(torch.int32))
        del g
        assert ane.lib.ane_device_timeouts() == 0
    finally:
        peer.close()


@pytest.mark.parametrize("shapes,layers,batch", [("small", 3, 16), ("small", 2, 5), ("config5", 1, 16)])
def test_peer_batch_equals_batched_stack(ane, shapes, layers, batch):
    """Decode at batch > 1 as a chain of batched MUL_MATs whose outputs go
    into the next projection's tagged vector (ane_mul_mat_q8_0_batch_gather_dev,
    a step-end launch) == the plain batched stack, bit for bit, on repeated
    steps (tags only grow) and under graph replay."""
    import torch

    from ane_b200.decode import LAYER_SHAPES, PeerBatchDecodeStack, gpu_stack

    sh = LAYER_SHAPES if shapes == "config5" else (("qkv", 512, 256), ("o", 256, 256), ("gate_up", 512, 256),
                                                   ("down", 256, 256))
    dev = torch.device("cuda", 0)
    stack = gpu_stack(layers, dev, shapes=sh, seed=29, batch=batch)
    ref = stack.forward().clone()
    peer = PeerBatchDecodeStack(stack, dev)
    try:
        for _ in range(3):
            out = peer.forward()
            torch.cuda.synchronize()
            assert out.shape == ref.shape
            assert torch.equal(out.view(torch.int32), ref.view(torch.int32))
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            peer.forward()
        for _ in range(2):
            peer.out.fill_(float("nan"))
            g.replay()
            torch.cuda.synchronize()
            assert torch.equal(peer.out.view(torch.int32), ref.view(torch.int32))
        del g
        assert ane.lib.ane_device_timeouts() == 0
    finally:
        peer.close()


@pytest.mark.parametrize("shapes,layers", [("small", 3), ("config5", 2)])
def test_peer_chain_equals_per_projection_chain(ane, shapes, layers):
    """The fused-gather chain (one MUL_MAT launch per projection writing every
    rank's next input, arrival counters, a token-end launch) == the plain chain
    of MUL_MAT launches, bit for bit, on repeated tokens (counters and token
    count only grow) and under graph replay."""
    import torch

    from ane_b200.decode import LAYER_SHAPES, PeerChainDecodeStack, gpu_stack

    sh = LAYER_SHAPES if shapes == "config5" else (("qkv", 512, 256), ("o", 256, 256), ("gate_up", 512, 256),
                                                   ("down", 256, 256))
    stack = gpu_stack(layers, torch.device("cuda", 0), shapes=sh, seed=23)
    ref = stack.forward().clone()
    peer = PeerChainDecodeStack(stack, torch.device("cuda", 0))
    try:
        for _ in range(3):
            out = peer.forward()
            torch.cuda.synchronize()
            assert torch.equal(out.view(torch.int32), ref.view(torch.int32))
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            peer.forward()
        for _ in range(2):
            peer.out.fill_(float("nan"))
            g.replay()
            torch.cuda.synchronize()
            assert torch.equal(peer.out.view(torch.int32), ref.view(torch.int32))
        del g
        assert ane.lib.ane_device_timeouts() == 0
    finally:
        peer.close()


@pytest.mark.parametrize("shapes,layers", [("small", 3), ("config5", 2)])
def test_fused_stack_equals_per_projection_chain(ane, shapes, layers):
    """One persistent launch per token == the chain of MUL_MAT launches, bit for
    bit, on repeated tokens (the counters only grow) and under graph replay."""
    import torch

    from ane_b200.decode import LAYER_SHAPES, FusedDecodeStack, gpu_stack

    sh = LAYER_SHAPES if shapes == "config5" else (("qkv", 512, 256), ("o", 256, 256), ("gate_up", 512, 256),
                                                   ("down", 256, 256))
    stack = gpu_stack(layers, torch.device("cuda", 0), shapes=sh, seed=21)
    ref = stack.forward().clone()
    fused = FusedDecodeStack(stack, torch.device("cuda", 0))
    try:
        for _ in range(3):
            out = fused.forward()
            torch.cuda.synchronize()
            assert torch.equal(out.view(torch.int32), ref.view(torch.int32))
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            fused.forward()
        for _ in range(2):
            fused.out.fill_(float("nan"))
            g.replay()
            torch.cuda.synchronize()
            assert torch.equal(fused.out.view(torch.int32), ref.view(torch.int32))
        del g
        assert ane.lib.ane_device_timeouts() == 0
    finally:
        fused.close()


@pytest.mark.parametrize("shapes,layers", [("small", 2), ("config5", 1)])
def test_decode_stack_mode_r_steps_exact(ane, shapes, layers):
    """Config 5 with the reference's arithmetic (mode R): each projection is
    q8_0_gemv on the fp32 activation -- what the reference's ggml MUL_MAT Q8_0
    branch dispatches (src/ggml-backend/ggml-ane.cpp:160-166) -- and equals
    the oracle's q8_0_gemv of that step's input bit for bit (the handler's
    16-lane FMA order and FADDV tree, src/bytecode_interpreter.s:7010-7063)."""
    import torch

    from ane_b200.decode import LAYER_SHAPES, gpu_stack

    sh = LAYER_SHAPES if shapes == "config5" else (("qkv", 512, 256), ("o", 256, 256), ("gate_up", 512, 256),
                                                   ("down", 256, 256))
    stack = gpu_stack(layers, torch.device("cuda", 0), shapes=sh, seed=13, mode="r")
    trace = []
    out = stack.forward(trace)
    torch.cuda.synchronize()
    assert torch.isfinite(out).all()
    assert len(trace) == layers * len(sh)
    for (l, p, x, y) in trace:
        _, M, K = sh[p]
        ref = oracle.q8_0_gemv(stack.weights[l][p].cpu().numpy(), x.contiguous().cpu().numpy(), M, K)
        assert np.array_equal(ref.view(np.uint32), y.contiguous().cpu().numpy().view(np.uint32)), (l, p)
