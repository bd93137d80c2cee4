"""Q8_0 MUL_MAT over NT <= 16 activation rows (config 5 at batch 16), through
the C ABI (ane_mul_mat_q8_0_batch_dev), against the oracle bit for bit: the
activation quantization, every int32 block dot and the fp32 segment order are
fixed, so the fp32 outputs are exact, not within a tolerance."""
import numpy as np
import pytest

import oracle

pytestmark = pytest.mark.gpu


def _same_bits(a, b):
    a = np.ascontiguousarray(a, np.float32)
    b = np.ascontiguousarray(b, np.float32)
    nan = np.isnan(a)
    assert np.array_equal(nan, np.isnan(b))
    assert np.array_equal(a[~nan].view(np.uint32), b[~nan].view(np.uint32)), \
        f"{int(((a != b) & ~nan).sum())} of {a.size} differ; max |diff| {np.nanmax(np.abs(a - b))}"


def _case(M, K, NT, seed):
    rng = np.random.default_rng(seed)
    w = (rng.standard_normal((M, K)) * 0.02).astype(np.float32)
    x = rng.standard_normal((NT, K)).astype(np.float32)
    return oracle.quantize_q8_0(w, M, K), x


@pytest.mark.parametrize("M,K,NT", [
    (4096, 4096, 16),    # O projection (config 5), batch 16
    (4096, 11008, 16),   # down projection: 11 segments, the last one 24 blocks
    (12288, 4096, 8),    # QKV, one token octet
    (100, 4096, 5),      # ragged rows and tokens
    (16, 256, 1),        # one unit
    (300, 11008, 9),
    (64, 512, 16),
    (2000, 1024, 12),
    (37, 512, 3),        # M % 4 != 0: the last tile's missing rows are never copied
    (1001, 4352, 16),    # K = 17 x 256: a last segment of 8 blocks
])
def test_mul_mat_q8_0_batch_exact(ane, M, K, NT):
    import torch

    W, x = _case(M, K, NT, M * 31 + K + NT)
    ref = oracle.mul_mat_q8_0_batch(W, oracle.quantize_q8_0(x, NT, K), M, K, NT)
    y = ane.mul_mat_q8_0_batch(torch.from_numpy(W).cuda(), torch.from_numpy(x).cuda(), M, K)
    _same_bits(y.cpu().numpy(), ref)


def test_mul_mat_q8_0_batch_strided_repeat_graph(ane):
    """Strided activation / output rows (a view into wider buffers), a reused
    workspace, static weights, graph replay."""
    import torch

    M, K, NT = 1024, 2048, 16
    W, x = _case(M, K, NT, 7)
    ref = oracle.mul_mat_q8_0_batch(W, oracle.quantize_q8_0(x, NT, K), M, K, NT)
    Wd = torch.from_numpy(W).cuda()
    xbuf = torch.zeros((NT, K + 512), device="cuda")
    xbuf[:, :K] = torch.from_numpy(x).cuda()
    ybuf = torch.full((NT, M + 64), -1.0, device="cuda")
    ws = ane.mul_mat_q8_0_batch_workspace(M, K, "cuda")
    for _ in range(3):
        ybuf[:, :M].zero_()
        ane.mul_mat_q8_0_batch(Wd, xbuf[:, :K], M, K, out=ybuf[:, :M], workspace=ws, static_weights=True)
        _same_bits(ybuf[:, :M].cpu().numpy(), ref)
    assert torch.all(ybuf[:, M:] == -1.0)
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        ane.mul_mat_q8_0_batch(Wd, xbuf[:, :K], M, K, out=ybuf[:, :M], workspace=ws, static_weights=True)
    torch.cuda.current_stream().wait_stream(s)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        for _ in range(4):
            ane.mul_mat_q8_0_batch(Wd, xbuf[:, :K], M, K, out=ybuf[:, :M], workspace=ws, static_weights=True)
    ybuf[:, :M].zero_()
    g.replay()
    torch.cuda.synchronize()
    _same_bits(ybuf[:, :M].cpu().numpy(), ref)


def test_mul_mat_q8_0_batch_special_scales(ane):
    """Zero, subnormal, inf and NaN block scales in W; an all-zero activation
    block (d = 0, codes 0)."""
    import torch

    M, K, NT = 256, 1024, 16
    W, x = _case(M, K, NT, 11)
    Wb = W.reshape(M, K // 32, 34)
    Wb[3, :, 0:2] = 0                                  # d = +0: every term +0
    Wb[5, 2, 0:2] = np.frombuffer(np.float16(6e-8).tobytes(), np.uint8)   # subnormal fp16
    Wb[7, 4, 0:2] = np.frombuffer(np.float16(np.inf).tobytes(), np.uint8)
    Wb[9, 1, 0:2] = np.frombuffer(np.float16(np.nan).tobytes(), np.uint8)
    Wb[11, :, 2:] = 0                                  # all codes 0: sumi = 0
    x[2, 64:96] = 0.0
    ref = oracle.mul_mat_q8_0_batch(W, oracle.quantize_q8_0(x, NT, K), M, K, NT)
    y = ane.mul_mat_q8_0_batch(torch.from_numpy(W).cuda(), torch.from_numpy(x).cuda(), M, K)
    _same_bits(y.cpu().numpy(), ref)


def test_mul_mat_q8_0_batch_row_shards(ane):
    """A row shard of W gives exactly the matching rows of the full product
    (the fp32 order depends on K only), as the N-sharded decode stack needs."""
    import torch

    M, K, NT = 2048, 4096, 16
    W, x = _case(M, K, NT, 13)
    Wd, xd = torch.from_numpy(W).cuda(), torch.from_numpy(x).cuda()
    full = ane.mul_mat_q8_0_batch(Wd, xd, M, K)
    rb = K // 32 * 34
    for r0, r1 in [(0, 512), (512, 1536), (1536, 2048)]:
        part = ane.mul_mat_q8_0_batch(Wd[r0 * rb:r1 * rb], xd, r1 - r0, K)
        assert torch.equal(part.view(torch.int32), full[:, r0:r1].contiguous().view(torch.int32))
