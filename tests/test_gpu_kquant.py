"""K-quant matvecs (q4_k / q2_k / q3_k / q5_k / q6_k _gemv, 0x75-0x79) and
get_rows_q4_0 (0x7D) on the GPU, through the C ABI (device entry points, the
synchronous host entry points and stream_exec), against the oracle bit for
bit: every element value, the 16 lane FMA chains and the FADDV tree are the
handlers' own, so the results are exact, not within a tolerance."""
import ctypes

import numpy as np
import pytest

import oracle
from kquant_util import BLOCK_BYTES, get_rows_q4_0_kat_tables, random_blocks, set_scale

pytestmark = pytest.mark.gpu

FMTS = sorted(BLOCK_BYTES)
OPS = {"q4_k": 0x75, "q2_k": 0x76, "q3_k": 0x77, "q5_k": 0x78, "q6_k": 0x79}


def _same_bits(a, b):
    a = np.ascontiguousarray(a, np.float32)
    b = np.ascontiguousarray(b, np.float32)
    nan = np.isnan(a)
    assert np.array_equal(nan, np.isnan(b))
    assert np.array_equal(a[~nan].view(np.uint32), b[~nan].view(np.uint32)), \
        f"{int(((a != b) & ~nan).sum())} of {a.size} differ; max |diff| {np.nanmax(np.abs(a - b))}"


def _x(K, rng):
    x = rng.standard_normal(K).astype(np.float32)
    x[::97] = 0.0                                    # q3_k: stale shift 0 keeps the codes
    x[5::211] = np.uint32(3).view(np.float32)        # tiny denormals: shifts of 3
    x[7::223] = -0.0                                 # -0.0: bits >= 32, code bits 0
    return x


@pytest.mark.parametrize("fmt", FMTS)
@pytest.mark.parametrize("M,K", [(1, 256), (37, 512), (4096, 4096), (1000, 11008), (64, 300), (8192, 512)])
def test_kquant_gemv_exact(ane, fmt, M, K):
    """8192 rows of K = 512: more four-row groups per CTA than two ring slots
    hold, so the plan spreads them over more CTAs."""
    import torch

    rng = np.random.default_rng(M * 7 + K + len(fmt))
    W = random_blocks(fmt, M, K, rng)
    x = _x(K, rng)
    ref = oracle.kquant_gemv(fmt, W, x, M, K)
    y = ane.kquant_gemv(fmt, torch.from_numpy(W).cuda(), torch.from_numpy(x).cuda(), M, K)
    _same_bits(y.cpu().numpy(), ref)


@pytest.mark.parametrize("fmt", ["q3_k", "q6_k"])
@pytest.mark.parametrize("offset", [2, 6])
def test_kquant_gemv_unaligned_base(ane, fmt, offset):
    """Rows of 110- / 210-byte super-blocks at a W base that is only 2-byte
    aligned: the bulk-copy path copies 16-byte-aligned spans and reads each row
    from its offset inside its span, bit-exact with the oracle."""
    import torch

    M, K = 100, 11008
    rng = np.random.default_rng(offset * 31 + len(fmt))
    W = random_blocks(fmt, M, K, rng)
    x = _x(K, rng)
    ref = oracle.kquant_gemv(fmt, W, x, M, K)
    buf = torch.zeros(W.size + 64, dtype=torch.uint8, device="cuda")
    buf[offset:offset + W.size] = torch.from_numpy(W).cuda()
    y = ane.kquant_gemv(fmt, buf[offset:offset + W.size], torch.from_numpy(x).cuda(), M, K)
    _same_bits(y.cpu().numpy(), ref)


@pytest.mark.parametrize("fmt", FMTS)
def test_kquant_gemv_special_scales(ane, fmt):
    """Zero, subnormal, inf and NaN super-block scales (d and, where the format
    has one, dmin)."""
    import torch

    M, K = 64, 1024
    rng = np.random.default_rng(3)
    W = random_blocks(fmt, M, K, rng)
    set_scale(W, fmt, M, K, 1, 0, 0.0)
    set_scale(W, fmt, M, K, 2, 1, 6e-8)
    set_scale(W, fmt, M, K, 3, 2, np.inf)
    set_scale(W, fmt, M, K, 4, 3, np.nan)
    set_scale(W, fmt, M, K, 5, 0, -np.inf)
    if fmt in ("q2_k", "q4_k", "q5_k"):
        set_scale(W, fmt, M, K, 6, 1, np.inf, which=1)
        set_scale(W, fmt, M, K, 7, 2, 0.0, which=1)
    x = _x(K, rng)
    ref = oracle.kquant_gemv(fmt, W, x, M, K)
    y = ane.kquant_gemv(fmt, torch.from_numpy(W).cuda(), torch.from_numpy(x).cuda(), M, K)
    _same_bits(y.cpu().numpy(), ref)


@pytest.mark.parametrize("fmt", FMTS)
@pytest.mark.parametrize("shapes", [((4096, 4096),) * 3, ((11008, 4096), (4096, 11008))], ids=["square", "ffn"])
def test_kquant_gemv_static_weights_chain(ane, fmt, shapes):
    """With the static-weights flag the next matvec streams its weights while
    the previous one still runs, and reads its activation only after that one
    has finished: a chain of matvecs, each output the next input, equals the
    plain calls bit for bit (and its first step the oracle).  The 7B FFN pair
    (11008 x 4096, then 4096 x 11008) also runs the bulk-copy producer, whose
    rows of 43 super-blocks of 84 / 110 / 210 bytes are not 16-byte multiples."""
    import torch

    rng = np.random.default_rng(17 + len(fmt) + len(shapes))
    Ws = [random_blocks(fmt, M, K, rng) for M, K in shapes]
    x = _x(shapes[0][1], rng)
    dWs = [torch.from_numpy(W).cuda() for W in Ws]
    dx = torch.from_numpy(x).cuda()

    def chain(static):
        v, outs = dx, []
        for W, (M, K) in zip(dWs, shapes):
            v = ane.kquant_gemv(fmt, W, v, M, K, static_weights=static)
            outs.append(v)
        return [o.cpu().numpy() for o in outs]

    plain, static = chain(False), chain(True)
    for a, b in zip(plain, static):
        _same_bits(b, a)
    M0, K0 = shapes[0]
    _same_bits(static[0], oracle.kquant_gemv(fmt, Ws[0], x, M0, K0))
    with pytest.raises(ane.AneError):
        ane.check(ane.lib.ane_kquant_gemv_ex_dev(0x74, M0, K0, dx.data_ptr(), dWs[0].data_ptr(),
                                                 dx.data_ptr(), 1, None))


@pytest.mark.parametrize("fmt", FMTS)
def test_kquant_gemv_host_and_stream_exec(ane, fmt):
    """Host buffers through ane_<fmt>_gemv and through a stream_exec byte stream."""
    from ane_b200 import Op, Ptr, U32, dispatch

    M, K = 300, 2048
    rng = np.random.default_rng(11)
    W = random_blocks(fmt, M, K, rng)
    x = _x(K, rng)
    ref = oracle.kquant_gemv(fmt, W, x, M, K)
    out = np.full(M, -1.0, np.float32)
    fn = getattr(ane.lib, "ane_%s_gemv" % fmt)
    ane.check(fn(M, K, x.ctypes.data, W.ctypes.data, out.ctypes.data))
    _same_bits(out, ref)
    out2 = np.full(M, -1.0, np.float32)
    dispatch(Op(OPS[fmt]), U32(M), U32(K), Ptr(x.ctypes.data), Ptr(W.ctypes.data), Ptr(out2.ctypes.data))
    _same_bits(out2, ref)


def test_kquant_gemv_k_below_one_superblock(ane):
    """floor(K / 256) = 0 super-blocks: every row is the FADDV of zero lanes, +0."""
    M, K = 8, 128
    out = np.full(M, 7.0, np.float32)
    W = np.zeros(16, np.uint8)
    x = np.ones(K, np.float32)
    ane.check(ane.lib.ane_q4_k_gemv(M, K, x.ctypes.data, W.ctypes.data, out.ctypes.data))
    assert np.array_equal(out.view(np.uint32), np.zeros(M, np.uint32))


def test_get_rows_q4_0_kat(ane):
    """The reference's get_rows_q4_0 tables (tests/test_remaining_ops.cpp:328-430)."""
    import torch

    for table, idx, dim, ref in get_rows_q4_0_kat_tables():
        got = ane.get_rows_q4_0(torch.from_numpy(table).cuda(), torch.from_numpy(idx.astype(np.int32)).cuda(), dim)
        _same_bits(got.cpu().numpy(), ref)
        out = np.zeros((idx.size, dim), np.float32)
        ane.check(ane.lib.ane_get_rows_q4_0(idx.size, dim, table.ctypes.data, idx.ctypes.data, out.ctypes.data))
        _same_bits(out, ref)


def test_get_rows_q4_0_random_with_special_scales(ane):
    import torch

    rng = np.random.default_rng(5)
    vocab, dim = 1000, 4096
    table = rng.integers(0, 256, size=(vocab, dim // 32, 18), dtype=np.uint8)
    table[:, :, 0:2] = (rng.random((vocab, dim // 32)) * 0.1).astype(np.float16).view(np.uint8).reshape(
        vocab, dim // 32, 2)
    table[3, 0, 0:2] = np.frombuffer(np.float16(np.inf).tobytes(), np.uint8)
    table[3, 1, 0:2] = np.frombuffer(np.float16(np.nan).tobytes(), np.uint8)
    table[3, 2, 0:2] = np.frombuffer(np.float16(6e-8).tobytes(), np.uint8)
    table = table.reshape(-1)
    idx = np.array([3, 999, 0, 3, 512], np.uint32)
    ref = oracle.get_rows_q4_0(table, idx, dim)
    got = ane.get_rows_q4_0(torch.from_numpy(table).cuda(), torch.from_numpy(idx.astype(np.int32)).cuda(), dim)
    _same_bits(got.cpu().numpy(), ref)
