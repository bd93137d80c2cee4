"""dense_u8s8 (0x1E), the integer CBLAS GEMMs (0x61 cblas_igemm, 0x62
cblas_ugemm, 0x63 cblas_usgemm), get_rows_q8_0 (0x7C) and q4_0_gemv (0x58) on
the GPU, bit-exact against the oracle, through the device entry point, the host
entry point and stream_exec."""
import numpy as np
import pytest

import oracle

pytestmark = pytest.mark.gpu
F32 = np.float32


def _layout(M, N, K, ta, tb, pad, rng):
    lda = (M if ta else K) + pad
    ldb = (K if tb else N) + pad
    A = rng.integers(0, 256, ((K if ta else M) * lda,), dtype=np.uint8)
    B = rng.integers(0, 256, ((N if tb else K) * ldb,), dtype=np.uint8)
    return A, B, lda, ldb


@pytest.mark.parametrize("kind", ["igemm", "ugemm", "usgemm"])
@pytest.mark.parametrize("M,N,K", [(16, 32, 64), (100, 77, 192), (300, 260, 256), (129, 513, 1024)])
@pytest.mark.parametrize("ta,tb", [(0, 0), (1, 0), (0, 1), (1, 1)])
def test_int_gemm_device_exact(ane, kind, M, N, K, ta, tb):
    import torch

    rng = np.random.default_rng(M * 7 + N + K + ta * 2 + tb)
    A, B, lda, ldb = _layout(M, N, K, ta, tb, 16, rng)
    ldc = N + 3
    for beta in (0.0, 0.75):
        C0 = rng.standard_normal(M * ldc).astype(F32)
        ref = C0.copy()
        oracle.int_gemm(kind, ta | (tb << 1), M, N, K, lda, ldb, ldc, np.float32(1.25), np.float32(beta), A, B, ref)
        Cd = torch.from_numpy(C0.copy()).cuda()
        ane.cblas_int_gemm(kind, torch.from_numpy(A).cuda(), torch.from_numpy(B).cuda(), Cd, M, N, K, lda, ldb, ldc,
                           1.25, beta, bool(ta), bool(tb))
        torch.cuda.synchronize()
        assert np.array_equal(Cd.cpu().numpy().view(np.uint32), ref.view(np.uint32)), (kind, beta)


def test_int_gemm_host_and_stream_exec(ane, kats):
    """The reference KAT (test_remaining_ops.cpp:131-184) through the synchronous
    host entry point and an ane::dispatch byte stream."""
    A, B = kats["igemm_A"], kats["igemm_B"]
    M, K = A.shape
    N = B.shape[1]
    C = np.zeros((M, N), F32)
    ane.check(ane.lib.ane_cblas_igemm(0, M, N, K, K, N, N, 0.5, 0.0, A.ctypes.data, B.ctypes.data, C.ctypes.data))
    assert np.array_equal(C, kats["igemm_ref_alpha05"])
    C2 = np.zeros((M, N), F32)
    ane.dispatch(ane.Op.cblas_igemm, ane.U8(0), ane.U32(M), ane.U32(N), ane.U32(K), ane.U32(K), ane.U32(N),
                 ane.U32(N), ane.F32(1.0), ane.F32(0.0), ane.Ptr(A.ctypes.data), ane.Ptr(B.ctypes.data),
                 ane.Ptr(C2.ctypes.data))
    assert ane.lib.ane_last_error() == 0
    assert np.array_equal(C2, kats["igemm_ref_alpha1"])
    # ugemm / usgemm through stream_exec with transposes
    rng = np.random.default_rng(3)
    for op, kind in ((ane.Op.cblas_ugemm, "ugemm"), (ane.Op.cblas_usgemm, "usgemm")):
        Au, Bu, lda, ldb = _layout(40, 24, 128, 1, 1, 0, rng)
        Cu = np.zeros(40 * 24, F32)
        ref = Cu.copy()
        oracle.int_gemm(kind, 3, 40, 24, 128, lda, ldb, 24, np.float32(2.0), np.float32(0.0), Au, Bu, ref)
        ane.dispatch(op, ane.U8(3), ane.U32(40), ane.U32(24), ane.U32(128), ane.U32(lda), ane.U32(ldb), ane.U32(24),
                     ane.F32(2.0), ane.F32(0.0), ane.Ptr(Au.ctypes.data), ane.Ptr(Bu.ctypes.data),
                     ane.Ptr(Cu.ctypes.data))
        assert ane.lib.ane_last_error() == 0
        assert np.array_equal(Cu, ref), kind


def test_int_gemm_rejects_k_not_multiple_of_64(ane):
    A = np.zeros(16 * 48, np.uint8)
    B = np.zeros(48 * 16, np.uint8)
    C = np.zeros(16 * 16, F32)
    rc = ane.lib.ane_cblas_igemm(0, 16, 16, 48, 48, 16, 16, 1.0, 0.0, A.ctypes.data, B.ctypes.data, C.ctypes.data)
    assert rc == 1  # ANE_ERR_INVALID_ARGUMENT (the reference requires K % 64 == 0)


@pytest.mark.parametrize("M,N,K,relu", [(50, 128, 784, True), (300, 200, 1000, False), (16, 16, 64, True)])
def test_dense_u8s8_exact(ane, M, N, K, relu):
    """MNIST layer 1 (test_mnist_i8.cpp:304-307 runs it as dense_u8s8) and ragged
    shapes: host entry point and stream_exec, padded rows included."""
    rng = np.random.default_rng(M + N + K)
    K64 = (K + 63) // 64 * 64
    M16 = (M + 15) // 16 * 16
    A = np.zeros((M16, K64), np.uint8)
    A[:M, :K] = rng.integers(0, 256, (M, K), dtype=np.uint8)
    B = rng.integers(-127, 128, (K64, N)).astype(np.int8)
    B[K:] = 0
    bias = rng.standard_normal((N + 31) // 32 * 32).astype(F32)
    Bp = oracle.pack_b_i8(B, K64, N)
    ref = oracle.dense_u8s8(M, N, K, 0.013, 0.021, int(relu), A, Bp, bias)
    C = np.empty((M16, N), F32)
    ane.check(ane.lib.ane_dense_u8s8(M, N, K, 0.013, 0.021, int(relu), A.ctypes.data, Bp.ctypes.data,
                                     bias.ctypes.data, C.ctypes.data))
    assert np.array_equal(C.view(np.uint32), ref.view(np.uint32))
    C2 = np.empty((M16, N), F32)
    ane.dispatch(ane.Op.dense_u8s8, ane.U32(M), ane.U32(N), ane.U32(K), ane.F32(0.013), ane.F32(0.021),
                 ane.U8(int(relu)), ane.Ptr(A.ctypes.data), ane.Ptr(Bp.ctypes.data), ane.Ptr(bias.ctypes.data),
                 ane.Ptr(C2.ctypes.data))
    assert ane.lib.ane_last_error() == 0
    assert np.array_equal(C2.view(np.uint32), ref.view(np.uint32))


@pytest.mark.parametrize("dim", [32, 64])
def test_get_rows_q8_0_kat(ane, kats, dim):
    """get_rows_q8_0 (0x7C) on the reference's Q8_0 tables
    (test_remaining_ops.cpp:230-325): host entry point and stream_exec equal the
    oracle bit for bit and the reference's expected values within its bound."""
    table = np.ascontiguousarray(kats[f"q8rows{dim}_table"]).astype(np.uint8)
    idx = np.ascontiguousarray(kats["q8rows_idx"]).astype(np.uint32)
    ref = oracle.get_rows_q8_0(table, idx, dim)
    out = np.empty(idx.size * dim, F32)
    ane.check(ane.lib.ane_get_rows_q8_0(idx.size, dim, table.ctypes.data, idx.ctypes.data, out.ctypes.data))
    assert np.array_equal(out.view(np.uint32), np.asarray(ref, F32).ravel().view(np.uint32))
    assert np.max(np.abs(out.reshape(idx.size, dim) - kats[f"q8rows{dim}_ref"])) <= kats["q8rows_tol"]
    out2 = np.empty_like(out)
    ane.dispatch(ane.Op.get_rows_q8_0, ane.U32(idx.size), ane.U32(dim), ane.Ptr(table.ctypes.data),
                 ane.Ptr(idx.ctypes.data), ane.Ptr(out2.ctypes.data))
    assert ane.lib.ane_last_error() == 0
    assert np.array_equal(out2, out)


def test_get_rows_q8_0_device_large(ane):
    """Device entry point: 4096 random row lookups from a 32000 x 4096 Q8_0 table
    (a 7B embedding shape), repeated and out-of-order indices."""
    import torch

    rows, dim, n = 32000, 4096, 4096
    g = torch.Generator(device="cuda").manual_seed(9)
    table = torch.randint(0, 256, (rows * (dim // 32) * 34,), dtype=torch.uint8, device="cuda", generator=g)
    table.view(-1, 34)[:, 1] = 0x1C  # finite fp16 scales
    idx = torch.randint(0, rows, (n,), dtype=torch.int32, device="cuda", generator=g)
    idx[:8] = idx[0]
    out = torch.empty(n * dim, dtype=torch.float32, device="cuda")
    ane.check(ane.lib.ane_get_rows_q8_0_dev(n, dim, table.data_ptr(), idx.data_ptr(), out.data_ptr(), None))
    torch.cuda.synchronize()
    ref = oracle.get_rows_q8_0(table.cpu().numpy(), idx.cpu().numpy().astype(np.uint32), dim)
    assert np.array_equal(out.cpu().numpy().view(np.uint32), np.asarray(ref, F32).ravel().view(np.uint32))


def _q4_weights(M, K, rng):
    W = rng.integers(0, 256, (M * (K // 32), 18), dtype=np.uint8)
    W[:, 0:2] = np.frombuffer((rng.standard_normal(M * (K // 32)) * 0.01).astype(np.float16).tobytes(),
                              np.uint8).reshape(-1, 2)
    return W


@pytest.mark.parametrize("M,K", [(4096, 4096), (11008, 4096), (4096, 11008), (333, 768), (64, 96), (5, 32)])
def test_q4_0_gemv_exact(ane, M, K):
    """q4_0_gemv (0x58): the streamed kernel (K % 256 == 0; K = 768 and 11008 end
    on a half chunk) and the generic kernel (K = 96, 32), bit-exact."""
    import torch

    rng = np.random.default_rng(M + K)
    W = _q4_weights(M, K, rng)
    x = rng.standard_normal(K).astype(F32)
    ref = oracle.q4_0_gemv(W, x, M, K)
    Wd, xd = torch.from_numpy(W.ravel()).cuda(), torch.from_numpy(x).cuda()
    for st in (False, True):
        y = ane.q4_0_gemv(Wd, xd, M, K, static_weights=st)
        assert np.array_equal(y.cpu().numpy().view(np.uint32), ref.view(np.uint32)), st


def test_q4_0_gemv_special_scales_host_and_stream_exec(ane):
    """inf / NaN / zero / subnormal fp16 scales (the non-finite rows take the
    replay path) through the host entry point and an ane::dispatch stream."""
    rng = np.random.default_rng(4)
    M, K = 96, 512
    W = _q4_weights(M, K, rng).reshape(M, K // 32, 18)
    for row, blk, val in ((1, 0, np.inf), (2, 3, -np.inf), (3, 5, np.nan), (4, 1, 0.0), (5, 2, 6e-8)):
        W[row, blk, 0:2] = np.frombuffer(np.float16(val).tobytes(), np.uint8)
    W[6, 4, 2:] = 0x88  # every nibble 8: value 0, times inf below
    W[6, 4, 0:2] = np.frombuffer(np.float16(np.inf).tobytes(), np.uint8)
    W = np.ascontiguousarray(W.ravel())
    x = rng.standard_normal(K).astype(F32)
    ref = oracle.q4_0_gemv(W, x, M, K)
    out = np.empty(M, F32)
    ane.check(ane.lib.ane_q4_0_gemv(M, K, x.ctypes.data, W.ctypes.data, out.ctypes.data))
    nan = np.isnan(ref)
    assert np.array_equal(np.isnan(out), nan) and np.array_equal(out[~nan].view(np.uint32), ref[~nan].view(np.uint32))
    out2 = np.empty(M, F32)
    ane.dispatch(ane.Op.q4_0_gemv, ane.U32(M), ane.U32(K), ane.Ptr(x.ctypes.data), ane.Ptr(W.ctypes.data),
                 ane.Ptr(out2.ctypes.data))
    assert ane.lib.ane_last_error() == 0
    assert np.array_equal(np.isnan(out2), nan) and np.array_equal(out2[~nan].view(np.uint32),
                                                                   ref[~nan].view(np.uint32))
