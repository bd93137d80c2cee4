"""Pin the CPU oracle against the reference's own known-answer tests (CPU only).

Fixtures come from tests/golden/make_golden.py, which restates the input
patterns and CPU checker loops of the reference's test files.  A second,
independent numpy restatement of each opcode is checked against the C oracle
on seeded random inputs, including the edge cases the asm handles specially
(all-zero input, NaN, ties at .5, the -127 clamp, fp16 subnormal scales).
"""
import numpy as np
import pytest

import oracle

F32 = np.float32


# ----------------------------------------------------------- reference fixtures
def test_igemm_exact_kat(kats):
    """test_remaining_ops.cpp:131-184: exact int8 GEMM, 16x32x64."""
    A, B, ref = kats["igemm_A"], kats["igemm_B"], kats["igemm_ref_i32"]
    acc = oracle.gemm_s8_s32(A, B)
    assert np.array_equal(acc, ref)


def test_cblas_igemm_oracle_kat(kats):
    """The KAT through the integer CBLAS GEMM (opcode 0x61) in all four transpose
    layouts, alpha 1 and 0.5 (test_remaining_ops.cpp:131-184)."""
    A, B = kats["igemm_A"], kats["igemm_B"]
    M, K = A.shape
    N = B.shape[1]
    for alpha, ref in ((1.0, kats["igemm_ref_alpha1"]), (0.5, kats["igemm_ref_alpha05"])):
        for ta in (0, 1):
            for tb in (0, 1):
                Aop = np.ascontiguousarray(A.T if ta else A)
                Bop = np.ascontiguousarray(B.T if tb else B)
                C = np.full(M * N, 7.0, F32)
                oracle.int_gemm("igemm", ta | (tb << 1), M, N, K, Aop.shape[1], Bop.shape[1], N, alpha, 0.0,
                                Aop.view(np.uint8), Bop.view(np.uint8), C)
                assert np.array_equal(C.reshape(M, N), ref), (alpha, ta, tb)


def test_int_gemm_oracle_numpy_restatement():
    """ugemm / usgemm (uint32 / int32 conversion) and the beta != 0 accumulator
    seeding, against an independent numpy restatement; strided ldc."""
    rng = np.random.default_rng(5)
    M, N, K, ldc = 20, 37, 128, 40
    A = rng.integers(0, 256, (M, K), dtype=np.uint8)
    B = rng.integers(0, 256, (K, N), dtype=np.uint8)
    for kind in ("igemm", "ugemm", "usgemm"):
        for beta in (0.0, 0.75):
            C0 = rng.standard_normal(M * ldc).astype(F32)
            C = C0.copy()
            oracle.int_gemm(kind, 0, M, N, K, K, N, ldc, np.float32(1.25), np.float32(beta), A, B, C)
            a = A.astype(np.int64) if kind != "igemm" else A.view(np.int8).astype(np.int64)
            b = B.astype(np.int64) if kind == "ugemm" else B.view(np.int8).astype(np.int64)
            acc = (a @ b) & 0xFFFFFFFF
            cin = C0.reshape(M, ldc)[:, :N]
            if beta != 0.0:
                seed = (cin * np.float32(beta)).astype(F32).view(np.uint32).astype(np.int64)
                acc = (acc + seed) & 0xFFFFFFFF
            acc = acc.astype(np.uint32)
            f = acc.astype(np.float32) if kind == "ugemm" else acc.view(np.int32).astype(np.float32)
            ref = (f * np.float32(1.25)).astype(F32)
            got = C.reshape(M, ldc)
            assert np.array_equal(got[:, :N], ref), (kind, beta)
            assert np.array_equal(got[:, N:], C0.reshape(M, ldc)[:, N:])  # columns past N untouched


def test_dense_u8s8_oracle_matches_widened_dense_i8():
    """dense_u8s8 = dense_i8 with unsigned A: exact int sums, same epilogue."""
    rng = np.random.default_rng(6)
    M, N, K = 50, 128, 784
    K64 = (K + 63) // 64 * 64
    M16 = (M + 15) // 16 * 16
    A = np.zeros((M16, K64), np.uint8)
    A[:M, :K] = rng.integers(0, 256, (M, K), dtype=np.uint8)
    B = rng.integers(-127, 128, (K64, N)).astype(np.int8)
    B[K:] = 0
    bias = rng.standard_normal(N).astype(F32)
    Bp = oracle.pack_b_i8(B, K64, N)
    C = oracle.dense_u8s8(M, N, K, 0.01, 0.02, 1, A, Bp, bias)
    acc = (A.astype(np.int64) @ B.astype(np.int64)).astype(np.float32)
    y = (acc * np.float32(np.float32(0.01) * np.float32(0.02))).astype(F32) + bias
    assert np.array_equal(C, np.maximum(y, F32(0)) + F32(0))


def test_igemm_via_pack_and_dense_i8(kats):
    """The same KAT through pack_b_i8 + dense_i8 (sa=sb=1, zero bias)."""
    A, B, ref = kats["igemm_A"], kats["igemm_B"], kats["igemm_ref_alpha1"]
    M, K = A.shape
    N = B.shape[1]
    Bp = oracle.pack_b_i8(B, K, N)
    C = oracle.dense_i8(M, N, K, 1.0, 1.0, 0, A, Bp, np.zeros(32, F32))
    assert np.max(np.abs(C[:M] - ref)) <= kats["igemm_tol"]
    assert np.array_equal(C[:M], ref)  # exact: |acc| < 2^24
    C5 = oracle.dense_i8(M, N, K, 0.5, 1.0, 0, A, Bp, np.zeros(32, F32))
    assert np.array_equal(C5[:M], kats["igemm_ref_alpha05"])


@pytest.mark.parametrize("dim", [32, 64])
def test_q8_0_format_kat(kats, dim):
    """test_remaining_ops.cpp:230-325: Q8_0 block layout and dequant."""
    table = kats[f"q8rows{dim}_table"]
    out = oracle.get_rows_q8_0(table, kats["q8rows_idx"], dim)
    ref = kats[f"q8rows{dim}_ref"]
    assert np.max(np.abs(out - ref)) <= kats["q8rows_tol"]


@pytest.mark.parametrize("dim", [32, 64])
def test_q8_0_gemv_on_kat_tables(kats, dim):
    """q8_0_gemv over the KAT tables: every row, x = pattern; compare with double."""
    table = kats[f"q8rows{dim}_table"]
    rows = table.shape[0]
    x = ((np.arange(dim) % 7) - 3).astype(F32) * F32(0.25)
    out = oracle.q8_0_gemv(table, x, rows, dim)
    deq = oracle.get_rows_q8_0(table, np.arange(rows), dim).astype(np.float64)
    ref = deq @ x.astype(np.float64)
    assert np.allclose(out, ref, rtol=1e-6, atol=1e-6)


def test_quantize_roundtrip_kat(kats):
    """test_dsl_coverage.cpp:334-368: quantize -> dequantize round trip."""
    x = kats["qrt_x"]
    q, s = oracle.quantize_fp32_i8(x)
    assert s == kats["qrt_scale"]
    assert np.array_equal(q, kats["qrt_q"])
    back = oracle.dequantize_i8_fp32(q, s)
    assert np.max(np.abs(back - x)) < s * kats["qrt_bound_factor"]


def test_mnist_packing_constants(kats):
    """test_mnist_i8.cpp:43-50,165-169: padded dims and packed-B byte counts."""
    _, HID, _, INP_K, HID_K, OUT_PAD = kats["mnist_dims"]
    assert oracle.packed_b_size(int(INP_K), int(HID)) == kats["mnist_packed_bytes"][0]
    assert oracle.packed_b_size(int(HID_K), int(OUT_PAD)) == kats["mnist_packed_bytes"][1]


# ------------------------------------------------- independent numpy restatement
def np_quantize(x):
    x = x.astype(F32).ravel()
    with np.errstate(invalid="ignore"):
        am = F32(0.0) if x.size == 0 else (F32(np.nan) if np.isnan(x).any() else np.max(np.abs(x)))
    if am == 0:
        s, inv = F32(1.0), F32(127.0)
    else:
        s, inv = am / F32(127.0), F32(127.0) / am
    with np.errstate(invalid="ignore", over="ignore"):
        y = x * inv
        y = np.where(np.isnan(y), y, np.minimum(np.maximum(y, F32(-127)), F32(127)))
        q = np.where(np.isnan(y), 0, np.rint(y)).astype(np.int8)
    return q, F32(s)


def np_relu(y):
    return np.where(np.isnan(y), y, np.where(y > 0, y, F32(0.0))).astype(F32)


def np_dense_fused(A, B, scale, relu):
    qa, sa = np_quantize(A)
    qb, sb = np_quantize(B)
    M, K = A.shape
    N = B.shape[1]
    acc = qa.reshape(M, K).astype(np.int64) @ qb.reshape(K, N).astype(np.int64)
    comb = F32(sa * sb)
    y = acc.astype(np.int32).astype(F32) * comb
    y = (y * F32(scale)).astype(F32)
    return (np_relu(y) if relu else y), acc.astype(np.int32), sa, sb


@pytest.mark.parametrize("seed,M,N,K,scale,relu", [
    (1, 50, 128, 784, 1.0, True),
    (2, 50, 10, 128, 1.0, False),
    (3, 7, 33, 96, 0.125, True),
    (4, 64, 64, 256, -2.0, True),
    (5, 1, 300, 64, 3.0, False),
])
def test_dense_fused_matches_numpy(seed, M, N, K, scale, relu):
    rng = np.random.default_rng(seed)
    A = rng.standard_normal((M, K)).astype(F32)
    B = rng.standard_normal((K, N)).astype(F32)
    A[rng.random((M, K)) < 0.01] *= 20
    C, Aq, Bq, acc, sa, sb = oracle.dense_fused_i8(A, B, scale, relu, full=True)
    Cn, accn, san, sbn = np_dense_fused(A, B, scale, relu)
    assert sa == san and sb == sbn
    assert np.array_equal(acc, accn)
    assert np.array_equal(C.view(np.uint32), Cn.view(np.uint32))
    Comp = oracle.dense_fused_i8_omp(A, B, scale, relu, threads=4)
    assert np.array_equal(C.view(np.uint32), Comp.view(np.uint32))


def test_quantize_edge_cases():
    # all zero -> scale 1, codes 0
    q, s = oracle.quantize_fp32_i8(np.zeros(32, F32))
    assert s == 1.0 and not q.any()
    # ties round to even; exact +-127 at the absmax
    x = np.array([127.0, -127.0, 0.5, 1.5, 2.5, -0.5, -1.5, 126.5], F32)
    q, s = oracle.quantize_fp32_i8(x)
    assert s == F32(1.0)
    assert list(q) == [127, -127, 0, 2, 2, 0, -2, 126]
    # NaN anywhere -> NaN scale, every code 0 (fcvtzs(NaN) = 0)
    x = np.ones(16, F32)
    x[5] = np.nan
    q, s = oracle.quantize_fp32_i8(x)
    assert np.isnan(s) and not q.any()
    # inf -> scale inf, inv 0 -> finite codes 0, inf*0 = NaN -> 0
    x = np.ones(16, F32)
    x[3] = np.inf
    q, s = oracle.quantize_fp32_i8(x)
    assert np.isinf(s) and not q.any()
    # never -128
    rng = np.random.default_rng(0)
    x = rng.standard_normal(4096).astype(F32)
    q, _ = oracle.quantize_fp32_i8(x)
    assert q.min() >= -127 and q.max() <= 127
    qn, _ = np_quantize(x)
    assert np.array_equal(q, qn)


def test_relu_max_semantics():
    assert np.signbit(F32(oracle.lib().ane_ref_relu_max(-0.0, 0.0))) == False  # noqa: E712
    assert np.isnan(oracle.lib().ane_ref_relu_max(float("nan"), 0.0))
    assert oracle.lib().ane_ref_relu_max(-5.0, 0.0) == 0.0


def test_fp16_conversions_match_numpy():
    bits = np.arange(65536, dtype=np.uint32).astype(np.uint16)
    ref = bits.view(np.float16).astype(F32)
    got = np.array([oracle.fp16_to_fp32(int(b)) for b in bits[::7]], F32)
    r = ref[::7]
    nan = np.isnan(r)
    assert np.array_equal(np.isnan(got), nan)
    assert np.array_equal(got[~nan].view(np.uint32), r[~nan].view(np.uint32))
    rng = np.random.default_rng(1)
    vals = np.concatenate([rng.standard_normal(2000).astype(F32) * F32(10.0) ** rng.integers(-9, 6, 2000),
                           np.array([65504, 65519.99, 65520, 1e-8, 2.98e-8, 5.96e-8, -6.1e-5, 0.0], F32)])
    for v in vals.astype(F32):
        assert oracle.fp32_to_fp16(float(v)) == np.array([v], F32).astype(np.float16).view(np.uint16)[0]


def test_channelwise_is_per_row_quantize():
    rng = np.random.default_rng(3)
    x = rng.standard_normal((9, 48)).astype(F32)
    x[4] = 0
    q, s = oracle.quantize_fp32_i8_channelwise(x)
    for r in range(9):
        qr, sr = np_quantize(x[r])
        assert s[r] == sr and np.array_equal(q[r], qr)


def test_pack_b_layout():
    rng = np.random.default_rng(5)
    K, N = 70, 37
    B = rng.integers(-127, 128, (K, N)).astype(np.int8)
    P = oracle.pack_b_i8(B, K, N)
    G = (K + 3) // 4
    for p in range((N + 15) // 16):
        for g in range(G):
            for c in range(16):
                for d in range(4):
                    k, n = 4 * g + d, 16 * p + c
                    exp = B[k, n] if (k < K and n < N) else 0
                    assert P[(p * G + g) * 64 + c * 4 + d] == exp


def test_dense_i8_reference_contract():
    """dense_i8 with K padded to 64, B packed with K64, bias of N32, relu floor."""
    rng = np.random.default_rng(7)
    M, N, K = 50, 10, 100
    K64 = 128
    A = np.zeros((64, K64), np.int8)
    A[:M, :K] = rng.integers(-127, 128, (M, K))
    B = np.zeros((K64, N), np.int8)
    B[:K] = rng.integers(-127, 128, (K, N))
    Bp = oracle.pack_b_i8(B, K64, N)
    bias = np.zeros(32, F32)
    bias[:N] = rng.standard_normal(N).astype(F32)
    C = oracle.dense_i8(M, N, K, 0.01, 0.02, 1, A, Bp, bias)
    acc = A[:, :K].astype(np.int64) @ B[:K].astype(np.int64)
    comb = F32(F32(0.01) * F32(0.02))
    y = (acc.astype(F32) * comb + bias[:N]).astype(F32)
    assert np.array_equal(C, np_relu(y))


def test_q8_0_gemv_lane_order_and_modes():
    rng = np.random.default_rng(11)
    M, K = 37, 256
    Wf = (rng.standard_normal((M, K)) * 0.02).astype(F32)
    W = oracle.quantize_q8_0(Wf, M, K)
    x = rng.standard_normal(K).astype(F32)
    out = oracle.q8_0_gemv(W, x, M, K)
    # numpy restatement of the 16-lane FMA chains and the FADDV tree
    Wb = W.reshape(M, K // 32, 34)
    d = Wb[:, :, 0:2].copy().view(np.float16)[..., 0].astype(F32)
    qs = Wb[:, :, 2:].view(np.int8).astype(F32)
    acc = np.zeros((M, 16), np.float64)
    accf = np.zeros((M, 16), F32)
    for b in range(K // 32):
        for half in range(2):
            dq = (qs[:, b, half * 16:(half + 1) * 16] * d[:, b:b + 1]).astype(F32)
            xv = x[b * 32 + half * 16: b * 32 + half * 16 + 16]
            # fma: exact product + acc, one rounding (float64 holds both exactly)
            accf = (dq.astype(np.float64) * xv.astype(np.float64) + accf.astype(np.float64)).astype(F32)
    s = accf
    while s.shape[1] > 1:
        s = (s[:, 0::2] + s[:, 1::2]).astype(F32)
    assert np.array_equal(out.view(np.uint32), s[:, 0].view(np.uint32))
    out_omp = oracle.q8_0_gemv_omp(W, x, M, K, threads=3)
    assert np.array_equal(out.view(np.uint32), out_omp.view(np.uint32))
    # mode Q: int32 block dots exact, fp32 output close to mode R
    xq = oracle.quantize_q8_0(x, 1, K)
    outq, dots = oracle.q8_0_gemv_q8(W, xq, M, K, with_dots=True)
    xqb = xq.reshape(K // 32, 34)[:, 2:].view(np.int8).astype(np.int64)
    ref_dots = np.einsum("mbj,bj->mb", Wb[:, :, 2:].view(np.int8).astype(np.int64), xqb)
    assert np.array_equal(dots, ref_dots.astype(np.int32))
    del acc
    assert np.allclose(outq, out, rtol=0.05, atol=0.05)


def test_mnist_fp32_ops_oracle_sanity():
    """The MNIST-i8 training opcodes' restatements against numpy: exact for the
    data movement ops, within the reference polynomial's accuracy for softmax."""
    rng = np.random.default_rng(8)
    x = rng.standard_normal((50, 128)).astype(F32)
    assert np.array_equal(oracle.transpose_fp32(x), x.T)
    g = rng.standard_normal(x.size).astype(F32)
    assert np.array_equal(oracle.relu_backward_fp32(x, g), np.where(x.ravel() > 0, g, F32(0)))
    pred = rng.integers(0, 10, 50).astype(np.int32)
    lab = rng.integers(0, 10, 50).astype(np.uint8)
    assert oracle.count_matches(pred, lab) == int((pred == lab).sum())
    # dense_fp32: K = 50 uses only the first 48 k (the handler's whole 16-blocks)
    A = rng.standard_normal((128, 50)).astype(F32)
    B = rng.standard_normal((50, 16)).astype(F32)
    bias = rng.standard_normal(16).astype(F32)
    C = oracle.dense_fp32(128, 16, 50, 0.5, 0, A, B, bias)
    ref = (bias.astype(np.float64) + A[:, :48].astype(np.float64) @ B[:48].astype(np.float64)) * 0.5
    assert np.max(np.abs(C - ref)) < 1e-4
    logits = (rng.standard_normal((50, 16)) * 4).astype(F32)
    labels = rng.integers(0, 10, 50).astype(np.uint8)
    probs, gout, am = oracle.softmax_argmax_fp32(logits, labels)
    sm = np.exp(logits.astype(np.float64) - logits.max(1, keepdims=True))
    sm /= sm.sum(1, keepdims=True)
    assert np.max(np.abs(probs - sm)) < 2e-4
    assert np.array_equal(am, probs.argmax(1))
    onehot = np.zeros_like(probs)
    onehot[np.arange(50), labels] = 1
    assert np.array_equal(gout, (probs - onehot).astype(F32))


# ------------------------------------------------ K-quant matvecs, get_rows_q4_0
from kquant_util import BLOCK_BYTES, dequant_row, get_rows_q4_0_kat_tables, random_blocks  # noqa: E402


def test_get_rows_q4_0_oracle_kat():
    """The reference's get_rows_q4_0 test tables and expectations."""
    for table, idx, dim, ref in get_rows_q4_0_kat_tables():
        got = oracle.get_rows_q4_0(table, idx, dim)
        assert np.array_equal(got.view(np.uint32), ref.view(np.uint32))


@pytest.mark.parametrize("fmt", sorted(BLOCK_BYTES))
def test_kquant_oracle_decoding_matches_numpy(fmt):
    """The C oracle's layouts against an independent numpy dequantizer (float64
    dot products, so a tolerance: the oracle's FMA order is checked on the GPU
    side, bit for bit, and by the lane-order test below)."""
    rng = np.random.default_rng(7)
    M, K = 6, 512
    W = random_blocks(fmt, M, K, rng)
    x = rng.standard_normal(K).astype(np.float32)
    x[3] = 0.0                                   # q3_k: a stale shift of 0 keeps the codes
    x[40] = np.uint32(5).view(np.float32)        # a tiny denormal: shift by 5
    got = oracle.kquant_gemv(fmt, W, x, M, K)
    rows = W.reshape(M, -1)
    for m in range(M):
        ref = float(np.dot(dequant_row(fmt, rows[m], x), x.astype(np.float64)))
        scale = float(np.abs(dequant_row(fmt, rows[m], x)).dot(np.abs(x.astype(np.float64)))) + 1e-30
        assert abs(float(got[m]) - ref) <= 1e-5 * scale, (fmt, m, got[m], ref)


def test_kquant_oracle_lane_order():
    """One nonzero lane of the 16: the FADDV tree and lane FMA chains reduce to
    that lane's fused chain; a q4_k row with a single 1.0 weight at element e
    returns x[e] exactly."""
    K = 256
    W = np.zeros(144, np.uint8)
    W[0:2] = np.frombuffer(np.float16(1.0).tobytes(), np.uint8)   # d = 1, dmin = 0
    W[4] = 1                                                      # sub-block 0: sc = 1, m = 0
    W[16 + 5] = 0x01                                              # element 5 = 1 (low nibble)
    x = np.arange(K, dtype=np.float32) * 0.5 + 1.0
    assert oracle.kquant_gemv("q4_k", W, x, 1, K)[0] == x[5]


def test_mul_mat_q8_0_batch_oracle_matches_numpy_segments():
    """The batched Q8_0 MUL_MAT oracle against a numpy restatement of its
    contract: per (token, row) the terms float(sumi) * (dw * dx) (separate fp32
    roundings), summed from +0 in block order within segments of 32 blocks, the
    segment sums added from +0 in segment order -- exact, float32 numpy."""
    rng = np.random.default_rng(17)
    for M, K, NT in [(24, 4096, 5), (9, 11008, 3), (16, 256, 2)]:
        W = oracle.quantize_q8_0((rng.standard_normal((M, K)) * 0.02).astype(np.float32), M, K)
        x = rng.standard_normal((NT, K)).astype(np.float32)
        xq = oracle.quantize_q8_0(x, NT, K)
        nb = K // 32
        Wb = W.reshape(M, nb, 34)
        Xb = xq.reshape(NT, nb, 34)
        dw = Wb[:, :, 0:2].copy().view(np.float16).reshape(M, nb).astype(np.float32)
        dx = Xb[:, :, 0:2].copy().view(np.float16).reshape(NT, nb).astype(np.float32)
        qw = Wb[:, :, 2:].view(np.int8).astype(np.int32)
        qx = Xb[:, :, 2:].view(np.int8).astype(np.int32)
        sumi = np.einsum("mbk,tbk->tmb", qw, qx)          # exact int32 block dots
        total = np.zeros((NT, M), np.float32)
        for s0 in range(0, nb, 32):
            seg = np.zeros((NT, M), np.float32)
            for b in range(s0, min(s0 + 32, nb)):
                p = (dw[None, :, b] * dx[:, None, b]).astype(np.float32)
                seg = (seg + sumi[:, :, b].astype(np.float32) * p).astype(np.float32)
            total = (total + seg).astype(np.float32)
        got = oracle.mul_mat_q8_0_batch(W, xq, M, K, NT)
        assert np.array_equal(got.view(np.uint32), total.view(np.uint32)), (M, K, NT)


def test_q4_0_gemv_oracle_layout():
    """q4_0_gemv oracle: element i < 16 of a block is the low nibble of byte i,
    element 16 + i its high nibble, value (nibble - 8) * d -- a numpy dequant
    dotted in float64 (a tolerance: the lane FMA order is checked on the GPU bit
    for bit), and a single nonzero weight returning x[e] * d exactly."""
    rng = np.random.default_rng(23)
    M, K = 5, 512
    nb = K // 32
    W = rng.integers(0, 256, size=(M, nb, 18), dtype=np.uint8)
    W[:, :, 0:2] = (rng.random((M, nb)) * 0.05 + 0.01).astype(np.float16).view(np.uint8).reshape(M, nb, 2)
    x = rng.standard_normal(K).astype(np.float32)
    got = oracle.q4_0_gemv(W.reshape(-1), x, M, K)
    d = W[:, :, 0:2].copy().view(np.float16).reshape(M, nb).astype(np.float64)
    q = W[:, :, 2:].astype(np.int64)
    vals = np.concatenate([(q & 15) - 8, (q >> 4) - 8], axis=2) * d[:, :, None]   # [M, nb, 32]
    ref = vals.reshape(M, K) @ x.astype(np.float64)
    scale = np.abs(vals.reshape(M, K)) @ np.abs(x.astype(np.float64))
    assert np.all(np.abs(got - ref) <= 1e-5 * scale)
    # one nonzero weight: element 21 of block 1 (high nibble of byte 5) = 9 - 8 = 1
    W1 = np.zeros((1, nb, 18), np.uint8)
    W1[:, :, 2:] = 0x88                                          # every code 8 -> value 0
    W1[0, 1, 0:2] = np.frombuffer(np.float16(0.5).tobytes(), np.uint8)
    W1[0, 1, 2 + 5] = 0x98                                       # high nibble 9 -> element 16 + 5
    assert oracle.q4_0_gemv(W1.reshape(-1), x, 1, K)[0] == np.float32(x[32 + 21] * np.float32(0.5))
