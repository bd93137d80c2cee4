"""GPU parity: every CUDA kernel of libane_b200 against the CPU oracle.

Bars: int8 codes, scales and int32 accumulators
bit-exact; fp32 outputs bit-exact as well, because the GPU epilogues replay the
reference's fp32 operation order (the stated tolerance, 1e-5 relative, is the
fallback bar and is asserted too).  All calls go through the C ABI.
"""
import ctypes

import numpy as np
import pytest

import oracle

pytestmark = pytest.mark.gpu

F32 = np.float32
REL_TOL = 1e-5  # north_star: fp32 outputs within 1e-5 relative


def bits_equal(a, b):
    a = np.ascontiguousarray(a, F32)
    b = np.ascontiguousarray(b, F32)
    nan = np.isnan(a) | np.isnan(b)
    ok = np.array_equal(np.isnan(a), np.isnan(b)) and np.array_equal(a[~nan].view(np.uint32),
                                                                     b[~nan].view(np.uint32))
    if not ok and a.shape == b.shape:
        diff = (a.view(np.uint32) != b.view(np.uint32)) & ~(np.isnan(a) & np.isnan(b))
        idx = np.argwhere(diff)
        print(f"bits_equal: {len(idx)} of {a.size} differ; first {idx[:8].tolist()}; "
              f"got {a[diff][:8].tolist()} want {b[diff][:8].tolist()}")
        if a.ndim == 2:
            rows, cols = np.unique(idx[:, 0]), np.unique(idx[:, 1])
            print(f"  rows {rows.min()}..{rows.max()} ({rows.size}), cols {cols.min()}..{cols.max()} ({cols.size})")
    return ok


def assert_close_rel(got, ref, rtol=REL_TOL):
    got = np.asarray(got, np.float64)
    ref = np.asarray(ref, np.float64)
    scale = np.maximum(np.abs(ref), 1e-30)
    assert np.all(np.abs(got - ref) <= rtol * scale + 1e-30)


def P(a):
    return a.ctypes.data


# ------------------------------------------------------------------ quantize
@pytest.mark.parametrize("count", [16, 256, 1000, 4096 * 17, 3 * 1024 * 1024 + 5])
def test_quantize_fp32_i8_host_entry(ane, count):
    rng = np.random.default_rng(count)
    x = rng.standard_normal(count).astype(F32)
    x[rng.random(count) < 0.01] *= 20
    q = np.empty(count, np.int8)
    s = np.zeros(1, F32)
    ane.check(ane.lib.ane_quantize_fp32_i8(count, P(x), P(q), P(s)))
    qr, sr = oracle.quantize_fp32_i8(x)
    assert s[0] == sr
    assert np.array_equal(q, qr)


@pytest.mark.parametrize("case", ["zeros", "nan", "inf", "ties", "neg_zero"])
def test_quantize_edge_cases(ane, case):
    x = np.zeros(64, F32)
    if case == "nan":
        x[:] = 1.0
        x[17] = np.nan
    elif case == "inf":
        x[:] = 2.0
        x[3] = -np.inf
    elif case == "ties":
        x[:8] = [127.0, -127.0, 0.5, 1.5, 2.5, -0.5, -1.5, 126.5]
    elif case == "neg_zero":
        x[:] = -0.0
    q = np.full(64, 99, np.int8)
    s = np.zeros(1, F32)
    ane.check(ane.lib.ane_quantize_fp32_i8(64, P(x), P(q), P(s)))
    qr, sr = oracle.quantize_fp32_i8(x)
    assert bits_equal(s, np.array([sr], F32))
    assert np.array_equal(q, qr)


def test_quantize_roundtrip_kat(ane, kats):
    x = kats["qrt_x"]
    q = np.empty(256, np.int8)
    s = np.zeros(1, F32)
    ane.dispatch(ane.Op.quantize_fp32_i8, ane.U32(256), ane.Ptr(P(x)), ane.Ptr(P(q)), ane.Ptr(P(s)))
    assert s[0] == kats["qrt_scale"] and np.array_equal(q, kats["qrt_q"])
    back = np.empty(256, F32)
    ane.dispatch(ane.Op.dequantize_i8_fp32, ane.U32(256), ane.F32(float(s[0])), ane.Ptr(P(q)), ane.Ptr(P(back)))
    assert bits_equal(back, oracle.dequantize_i8_fp32(q, s[0]))
    assert np.max(np.abs(back - x)) < s[0] * kats["qrt_bound_factor"]


def test_channelwise(ane):
    rng = np.random.default_rng(9)
    x = rng.standard_normal((37, 80)).astype(F32)
    x[5] = 0
    q = np.empty_like(x, dtype=np.int8)
    s = np.empty(37, F32)
    ane.check(ane.lib.ane_quantize_fp32_i8_channelwise(37, 80, P(x), P(q), P(s)))
    qr, sr = oracle.quantize_fp32_i8_channelwise(x)
    assert np.array_equal(q, qr) and bits_equal(s, sr)


# ---------------------------------------------------------------- pack / dense_i8
@pytest.mark.parametrize("K,N", [(64, 32), (832, 128), (128, 16), (70, 37), (4, 1)])
def test_pack_b_i8(ane, K, N):
    rng = np.random.default_rng(K * N)
    B = rng.integers(-127, 128, (K, N)).astype(np.int8)
    out = np.full(oracle.packed_b_size(K, N), 77, np.int8)
    ane.check(ane.lib.ane_pack_b_i8(K, N, P(B), P(out)))
    assert np.array_equal(out, oracle.pack_b_i8(B, K, N))


def _dense_i8_case(ane, M, N, K, sa, sb, relu, bias_vals, seed):
    rng = np.random.default_rng(seed)
    M16, K64, N32 = (M + 15) // 16 * 16, (K + 63) // 64 * 64, (N + 31) // 32 * 32
    A = np.zeros((M16, K64), np.int8)
    A[:M, :K] = rng.integers(-127, 128, (M, K))
    B = np.zeros((K64, N), np.int8)
    B[:K] = rng.integers(-127, 128, (K, N))
    Bp = oracle.pack_b_i8(B, K64, N)
    Bp_full = np.zeros(oracle.packed_b_size(K64, N32), np.int8)
    Bp_full[:Bp.size] = Bp
    bias = np.zeros(N32, F32)
    bias[:N] = bias_vals(rng, N)
    C = np.full((M16, N), np.nan, F32)
    ane.dispatch(ane.Op.dense_i8, ane.U32(M), ane.U32(N), ane.U32(K), ane.F32(sa), ane.F32(sb), bool(relu),
                 ane.Ptr(P(A)), ane.Ptr(P(Bp_full)), ane.Ptr(P(bias)), ane.Ptr(P(C)))
    ref = oracle.dense_i8(M, N, K, sa, sb, 1 if relu else 0, A, Bp, bias)
    assert bits_equal(C, ref)


def test_dense_i8_igemm_kat(ane, kats):
    A, B = kats["igemm_A"], kats["igemm_B"]
    Bp = oracle.pack_b_i8(B, 64, 32)
    C = np.zeros((16, 32), F32)
    ane.dispatch(ane.Op.dense_i8, ane.U32(16), ane.U32(32), ane.U32(64), ane.F32(1.0), ane.F32(1.0), False,
                 ane.Ptr(P(A)), ane.Ptr(P(Bp)), ane.Ptr(P(np.zeros(32, F32))), ane.Ptr(P(C)))
    assert np.array_equal(C, kats["igemm_ref_alpha1"])
    C5 = np.zeros((16, 32), F32)
    ane.dispatch(ane.Op.dense_i8, ane.U32(16), ane.U32(32), ane.U32(64), ane.F32(0.5), ane.F32(1.0), False,
                 ane.Ptr(P(A)), ane.Ptr(P(Bp)), ane.Ptr(P(np.zeros(32, F32))), ane.Ptr(P(C5)))
    assert np.array_equal(C5, kats["igemm_ref_alpha05"])


@pytest.mark.parametrize("M,N,K,relu", [(50, 128, 832, True), (50, 16, 128, False), (1, 16, 128, False),
                                        (200, 300, 1000, True), (129, 257, 192, False)])
def test_dense_i8_mnist_and_tails(ane, M, N, K, relu):
    def logit_bias(rng, n):
        b = rng.standard_normal(n).astype(F32)
        b[n - min(6, n - 1):] = -1000.0  # test_mnist_i8.cpp:46-48 padding-logit mask
        return b

    _dense_i8_case(ane, M, N, K, 0.0123, 0.0456, relu, logit_bias, M * N + K)


# ------------------------------------------------------------- int8 GEMM core
@pytest.mark.parametrize("M,N,K", [(128, 256, 128), (1, 8, 16), (7, 10, 48), (129, 257, 144), (300, 513, 1040),
                                   (512, 512, 4096), (64, 14336, 4096)])
def test_gemm_s8_int32_exact(ane, M, N, K):
    import torch

    rng = np.random.default_rng(M + N + K)
    K16 = (K + 15) // 16 * 16
    Aq = rng.integers(-127, 128, (M, K16)).astype(np.int8)
    Bt = rng.integers(-127, 128, (N, K16)).astype(np.int8)
    Aq[:, K:] = 0
    Bt[:, K:] = 0
    acc = ane.gemm_s8(torch.from_numpy(Aq).cuda(), torch.from_numpy(Bt).cuda(), raw_i32=True)
    torch.cuda.synchronize()
    ref = Aq.astype(np.int64) @ Bt.astype(np.int64).T
    assert np.array_equal(acc.cpu().numpy(), ref.astype(np.int32))


@pytest.mark.parametrize("M,N,K", [(4096, 4096, 256),   # 256 tiles on 74 pairs: last 34 cut in 2
                                   (1000, 1000, 256),   # 16 tiles: every tile cut in 4 (64 columns)
                                   (4096, 1100, 512),   # 80 tiles: last 6 cut in 4, ragged N, parts past N
                                   (3000, 2000, 384),   # 96 tiles: last 22 cut in 2, ragged M
                                   (2304, 2304, 128)])  # 81 tiles: last 7 cut in 4
def test_gemm_s8_tail_split_exact(ane, M, N, K):
    """The pair kernel's last partial wave runs as column parts of 128 or 64;
    every part is exact against an fp64 product (exact for these integers)."""
    import torch

    g = torch.Generator(device="cuda").manual_seed(M * 7 + N * 3 + K)
    Aq = torch.randint(-127, 128, (M, K), generator=g, device="cuda", dtype=torch.int8)
    Bt = torch.randint(-127, 128, (N, K), generator=g, device="cuda", dtype=torch.int8)
    acc = ane.gemm_s8(Aq, Bt, raw_i32=True)
    ref = (Aq.double() @ Bt.double().T).to(torch.int32)
    assert torch.equal(acc, ref)


def _kn_operands(torch, M, N, K, seed, pad_rows_garbage=True):
    """Random int8 Aq [M x K16] (zero pad columns) and Bq [K16 x N16] in the
    layout dense_fused_i8's prologue writes.  Bq's rows K..K16 are filled with
    nonzero codes: the GEMM must cancel them through Aq's zero pad columns."""
    g = torch.Generator(device="cuda").manual_seed(seed)
    K16, N16 = (K + 15) // 16 * 16, (N + 15) // 16 * 16
    Aq = torch.randint(-127, 128, (M, K16), generator=g, device="cuda", dtype=torch.int8)
    Aq[:, K:] = 0
    Bq = torch.randint(-127, 128, (K16, N16), generator=g, device="cuda", dtype=torch.int8)
    if not pad_rows_garbage:
        Bq[K:] = 0
    return Aq, Bq


@pytest.mark.parametrize("M,N,K", [
    (4096, 4096, 256),   # pair kernel, 256 tiles on 74 pairs: the last 34 cut in 2 (64-column halves, SWIZZLE_64B)
    (1000, 1000, 256),   # every tile cut in 4: 32-column halves (SWIZZLE_32B), ragged N
    (4096, 1104, 512),   # 80 tiles: last 6 cut in 4, parts past N
    (3000, 2000, 392),   # ragged M, K % 128 != 0 (last K block partly outside Bq)
    (512, 512, 4096),    # pair kernel, whole tiles only
    (128, 256, 128),     # single-CTA kernel (M <= 128), 64-column tiles (fewest waves x width)
    (7, 10, 48),         # single-CTA kernel, N inside one 64-column tile, K16 pad rows
    (64, 14336, 4096),   # config 4 shape (single-CTA kernel, 128-column tiles)
    (1, 7168, 4096),     # config 4 at 2 GPUs, M = 1: 112 tiles of 64 columns (SWIZZLE_64B)
    (1, 14336, 4096),    # config 4 at 1 GPU, M = 1: 112 tiles of 128 columns
    (100, 37888, 256),   # 148 tiles of 256 columns: two 128-column atoms per B stage
    (33, 200, 1040),     # 64-column tiles, ragged N, K % 128 != 0
])
def test_gemm_s8_kn_int32_exact(ane, M, N, K):
    """The GEMM with B stored K x N (MN-major tcgen05 operand, the layout the
    dense_fused_i8 prologue writes): raw int32 accumulators exact against an
    fp64 product, for every tile width the kernels use."""
    import torch

    Aq, Bq = _kn_operands(torch, M, N, K, M * 5 + N * 3 + K)
    acc = ane.gemm_s8_kn(Aq, Bq, N, raw_i32=True)
    K16 = Aq.shape[1]
    ref = (Aq.double() @ Bq[:K16, :N].double()).to(torch.int32)
    assert torch.equal(acc, ref)


def test_gemm_s8_kn_equals_kmajor(ane):
    """The same codes through both B layouts give the same fp32 C, bit for bit."""
    import torch

    M, N, K = 1024, 768, 1040
    Aq, Bq = _kn_operands(torch, M, N, K, 99, pad_rows_garbage=False)
    scales = torch.tensor([0.0123, 0.0456], device="cuda")
    c_kn = ane.gemm_s8_kn(Aq, Bq, N, scales, scale=0.5, relu=True)
    c_km = ane.gemm_s8(Aq, Bq[:, :N].t().contiguous(), scales, scale=0.5, relu=True)
    assert torch.equal(c_kn.view(torch.int32), c_km.view(torch.int32))


def test_gemm_s8_extreme_values(ane):
    """All -127 / +127 operands: the largest |acc| K allows, exact."""
    import torch

    M, N, K = 256, 256, 8192
    Aq = np.full((M, K), -127, np.int8)
    Bt = np.full((N, K), 127, np.int8)
    Bt[::2] = -127
    acc = ane.gemm_s8(torch.from_numpy(Aq).cuda(), torch.from_numpy(Bt).cuda(), raw_i32=True).cpu().numpy()
    ref = Aq[:1].astype(np.int64) @ Bt.astype(np.int64).T
    assert np.array_equal(acc, np.broadcast_to(ref, (M, N)).astype(np.int32))


# ------------------------------------------------------------- dense_fused_i8
@pytest.mark.parametrize("M,N,K,scale,relu", [
    (50, 128, 784, 1.0, True),      # MNIST layer 1 (config 1)
    (50, 10, 128, 1.0, False),      # MNIST layer 2
    (1, 14336, 4096, 0.125, True),  # config 4, M=1
    (8, 14336, 4096, 0.125, True),  # config 4, M=8
    (512, 512, 512, 1.0, False),    # config 2 sweep point
    (333, 250, 100, -0.5, True),    # ragged everything, K % 16 != 0
    (16, 16, 0, 2.0, False),        # empty K
])
def test_dense_fused_i8_host_entry(ane, M, N, K, scale, relu):
    rng = np.random.default_rng(M * 7 + N + K)
    A = rng.standard_normal((M, K)).astype(F32)
    B = rng.standard_normal((K, N)).astype(F32)
    if K:
        A[rng.random((M, K)) < 0.01] *= 20  # config 4 outliers
    C = np.full((M, N), np.nan, F32)
    ane.dispatch(ane.Op.dense_fused_i8, ane.U32(M), ane.U32(N), ane.U32(K), ane.F32(scale), bool(relu),
                 ane.Ptr(P(A)), ane.Ptr(P(B)), ane.Ptr(P(C)))
    ref = oracle.dense_fused_i8(A, B, scale, relu)
    assert bits_equal(C, ref)
    assert_close_rel(C, ref)


def test_dense_fused_i8_stages_bit_exact(ane):
    """Aq, Bq, both scales and the int32 accumulators, each against the oracle."""
    import torch

    M, N, K = 300, 520, 784
    rng = np.random.default_rng(42)
    A = rng.random((M, K)).astype(F32)                      # MNIST-like U[0,1)
    B = (rng.standard_normal((K, N)) * np.sqrt(2 / K)).astype(F32)
    C, Aq_r, Bq_r, acc_r, sa_r, sb_r = oracle.dense_fused_i8(A, B, 1.0, True, full=True)
    Aq, Bq, scales = ane.quantize_pair(torch.from_numpy(A).cuda(), torch.from_numpy(B).cuda())
    K16 = Aq.shape[1]
    s = scales.cpu().numpy()
    assert s[0] == sa_r and s[1] == sb_r
    Aqn, Bqn = Aq.cpu().numpy(), Bq.cpu().numpy()
    assert np.array_equal(Aqn[:, :K], Aq_r) and not Aqn[:, K:].any()
    assert np.array_equal(Bqn[:K, :N], Bq_r) and not Bqn[:K, N:].any()
    acc = ane.gemm_s8_kn(Aq, Bq, N, raw_i32=True).cpu().numpy()
    assert np.array_equal(acc, acc_r)
    Cg = ane.gemm_s8_kn(Aq, Bq, N, scales, scale=1.0, relu=True).cpu().numpy()
    assert bits_equal(Cg, C)
    assert K16 % 16 == 0


@pytest.mark.parametrize("M,N,K", [
    (1024, 1040, 4096),   # cooperative prologue, N % 256 != 0 (ragged last B chunk rows)
    (1024, 1280, 4112),   # cooperative prologue, K % 128 != 0 (the GEMM's last K block partly outside)
    (1024, 1028, 4096),   # N % 16 != 0: the staged prologue (B codes with 16-byte padded rows)
])
def test_dense_fused_i8_coop_prologue_edges(ane, M, N, K):
    """Shapes the one-launch cooperative prologue takes (M*K + K*N >= 2^22),
    away from 4096^3: quantized operands, scales and C against the oracle."""
    import torch

    rng = np.random.default_rng(M + N + K)
    A = rng.standard_normal((M, K)).astype(F32)
    B = rng.standard_normal((K, N)).astype(F32)
    Ad, Bd = torch.from_numpy(A).cuda(), torch.from_numpy(B).cuda()
    Aq, Bq, scales = ane.quantize_pair(Ad, Bd)
    C = ane.dense_fused_i8(Ad, Bd, 0.75, True)
    torch.cuda.synchronize()
    C_r, Aq_r, Bq_r, _, sa, sb = oracle.dense_fused_i8(A, B, 0.75, True, full=True)
    s = scales.cpu().numpy()
    assert s[0] == sa and s[1] == sb
    Aqn, Bqn = Aq.cpu().numpy(), Bq.cpu().numpy()
    assert np.array_equal(Aqn[:, :K], Aq_r)
    assert np.array_equal(Bqn[:K, :N], Bq_r) and not Bqn[:K, N:].any()
    assert bits_equal(C.cpu().numpy(), C_r)


# ---------------------------------------------------------------- q8_0_gemv
@pytest.mark.parametrize("M,K", [(4096, 4096), (11008, 4096), (4096, 11008), (37, 256), (1, 32), (100, 96)])
def test_q8_0_gemv_bit_exact(ane, M, K):
    rng = np.random.default_rng(M + K)
    Wf = (rng.standard_normal((M, K)) * 0.02).astype(F32)
    W = oracle.quantize_q8_0(Wf, M, K)
    x = rng.standard_normal(K).astype(F32)
    out = np.full(M, np.nan, F32)
    ane.dispatch(ane.Op.q8_0_gemv, ane.U32(M), ane.U32(K), ane.Ptr(P(x)), ane.Ptr(P(W)), ane.Ptr(P(out)))
    ref = oracle.q8_0_gemv(W, x, M, K)
    assert bits_equal(out, ref)


def test_q8_0_gemv_special_scales(ane, kats):
    """fp16 subnormal / inf / NaN / zero block scales and the KAT tables."""
    rng = np.random.default_rng(5)
    M, K = 64, 256
    W = oracle.quantize_q8_0((rng.standard_normal((M, K)) * 0.02).astype(F32), M, K).reshape(M, K // 32, 34)
    specials = [0x0001, 0x03FF, 0x7C00, 0xFC00, 0x7E00, 0x0000, 0x8000, 0x7BFF]
    for i, h in enumerate(specials):
        W[i, i % (K // 32), 0] = h & 0xFF
        W[i, i % (K // 32), 1] = h >> 8
    W = np.ascontiguousarray(W.reshape(-1))
    x = rng.standard_normal(K).astype(F32)
    out = np.empty(M, F32)
    ane.check(ane.lib.ane_q8_0_gemv(M, K, P(x), P(W), P(out)))
    assert bits_equal(out, oracle.q8_0_gemv(W, x, M, K))
    for dim in (32, 64):
        t = kats[f"q8rows{dim}_table"]
        xx = ((np.arange(dim) % 7) - 3).astype(F32) * F32(0.25)
        o = np.empty(t.shape[0], F32)
        ane.check(ane.lib.ane_q8_0_gemv(t.shape[0], dim, P(xx), P(np.ascontiguousarray(t)), P(o)))
        assert bits_equal(o, oracle.q8_0_gemv(t, xx, t.shape[0], dim))


def test_q8_0_gemv_device_entry(ane):
    import torch

    M, K = 4096, 4096
    rng = np.random.default_rng(3)
    W = oracle.quantize_q8_0((rng.standard_normal((M, K)) * 0.02).astype(F32), M, K)
    x = rng.standard_normal(K).astype(F32)
    out = ane.q8_0_gemv(torch.from_numpy(W).cuda(), torch.from_numpy(x).cuda(), M, K)
    assert bits_equal(out.cpu().numpy(), oracle.q8_0_gemv(W, x, M, K))


# ------------------------------------------------------------------ plumbing
def test_program_runs_mnist_int8_pipeline(ane):
    """quantize W -> pack -> quantize h -> dense_i8, in one ane::program stream."""
    rng = np.random.default_rng(77)
    HID_K, OUT_PAD, M = 128, 16, 50
    W2 = (rng.standard_normal((HID_K, OUT_PAD)) * 0.1).astype(F32)
    h = np.maximum(rng.standard_normal((64, HID_K)).astype(F32), 0)
    W2q = np.zeros(HID_K * OUT_PAD, np.int8)
    W2p = np.zeros(oracle.packed_b_size(HID_K, OUT_PAD) * 2, np.int8)
    hq = np.zeros(64 * HID_K, np.int8)
    sW = np.zeros(1, F32)
    sh = np.zeros(1, F32)
    prog = ane.Program()
    prog.emit(ane.Op.quantize_fp32_i8, ane.U32(HID_K * OUT_PAD), ane.Ptr(P(W2)), ane.Ptr(P(W2q)), ane.Ptr(P(sW)))
    prog.emit(ane.Op.pack_b_i8, ane.U32(HID_K), ane.U32(OUT_PAD), ane.Ptr(P(W2q)), ane.Ptr(P(W2p)))
    prog.emit(ane.Op.quantize_fp32_i8, ane.U32(M * HID_K), ane.Ptr(P(h)), ane.Ptr(P(hq)), ane.Ptr(P(sh)))
    prog.exec()
    qW, sWr = oracle.quantize_fp32_i8(W2)
    qh, shr = oracle.quantize_fp32_i8(h[:M])
    assert sW[0] == sWr and sh[0] == shr and np.array_equal(W2q, qW) and np.array_equal(hq[:M * HID_K], qh)
    assert np.array_equal(W2p[:oracle.packed_b_size(HID_K, OUT_PAD)], oracle.pack_b_i8(qW, HID_K, OUT_PAD))


def test_launch_counter_moves(ane):
    before = ane.launch_count()
    x = np.ones(32, F32)
    q = np.empty(32, np.int8)
    s = np.empty(1, F32)
    ane.check(ane.lib.ane_quantize_fp32_i8(32, P(x), P(q), P(s)))
    assert ane.launch_count() >= before + 2
    assert ane.lib.ane_device_timeouts() == 0


def test_threads_are_independent(ane):
    """Hogwild-style concurrent callers (test_mnist_i8.cpp:437-449): per-thread streams."""
    import threading

    rng = np.random.default_rng(8)
    cases = [(rng.standard_normal((50, 784)).astype(F32), rng.standard_normal((784, 128)).astype(F32))
             for _ in range(6)]
    outs = [np.empty((50, 128), F32) for _ in cases]
    errs = []

    def work(i):
        try:
            A, B = cases[i]
            for _ in range(5):
                ane.check(ane.lib.ane_dense_fused_i8(50, 128, 784, 1.0, 1, P(A), P(B), P(outs[i])))
        except Exception as e:  # pragma: no cover
            errs.append(e)

    ts = [threading.Thread(target=work, args=(i,)) for i in range(len(cases))]
    [t.start() for t in ts]
    [t.join() for t in ts]
    assert not errs
    for (A, B), o in zip(cases, outs):
        assert bits_equal(o, oracle.dense_fused_i8(A, B, 1.0, True))


# ------------------------------------------------------- Q8_0 x Q8_0 (mode Q)
@pytest.mark.parametrize("M,K", [(4096, 4096), (11008, 4096), (4096, 11008), (40, 256)])
def test_q8_0_gemv_q8_mode(ane, M, K):
    """Activation quantizer bytes exact; int32 block dots exact; fp32 out within
    1e-5 of the sum of |block terms| (its own fp32 order)."""
    import torch

    rng = np.random.default_rng(M * 3 + K)
    W = oracle.quantize_q8_0((rng.standard_normal((M, K)) * 0.02).astype(F32), M, K)
    x = rng.standard_normal(K).astype(F32)
    x[64:96] = 0.0  # an all-zero block (d = 0, id = 0)
    xq_ref = oracle.quantize_q8_0(x, 1, K)
    xg = torch.from_numpy(x).cuda()
    xq = ane.quantize_q8_0(xg)
    assert np.array_equal(xq.cpu().numpy(), xq_ref)
    Wg = torch.from_numpy(W).cuda()
    dots = torch.empty((M, K // 32), dtype=torch.int32, device="cuda")
    out = ane.q8_0_gemv_q8(Wg, xq, M, K, block_dots=dots)
    ref, ref_dots = oracle.q8_0_gemv_q8(W, xq_ref, M, K, with_dots=True)
    assert np.array_equal(dots.cpu().numpy(), ref_dots)
    Wb = W.reshape(M, K // 32, 34)
    dw = Wb[:, :, 0:2].copy().view(np.float16)[..., 0].astype(np.float64)
    dx = xq_ref.reshape(K // 32, 34)[:, 0:2].copy().view(np.float16)[:, 0].astype(np.float64)
    bound = np.abs(ref_dots.astype(np.float64) * dw * dx[None, :]).sum(axis=1)
    got = out.cpu().numpy().astype(np.float64)
    assert np.all(np.abs(got - ref.astype(np.float64)) <= 1e-5 * bound + 1e-30)


# ------------------------------------- back-to-back matvecs (early launch, PDL)
@pytest.mark.parametrize("static_weights", [False, True])
def test_q8_chain_reads_previous_output(ane, static_weights):
    """Each matvec reads the vector the previous kernel just wrote and writes the
    buffer the previous kernel read (ping-pong), with no host sync in between:
    the streamed kernels start early but must see x only after the previous
    kernel has finished, and must not overwrite its input while it runs."""
    import torch

    M = K = 4096
    rng = np.random.default_rng(404)
    Ws = [oracle.quantize_q8_0((rng.standard_normal((M, K)) * 0.02).astype(F32), M, K) for _ in range(2)]
    x0 = rng.standard_normal(K).astype(F32)
    Wg = [torch.from_numpy(w).cuda() for w in Ws]
    bufs = [torch.from_numpy(x0).cuda(), torch.empty(K, device="cuda")]
    steps = 6
    snaps = []
    for i in range(steps):  # mode R chain, no synchronisation inside
        ane.q8_0_gemv(Wg[i % 2], bufs[i % 2], M, K, out=bufs[(i + 1) % 2], static_weights=static_weights)
        snaps.append(bufs[(i + 1) % 2].clone())
    x = x0
    for i in range(steps):
        y = oracle.q8_0_gemv(Ws[i % 2], x, M, K)
        assert bits_equal(snaps[i].cpu().numpy(), y), f"step {i}"
        x = y
    # mode Q chain: quantize -> matvec -> quantize -> ..., again without syncs
    xg = torch.from_numpy(x0).cuda()
    outs = []
    for i in range(steps):
        xq = ane.quantize_q8_0(xg)
        xg = ane.q8_0_gemv_q8(Wg[i % 2], xq, M, K, static_weights=static_weights)
        outs.append(xg)
    x = x0
    for i in range(steps):
        xq_ref = oracle.quantize_q8_0(x, 1, K)
        ref = oracle.q8_0_gemv_q8(Ws[i % 2], xq_ref, M, K)
        got = outs[i].cpu().numpy()
        assert np.allclose(got, ref, rtol=1e-4, atol=1e-4), f"step {i}"
        x = got  # continue from the GPU's own vector so rounding differences do not compound


def test_q8_chain_in_cuda_graph(ane):
    """The same early-launching kernels captured back to back in a CUDA graph."""
    import torch

    M, K = 11008, 4096
    rng = np.random.default_rng(405)
    W = oracle.quantize_q8_0((rng.standard_normal((M, K)) * 0.02).astype(F32), M, K)
    x = rng.standard_normal(K).astype(F32)
    Wg, xg = torch.from_numpy(W).cuda(), torch.from_numpy(x).cuda()
    outs = [torch.empty(M, device="cuda") for _ in range(4)]
    ane.q8_0_gemv(Wg, xg, M, K, out=outs[0], static_weights=True)  # first call outside capture
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        for o in outs:
            ane.q8_0_gemv(Wg, xg, M, K, out=o, static_weights=True)
    for o in outs:
        o.fill_(float("nan"))
    g.replay()
    torch.cuda.synchronize()
    ref = oracle.q8_0_gemv(W, x, M, K)
    for o in outs:
        assert bits_equal(o.cpu().numpy(), ref)
    del g


# ------------------------------------- cooperative single-read quantize prologue
@pytest.mark.parametrize("M,N,K,special", [
    (2048, 2064, 2048, None),       # smallest shapes that take the cooperative prologue (all chunks resident)
    (4100, 1024, 4096, "inf"),      # ragged last chunk of A; +-inf in A (general quantize rule)
    (1024, 4096, 4112, "nan"),      # K not a multiple of 64; NaN in B
    (1024, 2064, 8192, None),       # remainder chunks of B read back from L2
    (8192, 4096, 1024, "nanA"),     # NaN in a remainder chunk of A (the last rows)
    (4096, 4096, 4096, "zeroB"),    # the benchmark shape; B all zero (absmax 0: scale 1)
])
def test_quantize_prologue_single_read(ane, M, N, K, special):
    """Aq, Bq and both scales from the one-kernel prologue, each bit-exact."""
    import torch

    rng = np.random.default_rng(M + 3 * N + 7 * K)
    A = rng.standard_normal((M, K)).astype(F32)
    B = rng.standard_normal((K, N)).astype(F32)
    A[rng.random((M, K)) < 0.001] *= 50
    if special == "inf":
        A[3, 5], A[M - 1, K - 1] = np.inf, -np.inf
    if special == "nan":
        B[K // 2, N - 3] = np.nan
    if special == "nanA":
        A[M - 1, K - 2] = np.nan
    if special == "zeroB":
        B[:] = 0.0
    Aq, Bq, scales = ane.quantize_pair(torch.from_numpy(A).cuda(), torch.from_numpy(B).cuda())
    qa, sa = oracle.quantize_fp32_i8(A)
    qb, sb = oracle.quantize_fp32_i8(B)
    s = scales.cpu().numpy()
    assert bits_equal(s, np.array([sa, sb], F32))
    assert np.array_equal(Aq.cpu().numpy(), qa.reshape(M, K))
    assert np.array_equal(Bq.cpu().numpy()[:K, :N], qb.reshape(K, N))


# ----------------------------------- ggml MUL_MAT: activation quantized in-kernel
@pytest.mark.parametrize("M,K", [(4096, 4096), (22016, 4096), (4096, 11008), (40, 256)])
def test_mul_mat_q8_0_equals_quantize_then_gemv(ane, M, K):
    """One-launch MUL_MAT (fp32 x) == quantize_q8_0 + Q8_0 x Q8_0 matvec, bit for
    bit, block dots included; the block dots also match the oracle."""
    import torch

    rng = np.random.default_rng(M + 5 * K)
    W = oracle.quantize_q8_0((rng.standard_normal((M, K)) * 0.02).astype(F32), M, K)
    x = rng.standard_normal(K).astype(F32)
    x[32:64] = 0.0         # d = 0 block
    x[96] = 3e-39          # subnormal input
    Wg, xg = torch.from_numpy(W).cuda(), torch.from_numpy(x).cuda()
    d1 = torch.empty((M, K // 32), dtype=torch.int32, device="cuda")
    d2 = torch.empty_like(d1)
    y1 = ane.mul_mat_q8_0(Wg, xg, M, K, block_dots=d1)
    y2 = ane.q8_0_gemv_q8(Wg, ane.quantize_q8_0(xg), M, K, block_dots=d2)
    assert torch.equal(d1, d2)
    assert torch.equal(y1.view(torch.int32), y2.view(torch.int32))
    _, ref_dots = oracle.q8_0_gemv_q8(W, oracle.quantize_q8_0(x, 1, K), M, K, with_dots=True)
    assert np.array_equal(d1.cpu().numpy(), ref_dots)
