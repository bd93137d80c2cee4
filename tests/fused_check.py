"""Whole-matrix parity check of one dense_fused_i8 result against the oracle.

Used by the GPU tests at the benchmarked shapes (up to 8192^3), where running
the oracle's scalar GEMM would take minutes.  The composition is checked piece
by piece instead, every piece over the whole tensor:

* the int8 codes and scale of A and of B: the oracle's quantize_fp32_i8
  (src/bytecode_interpreter.s:1876-1950) on the same fp32 inputs;
* the int32 accumulators: the oracle's codes multiplied in fp64 on the GPU,
  which is exact here (every product and partial sum is an integer below
  127^2 * K < 2^53);
* C: the oracle's dense_fused_i8 epilogue applied to those accumulators,
  compared bit for bit (and within the 1e-5 relative bar of the north star).
"""
import numpy as np

import oracle

F32 = np.float32
REL_TOL = 1e-5


def bits_equal(a, b):
    a = np.ascontiguousarray(a, F32)
    b = np.ascontiguousarray(b, F32)
    nan = np.isnan(a) | np.isnan(b)
    ok = np.array_equal(np.isnan(a), np.isnan(b)) and np.array_equal(a[~nan].view(np.uint32),
                                                                     b[~nan].view(np.uint32))
    if not ok and a.shape == b.shape:
        diff = (a.view(np.uint32) != b.view(np.uint32)) & ~(np.isnan(a) & np.isnan(b))
        print(f"bits_equal: {int(diff.sum())} of {a.size} differ; got {a[diff][:8].tolist()} "
              f"want {b[diff][:8].tolist()}")
    return ok


def exact_acc(torch, Aq, Bq, device, rows_per_chunk=2048):
    """int32 Aq[M x K] @ Bq[K x N] from int8 numpy codes, exact (fp64 on the GPU)."""
    B64 = torch.from_numpy(Bq).to(device).double()
    out = np.empty((Aq.shape[0], Bq.shape[1]), np.int32)
    for r in range(0, Aq.shape[0], rows_per_chunk):
        a = torch.from_numpy(Aq[r:r + rows_per_chunk]).to(device).double()
        out[r:r + rows_per_chunk] = (a @ B64).to(torch.int64).cpu().numpy().astype(np.int32)
        del a
    del B64
    return out


def reference_parts(torch, A, B, scale, relu):
    """Oracle codes, scales, exact accumulators and C for fp32 CUDA tensors A, B."""
    An = A.cpu().numpy()
    Bn = B.cpu().numpy()
    M, K = An.shape
    N = Bn.shape[1]
    qa, sa = oracle.quantize_fp32_i8(An)
    qb, sb = oracle.quantize_fp32_i8(Bn)
    Aq = qa.reshape(M, K)
    Bq = qb.reshape(K, N)
    acc = exact_acc(torch, Aq, Bq, A.device)
    C = oracle.dense_fused_epilogue(acc, sa, sb, scale, relu)
    return Aq, Bq, sa, sb, acc, C


def check_dense_fused(ane, torch, A, B, C, scale, relu, parts=None, check_stages=True):
    """Asserts that the GPU result C of dense_fused_i8(A, B) equals the oracle's,
    bit for bit, over the whole matrix.  With check_stages, the GPU's own
    quantized operands and raw int32 accumulators are compared as well."""
    Aq_r, Bq_r, sa, sb, acc_r, C_r = parts or reference_parts(torch, A, B, scale, relu)
    M, K = Aq_r.shape
    N = Bq_r.shape[1]
    if check_stages:
        Aq, Bq, scales = ane.quantize_pair(A, B)
        acc = ane.gemm_s8_kn(Aq, Bq, N, scales, raw_i32=True)
        torch.cuda.synchronize()
        s = scales.cpu().numpy()
        assert s[0] == sa and s[1] == sb, (s, sa, sb)
        assert np.array_equal(Aq.cpu().numpy()[:, :K], Aq_r)
        assert np.array_equal(Bq.cpu().numpy()[:K, :N], Bq_r)
        assert np.array_equal(acc.cpu().numpy(), acc_r)
        del Aq, Bq, acc
    Cn = C.cpu().numpy()
    assert bits_equal(Cn, C_r)
    ref = C_r.astype(np.float64)
    assert np.all(np.abs(Cn.astype(np.float64) - ref) <= REL_TOL * np.abs(ref))
