"""CPU oracle for the quantized dense hot path -- TEST INFRASTRUCTURE ONLY.

This package loads ``oracle/_build/libane_oracle.so`` (a plain C restatement of
the reference interpreter's opcode handlers, see ``ane_oracle.h`` for the
``bytecode_interpreter.s`` line ranges it follows) and exposes numpy wrappers.

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline leg
may import it, and only as the checker or the reported CPU baseline.  The
product package ``ane_b200`` never imports it and has no CPU fallback.
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "_build", "libane_oracle.so")
_lib = None

_f32p = np.ctypeslib.ndpointer(dtype=np.float32, flags="C_CONTIGUOUS")
_i8p = np.ctypeslib.ndpointer(dtype=np.int8, flags="C_CONTIGUOUS")
_u8p = np.ctypeslib.ndpointer(dtype=np.uint8, flags="C_CONTIGUOUS")
_i32p = np.ctypeslib.ndpointer(dtype=np.int32, flags="C_CONTIGUOUS")
_u32p = np.ctypeslib.ndpointer(dtype=np.uint32, flags="C_CONTIGUOUS")
_sz = ctypes.c_size_t
_u32 = ctypes.c_uint32
_f = ctypes.c_float
_vp = ctypes.c_void_p


def build() -> None:
    """Compile the oracle with its Makefile (gcc, -ffp-contract=off)."""
    subprocess.run(["make", "-s", "-C", _HERE], check=True)


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(_LIB_PATH):
            build()
        L = ctypes.CDLL(_LIB_PATH)
        sig = {
            "ane_ref_fp16_to_fp32": (_f, [ctypes.c_uint16]),
            "ane_ref_fp32_to_fp16": (ctypes.c_uint16, [_f]),
            "ane_ref_relu_max": (_f, [_f, _f]),
            "ane_ref_quantize_fp32_i8": (_f, [_f32p, _i8p, _sz, _vp]),
            "ane_ref_absmax": (_f, [_f32p, _sz]),
            "ane_ref_quantize_with_absmax": (_f, [_f32p, _i8p, _sz, _f]),
            "ane_ref_quantize_fp32_i8_channelwise": (None, [_u32, _u32, _f32p, _i8p, _f32p]),
            "ane_ref_dequantize_i8_fp32": (None, [_sz, _f, _i8p, _f32p]),
            "ane_ref_packed_b_size": (_sz, [_u32, _u32]),
            "ane_ref_pack_b_i8": (None, [_u32, _u32, _i8p, _i8p]),
            "ane_ref_gemm_s8_s32": (None, [_u32, _u32, _u32, _i8p, _sz, _i8p, _sz, _i32p]),
            "ane_ref_dense_i8": (None, [_u32, _u32, _u32, _f, _f, ctypes.c_uint8, _i8p, _i8p, _f32p, _f32p]),
            "ane_ref_dense_fused_i8": (None, [_u32, _u32, _u32, _f, ctypes.c_int, _f32p, _f32p, _f32p,
                                              _vp, _vp, _vp, _vp, _vp]),
            "ane_ref_dense_fused_epilogue": (None, [_u32, _u32, _i32p, _f, _f, _f, ctypes.c_int, _f32p]),
            "ane_ref_q8_0_gemv": (None, [_u32, _u32, _f32p, _u8p, _f32p]),
            "ane_ref_q4_0_gemv": (None, [_u32, _u32, _f32p, _u8p, _f32p]),
            "ane_ref_q4_k_gemv": (None, [_u32, _u32, _f32p, _u8p, _f32p]),
            "ane_ref_q2_k_gemv": (None, [_u32, _u32, _f32p, _u8p, _f32p]),
            "ane_ref_q3_k_gemv": (None, [_u32, _u32, _f32p, _u8p, _f32p]),
            "ane_ref_q5_k_gemv": (None, [_u32, _u32, _f32p, _u8p, _f32p]),
            "ane_ref_q6_k_gemv": (None, [_u32, _u32, _f32p, _u8p, _f32p]),
            "ane_ref_get_rows_q4_0": (None, [_u32, _u32, _u8p, _u32p, _f32p]),
            "ane_ref_quantize_q8_0": (None, [_f32p, _u8p, _sz, _sz]),
            "ane_ref_q8_0_gemv_q8": (None, [_u32, _u32, _u8p, _u8p, _f32p, _vp]),
            "ane_ref_get_rows_q8_0": (None, [_u32, _u32, _u8p, _u32p, _f32p]),
            "ane_ref_mul_mat_q8_0_batch": (None, [_u32, _u32, _u32, _u8p, _u8p, _f32p, _sz]),
            "ane_ref_dense_u8s8": (None, [_u32, _u32, _u32, _f, _f, ctypes.c_uint8, _u8p, _i8p, _f32p, _f32p]),
            "ane_ref_elementwise_scaled_add_fp32": (None, [_u32, _f, _f32p, _f32p, _f32p]),
            "ane_ref_relu_backward_fp32": (None, [_u32, _f32p, _f32p, _f32p]),
            "ane_ref_transpose_fp32": (None, [_u32, _u32, _f32p, _f32p]),
            "ane_ref_count_matches": (None, [_u32, _i32p, _u8p, _i32p]),
            "ane_ref_dense_fp32": (None, [_u32, _u32, _u32, _f, ctypes.c_uint8, _f32p, _f32p, _f32p, _f32p]),
            "ane_ref_softmax_argmax_fp32": (None, [_u32, _u32, _f32p, _f32p, _u8p, _f32p, _i32p]),
            "ane_ref_int_gemm": (None, [ctypes.c_int, ctypes.c_uint8, _u32, _u32, _u32, _u32, _u32, _u32, _f, _f,
                                        _u8p, _u8p, _f32p]),
            "ane_ref_dense_fused_i8_omp": (None, [_u32, _u32, _u32, _f, ctypes.c_int, _f32p, _f32p, _f32p,
                                                  ctypes.c_int]),
            "ane_ref_q8_0_gemv_omp": (None, [_u32, _u32, _f32p, _u8p, _f32p, ctypes.c_int]),
            "ane_ref_max_threads": (ctypes.c_int, []),
        }
        for name, (res, args) in sig.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


def _c(a, dtype):
    return np.ascontiguousarray(a, dtype=dtype)


def _ptr(a):
    return a.ctypes.data_as(ctypes.c_void_p)


# --------------------------------------------------------------------------- scalars
def fp16_to_fp32(h: int) -> float:
    return lib().ane_ref_fp16_to_fp32(h)


def fp32_to_fp16(f: float) -> int:
    return lib().ane_ref_fp32_to_fp16(f)


# --------------------------------------------------------------------------- quantize
def quantize_fp32_i8(x):
    x = _c(x, np.float32).ravel()
    q = np.empty(x.size, np.int8)
    s = lib().ane_ref_quantize_fp32_i8(x, q, x.size, None)
    return q, np.float32(s)


def absmax(x) -> np.float32:
    x = _c(x, np.float32).ravel()
    return np.float32(lib().ane_ref_absmax(x, x.size))


def quantize_with_absmax(x, absmax):
    """Quantize with an absmax reduced elsewhere; returns (codes, scale)."""
    x = _c(x, np.float32).ravel()
    q = np.empty(x.size, np.int8)
    s = lib().ane_ref_quantize_with_absmax(x, q, x.size, float(absmax))
    return q, np.float32(s)


def quantize_fp32_i8_channelwise(x):
    x = _c(x, np.float32)
    rows, cols = x.shape
    q = np.empty((rows, cols), np.int8)
    s = np.empty(rows, np.float32)
    lib().ane_ref_quantize_fp32_i8_channelwise(rows, cols, x, q, s)
    return q, s


def dequantize_i8_fp32(q, scale):
    q = _c(q, np.int8).ravel()
    out = np.empty(q.size, np.float32)
    lib().ane_ref_dequantize_i8_fp32(q.size, float(scale), q, out)
    return out


# --------------------------------------------------------------------------- pack / dense
def packed_b_size(K: int, N: int) -> int:
    return int(lib().ane_ref_packed_b_size(K, N))


def pack_b_i8(B, K: int, N: int):
    B = _c(B, np.int8).ravel()
    out = np.empty(packed_b_size(K, N), np.int8)
    lib().ane_ref_pack_b_i8(K, N, B, out)
    return out


def gemm_s8_s32(A, B):
    A = _c(A, np.int8)
    B = _c(B, np.int8)
    M, K = A.shape
    N = B.shape[1]
    acc = np.empty((M, N), np.int32)
    lib().ane_ref_gemm_s8_s32(M, N, K, A, K, B, N, acc)
    return acc


def dense_i8(M, N, K, sa, sb, flags, A_pad, B_packed, bias, C_rows=None):
    """dense_i8 with the reference's memory contract (A: M16 x K64, C: M16 x N)."""
    M16 = (M + 15) // 16 * 16
    C = np.zeros(M16 * N, np.float32) if C_rows is None else _c(C_rows, np.float32).ravel().copy()
    lib().ane_ref_dense_i8(M, N, K, float(sa), float(sb), int(flags), _c(A_pad, np.int8).ravel(),
                           _c(B_packed, np.int8).ravel(), _c(bias, np.float32).ravel(), C)
    return C.reshape(M16, N)


def dense_fused_i8(A, B, scale=1.0, relu=False, full=False):
    """Reference composition.  Returns C, or (C, Aq, Bq, acc, sa, sb) when full."""
    A = _c(A, np.float32)
    B = _c(B, np.float32)
    M, K = A.shape
    N = B.shape[1]
    C = np.empty((M, N), np.float32)
    if not full:
        lib().ane_ref_dense_fused_i8(M, N, K, float(scale), int(bool(relu)), A, B, C,
                                     None, None, None, None, None)
        return C
    Aq = np.empty((M, K), np.int8)
    Bq = np.empty((K, N), np.int8)
    acc = np.empty((M, N), np.int32)
    sa = np.zeros(1, np.float32)
    sb = np.zeros(1, np.float32)
    lib().ane_ref_dense_fused_i8(M, N, K, float(scale), int(bool(relu)), A, B, C,
                                 _ptr(Aq), _ptr(Bq), _ptr(acc), _ptr(sa), _ptr(sb))
    return C, Aq, Bq, acc, sa[0], sb[0]


def dense_fused_epilogue(acc, sa, sb, scale, relu):
    acc = _c(acc, np.int32)
    M, N = acc.shape
    C = np.empty((M, N), np.float32)
    lib().ane_ref_dense_fused_epilogue(M, N, acc, float(sa), float(sb), float(scale), int(bool(relu)), C)
    return C


def dense_fused_i8_omp(A, B, scale=1.0, relu=False, threads=0):
    A = _c(A, np.float32)
    B = _c(B, np.float32)
    M, K = A.shape
    N = B.shape[1]
    C = np.empty((M, N), np.float32)
    lib().ane_ref_dense_fused_i8_omp(M, N, K, float(scale), int(bool(relu)), A, B, C, int(threads))
    return C


# --------------------------------------------------------------------------- Q8_0
def q8_0_gemv(W_blocks, x, M: int, K: int):
    out = np.empty(M, np.float32)
    lib().ane_ref_q8_0_gemv(M, K, _c(x, np.float32).ravel(), _c(W_blocks, np.uint8).ravel(), out)
    return out


def q4_0_gemv(W_blocks, x, M: int, K: int):
    out = np.empty(M, np.float32)
    lib().ane_ref_q4_0_gemv(M, K, _c(x, np.float32).ravel(), _c(W_blocks, np.uint8).ravel(), out)
    return out


# K-quant super-block sizes (bytes per 256 weights), by format name
KQUANT_BLOCK_BYTES = {"q2_k": 84, "q3_k": 110, "q4_k": 144, "q5_k": 176, "q6_k": 210}


def kquant_gemv(fmt: str, W_blocks, x, M: int, K: int):
    """out[M] = K-quant matrix W (M rows of K/256 super-blocks) times fp32 x[K],
    the reference handler's arithmetic (fmt in KQUANT_BLOCK_BYTES)."""
    out = np.empty(M, np.float32)
    getattr(lib(), "ane_ref_%s_gemv" % fmt)(M, K, _c(x, np.float32).ravel(), _c(W_blocks, np.uint8).ravel(), out)
    return out


def q8_0_gemv_omp(W_blocks, x, M: int, K: int, threads=0):
    out = np.empty(M, np.float32)
    lib().ane_ref_q8_0_gemv_omp(M, K, _c(x, np.float32).ravel(), _c(W_blocks, np.uint8).ravel(), out,
                                int(threads))
    return out


def quantize_q8_0(x, n_rows: int, K: int):
    out = np.empty(n_rows * (K // 32) * 34, np.uint8)
    lib().ane_ref_quantize_q8_0(_c(x, np.float32).ravel(), out, n_rows, K)
    return out


def q8_0_gemv_q8(W_blocks, xq_blocks, M: int, K: int, with_dots=False):
    out = np.empty(M, np.float32)
    dots = np.empty(M * (K // 32), np.int32) if with_dots else None
    lib().ane_ref_q8_0_gemv_q8(M, K, _c(xq_blocks, np.uint8).ravel(), _c(W_blocks, np.uint8).ravel(), out,
                               _ptr(dots) if with_dots else None)
    return (out, dots.reshape(M, K // 32)) if with_dots else out


def dense_u8s8(M, N, K, sa, sb, flags, A_pad, B_packed, bias, C_rows=None):
    """Reference dense_u8s8 on padded buffers: A uint8 [M16 x K64], B packed (pack_b_i8
    with K64), bias [>= N]; returns C [M16 x N] (padded rows included)."""
    M16 = (M + 15) // 16 * 16
    C = np.empty(M16 * N, np.float32)
    lib().ane_ref_dense_u8s8(M, N, K, sa, sb, flags, _c(A_pad, np.uint8).ravel(), _c(B_packed, np.int8).ravel(),
                             _c(bias, np.float32).ravel(), C)
    return C.reshape(M16, N)


INT_GEMM_KINDS = {"igemm": 0, "ugemm": 1, "usgemm": 2}


def int_gemm(kind, flags, M, N, K, lda, ldb, ldc, alpha, beta, A_bytes, B_bytes, C):
    """Reference integer CBLAS GEMM; C (float32, >= (M-1)*ldc+N) is updated in place."""
    assert C.dtype == np.float32 and C.flags["C_CONTIGUOUS"]
    lib().ane_ref_int_gemm(INT_GEMM_KINDS[kind], flags, M, N, K, lda, ldb, ldc, alpha, beta,
                           _c(A_bytes, np.uint8).ravel(), _c(B_bytes, np.uint8).ravel(), C.ravel())
    return C


def elementwise_scaled_add_fp32(scale, a, b):
    a, b = _c(a, np.float32).ravel(), _c(b, np.float32).ravel()
    out = np.empty_like(a)
    lib().ane_ref_elementwise_scaled_add_fp32(a.size, scale, a, b, out)
    return out


def relu_backward_fp32(act, grad):
    act, grad = _c(act, np.float32).ravel(), _c(grad, np.float32).ravel()
    out = np.empty_like(act)
    lib().ane_ref_relu_backward_fp32(act.size, act, grad, out)
    return out


def transpose_fp32(src):
    src = _c(src, np.float32)
    M, N = src.shape
    dst = np.empty((N, M), np.float32)
    lib().ane_ref_transpose_fp32(M, N, src.ravel(), dst.ravel())
    return dst


def count_matches(pred, labels):
    out = np.zeros(1, np.int32)
    pred, labels = _c(pred, np.int32).ravel(), _c(labels, np.uint8).ravel()
    lib().ane_ref_count_matches(pred.size, pred, labels, out)
    return int(out[0])


def dense_fp32(M, N, K, scale, flags, A_pad, B, bias):
    """A [M16 x K], B [K x N], bias [>= N]: C [M16 x N] (padded rows included)."""
    M16 = (M + 15) // 16 * 16
    C = np.empty((M16, N), np.float32)
    lib().ane_ref_dense_fp32(M, N, K, scale, flags, _c(A_pad, np.float32).ravel(), _c(B, np.float32).ravel(),
                             _c(bias, np.float32).ravel(), C.ravel())
    return C


def softmax_argmax_fp32(logits, labels, g_out=None):
    """logits [batch x cols]; returns probs, g_out (only its first 16 columns are
    written: pass the previous contents), argmax."""
    logits = _c(logits, np.float32)
    batch, cols = logits.shape
    probs = np.empty_like(logits)
    g = np.zeros_like(logits) if g_out is None else np.array(g_out, np.float32, copy=True)
    am = np.empty(batch, np.int32)
    lib().ane_ref_softmax_argmax_fp32(batch, cols, logits.ravel(), probs.ravel(), _c(labels, np.uint8).ravel(),
                                      g.ravel(), am)
    return probs, g, am


def mul_mat_q8_0_batch(W_blocks, xq_blocks, M: int, K: int, NT: int):
    """[NT, M] fp32: Q8_0 weights against NT Q8_0 activation rows, segment order."""
    out = np.empty((NT, M), np.float32)
    lib().ane_ref_mul_mat_q8_0_batch(M, K, NT, _c(xq_blocks, np.uint8).ravel(), _c(W_blocks, np.uint8).ravel(),
                                     out, M)
    return out


def get_rows_q8_0(table, indices, dim: int):
    idx = _c(indices, np.uint32).ravel()
    out = np.empty(idx.size * dim, np.float32)
    lib().ane_ref_get_rows_q8_0(idx.size, dim, _c(table, np.uint8).ravel(), idx, out)
    return out.reshape(idx.size, dim)


def get_rows_q4_0(table, indices, dim: int):
    idx = _c(indices, np.uint32).ravel()
    out = np.empty(idx.size * dim, np.float32)
    lib().ane_ref_get_rows_q4_0(idx.size, dim, _c(table, np.uint8).ravel(), idx, out)
    return out.reshape(idx.size, dim)


def max_threads() -> int:
    return int(lib().ane_ref_max_threads())
